"""Attention dropout on alpha (multiscreen/attention.py:68,190) on the CUDA
path.  The mask comes from a counter-based hash of (seed, b*H+h, i, j) that
the backward regenerates; the oracle restates the same hash, so the CUDA
output and all gradients are compared with the oracle under the identical
mask, within the parity tolerances (max |x - ref| / max |ref| <= 1e-4 for
float32 I/O, <= 2e-2 for bfloat16 I/O)."""
import math

import pytest
import torch

from tests.conftest import rel_err
from tests.test_parity_gpu import make_case

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
CASES = [
    # B, Tq, Tk, H, D, causal, q_offset, w list, r list, kpm, corr
    (2, 129, 129, 2, 64, True, 0, [5.5, 1000.0], [1.2, 1.7], True, 0.5),
    (1, 300, 300, 3, 64, True, 0, [0.7, 64.0, 129.0], [1.5, 1.001, 1.3], False, 0.4),
    (1, 257, 257, 2, 64, False, 0, [17.0, 300.0], [1.2, 1.05], True, 0.5),
    (1, 100, 612, 2, 64, True, 512, [64.0, 600.0], [1.2, 1.05], False, 0.0),
    (1, 200, 200, 2, 32, True, 0, [20.0, 150.0], [1.2, 1.05], False, 0.4),
]
NAMES = ("y", "dq", "dk", "dv", "ds_r", "ds_v")


def _run_cuda(ms, q, k, v, s_r, s_v, causal, kpm, cot, dtype, q_offset, p, seed):
    dev = torch.device("cuda:0")
    qc = q.to(dev, dtype).requires_grad_(True)
    kc = k.to(dev, dtype).requires_grad_(True)
    vc = v.to(dev, dtype).requires_grad_(True)
    sr = s_r.to(dev).requires_grad_(True)
    sv = s_v.to(dev).requires_grad_(True)
    y = ms.screening_attention(qc, kc, vc, torch.exp(sr) + 1.0, torch.exp(sv) + 1.0, causal,
                               None if kpm is None else kpm.to(dev), 1e-8, q_offset,
                               dropout_p=p, dropout_seed=seed)
    (y.float() * cot.to(dev).view_as(y)).sum().backward()
    return [t.detach().float().cpu() for t in (y, qc.grad, kc.grad, vc.grad, sr.grad, sv.grad)]


def _run_oracle(oracle, q, k, v, s_r, s_v, causal, kpm, cot, q_offset, dropout):
    q = q.double().requires_grad_(True)
    k = k.double().requires_grad_(True)
    v = v.double().requires_grad_(True)
    sr = s_r.double().requires_grad_(True)
    sv = s_v.double().requires_grad_(True)
    y = oracle.screening_core_windowed(q, k, v, torch.exp(sr) + 1.0, torch.exp(sv) + 1.0, causal,
                                       kpm, 1e-8, q_offset, chunk=128, dropout=dropout)
    (y * cot.double().view_as(y)).sum().backward()
    return [t.detach() for t in (y, q.grad, k.grad, v.grad, sr.grad, sv.grad)]


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_dropout_parity_same_mask(ms, oracle, ci, dtype, deterministic):
    B, Tq, Tk, H, D, causal, qo, ws, rs, kpm, corr = CASES[ci]
    q, k, v, s_r, s_v, mask, cot = make_case(*CASES[ci], seed=300 + ci)
    if dtype == torch.bfloat16:
        q, k, v = q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float()
    p, seed = 0.2, 0xC0FFEE + ci
    from importlib import import_module
    lib = import_module("pytorch-implementation-of-screening-attention_b200._lib")
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(deterministic)
    try:
        got = _run_cuda(ms, q, k, v, s_r, s_v, causal, mask, cot, dtype, qo, p, seed)
    finally:
        torch.use_deterministic_algorithms(prev)
    ref = _run_oracle(oracle, q, k, v, s_r, s_v, causal, mask, cot, qo,
                      (lib.dropout_threshold(p), seed))
    errs = {n: rel_err(a, b.reshape(a.shape)) for n, a, b in zip(NAMES, got, ref)}
    bad = {n: e for n, e in errs.items() if not e <= TOL[dtype]}
    assert not bad, f"case {ci} {dtype}: " + ", ".join(f"{n}={e:.2e}" for n, e in errs.items())
    # the mask changed the result: without dropout the output differs
    ref0 = _run_oracle(oracle, q, k, v, s_r, s_v, causal, mask, cot, qo, None)
    assert rel_err(ref[0], ref0[0]) > 10 * TOL[dtype]


def test_module_dropout_training(ms, cuda):
    """ScreeningAttention(dropout=p) in training mode: reproducible under
    torch.manual_seed, different across seeds, finite gradients for every
    parameter; eval mode equals p = 0."""
    torch.manual_seed(0)
    a = ms.ScreeningAttention(256, 4, dropout=0.3)
    with torch.no_grad():
        # r = 1.05, w = 256: about a fifth of the scores of random projections
        # clear the trim threshold (with the default r = 2 almost none do)
        a.s_r.fill_(math.log(0.05))
        a.s_v.fill_(math.log(255.0))
    a = a.to(cuda).to(torch.bfloat16)
    x = torch.randn(2, 384, 256, device=cuda).to(torch.bfloat16)

    def run(seed):
        torch.manual_seed(seed)
        for prm in a.parameters():
            prm.grad = None
        y = a(x, x, x)
        y.float().pow(2).sum().backward()
        return y.detach().float(), [prm.grad.detach().float().clone() for prm in a.parameters()]

    a.train()
    y1, g1 = run(11)
    y2, g2 = run(11)
    y3, _ = run(12)
    assert torch.equal(y1, y2)
    assert all(torch.equal(u, v) for u, v in zip(g1, g2))
    assert not torch.equal(y1, y3)
    assert all(torch.isfinite(g).all() for g in g1)
    assert y1.abs().max() > 0
    a.eval()
    with torch.no_grad():
        ye = a(x, x, x).float()
        a.attn_dropout.p = 0.0
        a.train()
        y0 = a(x, x, x).float()
    assert torch.equal(ye, y0)
    assert not torch.equal(y1, ye)
