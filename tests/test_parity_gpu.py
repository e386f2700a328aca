"""CUDA path vs the reference's numbers and the CPU oracle.

Tolerances (from the parity contract): max |x - ref| / max |ref| <= 1e-4 for
float32 I/O, <= 2e-2 for bfloat16 I/O (fp32 accumulation), on the output and
on every gradient (q, k, v, r, w).
"""
import math

import pytest
import torch

from tests.conftest import rel_err
from tests.helpers import golden_module

MG = golden_module()
pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def run_cuda(ms, q, k, v, s_r, s_v, causal, kpm, cot, dtype, q_offset=0):
    dev = torch.device("cuda:0")
    qc = q.to(dev, dtype).requires_grad_(True)
    kc = k.to(dev, dtype).requires_grad_(True)
    vc = v.to(dev, dtype).requires_grad_(True)
    sr = s_r.to(dev).requires_grad_(True)
    sv = s_v.to(dev).requires_grad_(True)
    r = torch.exp(sr) + 1.0
    w = torch.exp(sv) + 1.0
    y = ms.screening_attention(qc, kc, vc, r, w, causal,
                               None if kpm is None else kpm.to(dev), 1e-8, q_offset)
    (y.float() * cot.to(dev).view_as(y)).sum().backward()
    return [t.detach().float().cpu() for t in (y, qc.grad, kc.grad, vc.grad, sr.grad, sv.grad)]


def run_oracle(oracle, q, k, v, s_r, s_v, causal, kpm, cot, q_offset=0):
    q = q.double().requires_grad_(True)
    k = k.double().requires_grad_(True)
    v = v.double().requires_grad_(True)
    sr = s_r.double().requires_grad_(True)
    sv = s_v.double().requires_grad_(True)
    y = oracle.screening_core_windowed(q, k, v, torch.exp(sr) + 1.0, torch.exp(sv) + 1.0,
                                       causal, kpm, 1e-8, q_offset, chunk=128)
    (y * cot.double().view_as(y)).sum().backward()
    return [t.detach() for t in (y, q.grad, k.grad, v.grad, sr.grad, sv.grad)]


def assert_all_close(got, ref, tol, what=""):
    names = ("y", "dq", "dk", "dv", "ds_r", "ds_v")
    errs = {n: rel_err(a, b.reshape(a.shape)) for n, a, b in zip(names, got, ref)}
    bad = {n: e for n, e in errs.items() if not e <= tol}
    assert not bad, f"{what}: rel errs " + ", ".join(f"{n}={e:.2e}" for n, e in errs.items())


# ---------------------------------------------------------------------------
# 1. the reference's own numbers (golden), fp32
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(MG.ATTN_CASES))
def test_golden_fp32(ms, golden, name):
    rec = golden["attention"][name]
    spec = rec["spec"]
    inp = MG.case_inputs(spec)
    B, Tq, Tk, H, D = spec["B"], spec["Tq"], spec["Tk"], spec["H"], spec["D"]
    got = run_cuda(ms, inp["q"].view(B, Tq, H, D), inp["k"].view(B, Tk, H, D),
                   inp["v"].view(B, Tk, H, D), inp["s_r"], inp["s_v"], spec["causal"],
                   inp["kpm"], inp["cot"], torch.float32)
    ref = [rec["y"], rec["dq"], rec["dk"], rec["dv"], rec["ds_r"], rec["ds_v"]]
    assert_all_close(got, ref, 1e-4, name)


# ---------------------------------------------------------------------------
# 2. same cases in bf16 against the oracle on the bf16-rounded inputs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(MG.ATTN_CASES))
def test_golden_cases_bf16(ms, oracle, name):
    spec = MG.ATTN_CASES[name]
    inp = MG.case_inputs(spec)
    B, Tq, Tk, H, D = spec["B"], spec["Tq"], spec["Tk"], spec["H"], spec["D"]
    q = inp["q"].view(B, Tq, H, D).bfloat16().float()
    k = inp["k"].view(B, Tk, H, D).bfloat16().float()
    v = inp["v"].view(B, Tk, H, D).bfloat16().float()
    got = run_cuda(ms, q, k, v, inp["s_r"], inp["s_v"], spec["causal"], inp["kpm"], inp["cot"],
                   torch.bfloat16)
    ref = run_oracle(oracle, q, k, v, inp["s_r"], inp["s_v"], spec["causal"], inp["kpm"],
                     inp["cot"])
    assert_all_close(got, ref, 2e-2, name)


# ---------------------------------------------------------------------------
# 3. seeded random shapes (ragged T, cross-attention, offsets, masks, windows)
# ---------------------------------------------------------------------------
CASES = [
    # B, Tq, Tk, H, D, causal, q_offset, w list, r list, kpm, corr
    (1, 1, 1, 2, 64, True, 0, [3.0, 100.0], [1.5, 1.1], False, 0.5),
    (2, 63, 63, 2, 64, True, 0, [10.0, 70.0], [1.3, 1.05], False, 0.5),
    (1, 65, 65, 1, 64, True, 0, [200.0], [1.02], False, 0.2),
    (2, 129, 129, 2, 64, True, 0, [5.5, 1000.0], [1.2, 1.7], True, 0.5),
    (1, 300, 300, 3, 64, True, 0, [0.7, 64.0, 129.0], [1.5, 1.001, 1.3], False, 0.4),
    (1, 257, 257, 2, 64, False, 0, [17.0, 300.0], [1.2, 1.05], True, 0.5),
    (2, 40, 170, 2, 64, False, 0, [30.0, 90.0], [1.1, 1.4], True, 0.0),
    (1, 100, 612, 2, 64, True, 512, [64.0, 600.0], [1.2, 1.05], False, 0.0),
    (1, 520, 520, 2, 128, True, 0, [50.0, 500.0], [1.2, 1.05], False, 0.4),
    (1, 333, 333, 2, 32, True, 0, [50.0, 500.0], [1.2, 1.05], True, 0.4),
    (1, 200, 200, 2, 16, False, 0, [20.0, 150.0], [1.2, 1.05], False, 0.4),
    # head dim 128: tensor-core forward (two 64-column operand halves), SIMT backward
    (2, 200, 333, 2, 128, False, 0, [40.0, 300.0], [1.1, 1.3], True, 0.0),
    (1, 150, 700, 2, 128, True, 550, [64.0, 700.0], [1.2, 1.05], False, 0.0),
    (1, 1100, 1100, 3, 128, True, 0, [9.5, 333.0, 1100.0], [1.5, 1.02, 1.3], True, 0.4),
]


def make_case(B, Tq, Tk, H, D, causal, q_offset, ws, rs, kpm, corr, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Tq, H, D, generator=g) * 3.0
    k = torch.randn(B, Tk, H, D, generator=g)
    v = torch.randn(B, Tk, H, D, generator=g) * 0.5
    if corr:
        n = min(Tq, Tk - q_offset)
        k[:, q_offset:q_offset + n] = q[:, :n] + corr * k[:, q_offset:q_offset + n]
    s_v = torch.log(torch.tensor(ws) - 1.0) if min(ws) > 1 else torch.tensor(
        [math.log(max(x - 1.0, 1e-6)) for x in ws])
    s_r = torch.log(torch.tensor(rs) - 1.0)
    mask = None
    if kpm:
        mask = torch.rand(B, Tk, generator=g) < 0.2
    cot = torch.randn(B, Tq, H * D, generator=g)
    return q, k, v, s_r, s_v, mask, cot


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_random_cases(ms, oracle, ci, dtype):
    B, Tq, Tk, H, D, causal, qo, ws, rs, kpm, corr = CASES[ci]
    q, k, v, s_r, s_v, mask, cot = make_case(*CASES[ci], seed=100 + ci)
    if dtype == torch.bfloat16:
        q, k, v = q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float()
    got = run_cuda(ms, q, k, v, s_r, s_v, causal, mask, cot, dtype, qo)
    ref = run_oracle(oracle, q, k, v, s_r, s_v, causal, mask, cot, qo)
    assert_all_close(got, ref, TOL[dtype], f"case {ci} {dtype}")


# ---------------------------------------------------------------------------
# 4. large T, bf16 tensor-core path: parity on a strip + invariants
# ---------------------------------------------------------------------------
def test_t4096_bf16_against_oracle(ms, oracle):
    B, T, H, D = 1, 4096, 2, 64
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, T, H, D, generator=g)
    k = q + 0.7 * torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    q, k, v = q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float()
    s_r = torch.log(torch.tensor([0.3, 0.05]))
    s_v = torch.log(torch.tensor([300.0, 3000.0]))
    cot = torch.randn(B, T, H * D, generator=g)
    got = run_cuda(ms, q, k, v, s_r, s_v, True, None, cot, torch.bfloat16)
    ref = run_oracle(oracle, q, k, v, s_r, s_v, True, None, cot)
    assert_all_close(got, ref, 2e-2, "T=4096")


@pytest.mark.parametrize("D", [64, 128])
def test_backward_is_deterministic(ms, D):
    """With torch.use_deterministic_algorithms(True) the backward takes the
    fixed-order path (dq by its own kernel): bitwise reproducible.  At
    D = 128 that is the only tensor-core backward, deterministic or not."""
    prev = torch.are_deterministic_algorithms_enabled()
    if D == 64:
        torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        _backward_twice_equal(ms, D)
    finally:
        torch.use_deterministic_algorithms(prev)


def test_fused_dq_backward_matches_fixed_order(ms):
    """Default path (dq formed inside the dk/dv kernel, fp32 reductions) ==
    the fixed-order path within the bf16 contract; dk, dv, dr, dw identical
    in value up to summation order."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(13)
    B, T, H, D = 2, 1100, 3, 64
    q = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()
    k = (q.float() + 0.5 * torch.randn(B, T, H, D, device=dev, generator=g)).bfloat16()
    v = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()
    r = torch.tensor([1.2, 1.05, 1.6], device=dev)
    w = torch.tensor([70.0, 300.0, 1500.0], device=dev)
    dy = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()

    def run():
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        rr, ww = r.clone().requires_grad_(True), w.clone().requires_grad_(True)
        y = ms.screening_attention(qq, kk, vv, rr, ww, True)
        y.backward(dy)
        return [qq.grad, kk.grad, vv.grad, rr.grad, ww.grad]

    fused = run()
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        fixed = run()
    finally:
        torch.use_deterministic_algorithms(prev)
    for name, a, b in zip(("dq", "dk", "dv", "dr", "dw"), fused, fixed):
        assert rel_err(a, b) <= 1e-2, name
    assert ms._lib.device_status() == 0


def _backward_twice_equal(ms, D=64):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    B, T, H = 2, 1000, 4
    q = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()
    k = (q.float() + 0.5 * torch.randn(B, T, H, D, device=dev, generator=g)).bfloat16()
    v = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()
    r = torch.full((H,), 1.2, device=dev)
    w = torch.tensor([20.0, 100.0, 400.0, 2000.0], device=dev)
    dy = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()
    outs = []
    for _ in range(2):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        rr, ww = r.clone().requires_grad_(True), w.clone().requires_grad_(True)
        y = ms.screening_attention(qq, kk, vv, rr, ww, True)
        y.backward(dy)
        outs.append([y, qq.grad, kk.grad, vv.grad, rr.grad, ww.grad])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_causal_invariance_long(ms):
    """Perturbing the future never changes the past (attention.py:117)."""
    dev = torch.device("cuda:0")
    B, T, H, D = 1, 700, 2, 64
    x = torch.randn(B, T, H, D, device=dev).bfloat16()
    x2 = x.clone()
    x2[:, 500:] = torch.randn_like(x2[:, 500:])
    r = torch.tensor([1.05, 1.3], device=dev)
    w = torch.tensor([40.0, 5000.0], device=dev)
    y1 = ms.screening_attention(x, x, x, r, w, True)
    y2 = ms.screening_attention(x2, x2, x2, r, w, True)
    assert torch.equal(y1[:, :500], y2[:, :500])


def test_empty_and_masked_everything(ms):
    dev = torch.device("cuda:0")
    B, T, H, D = 2, 50, 2, 64
    x = torch.randn(B, T, H, D, device=dev).bfloat16().requires_grad_(True)
    r = torch.tensor([1.1, 1.2], device=dev)
    w = torch.tensor([10.0, 20.0], device=dev)
    mask = torch.ones(B, T, dtype=torch.bool, device=dev)
    y = ms.screening_attention(x, x, x, r, w, True, mask)
    assert torch.count_nonzero(y) == 0
    y.float().sum().backward()
    assert torch.isfinite(x.grad.float()).all()
    # zero-length key axis
    q = torch.randn(1, 5, H, D, device=dev)
    kv = torch.randn(1, 0, H, D, device=dev)
    y = ms.screening_attention(q, kv, kv, r, w, False)
    assert y.shape == (1, 5, H, D) and torch.count_nonzero(y) == 0


def test_head_dim_128_forward_runs_on_tensor_cores(ms):
    """bf16 D = 128 takes the tcgen05 forward (it reports tile statistics,
    which only the tensor-core kernel counts)."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v = (torch.randn(1, 300, 2, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    r = torch.tensor([1.2, 1.5], device=dev)
    w = torch.tensor([50.0, 200.0], device=dev)
    stats = torch.zeros(2, dtype=torch.int64, device=dev)
    ms._lib.screen_fwd(q, k, v, r, w, True, tile_stats=stats)
    torch.cuda.synchronize()
    assert int(stats[0]) > 0


def test_head_dim_128_core_long(ms, oracle):
    """D = 128 forward and backward on the tensor cores at T = 2048 with
    windows from 40 to 2000, against the fp64 chunked oracle, bf16 contract."""
    g = torch.Generator().manual_seed(128)
    B, T, H, D = 1, 2048, 4, 128
    q = torch.randn(B, T, H, D, generator=g)
    k = 0.6 * q + torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    q, k, v = (t.bfloat16().float() for t in (q, k, v))
    r = torch.tensor([1.02, 1.3, 1.8, 1.1])
    w = torch.tensor([40.0, 300.0, 2000.0, 900.5])
    dy = torch.randn(B, T, H, D, generator=g)
    dev = torch.device("cuda:0")
    qc, kc, vc = (t.to(dev, torch.bfloat16).requires_grad_(True) for t in (q, k, v))
    rc, wc = r.to(dev).requires_grad_(True), w.to(dev).requires_grad_(True)
    y = ms.screening_attention(qc, kc, vc, rc, wc, True)
    y.backward(dy.to(dev, torch.bfloat16))
    ref = oracle.windowed_core_grads(q, k, v, r, w, dy.bfloat16().float(), True)
    got = [t.detach().float().cpu() for t in (y, qc.grad, kc.grad, vc.grad, rc.grad, wc.grad)]
    for name, a, b in zip(("y", "dq", "dk", "dv", "dr", "dw"), got, ref):
        assert rel_err(a, b) <= 2e-2, name
    assert ms._lib.device_status() == 0
