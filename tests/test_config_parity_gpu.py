"""Parity at the benchmark configurations' own sizes and input
distributions, against the fp64 windowed oracle (restating
multiscreen/attention.py:156-196 and multiscreen/model.py:71-141).

  cfg3  ScreeningAttention(1024, 16), all 16 heads, r ~ U[1,2],
        w ~ U[256,4096] (the bench's draws), bf16, T = 4096: module output,
        input and projection-weight gradients, d s_r, d s_v
  cfg4  T = 131072, w = 2048, 16 heads: the first and last 4096 rows
  cfg5  decode of the newest token after a 100K-token prefix through the
        paged ring cache, at the default w = 2..256 and at w = 4096
  cfg2  one bf16-autocast training step of MultiscreenLM(50257, 256, 4, 4),
        B = 16, T = 512: loss and the s_r / s_v / embedding gradients

Tolerance: max |cuda - oracle| / max |oracle| <= 2e-2 for bf16 I/O (fp32
accumulation), the contract the kernels are held to; the oracle runs in fp64
on the same bf16-rounded inputs and weights.
"""
import math

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = 2e-2


def _cfg3_heads(seed=0, H=16):
    # the bench's per-head draws: r ~ U[1, 2], w ~ U[256, 4096]
    g = torch.Generator().manual_seed(seed)
    r = 1.0 + torch.rand(H, generator=g)
    w = 256.0 + (4096.0 - 256.0) * torch.rand(H, generator=g)
    return r, w


def _low_rank(shape, basis, gen):
    """Rows in the subspace spanned by `basis` (rank x D): with queries and
    keys in one low-rank subspace the cosine similarities spread ~
    1/sqrt(rank), so a useful share of the scores clears the trim threshold
    at r = 2 (random 64-d rows would be trimmed almost everywhere)."""
    *lead, D = shape
    return torch.randn(*lead, basis.shape[0], generator=gen) @ basis


def test_cfg3_module_all_heads_full_size(ms, oracle):
    torch.manual_seed(0)
    H, d, T = 16, 1024, 4096
    attn = ms.ScreeningAttention(d, H)
    r_h, w_h = _cfg3_heads()
    with torch.no_grad():
        attn.s_r.copy_(torch.log((r_h - 1.0).clamp_min(1e-6)))
        attn.s_v.copy_(torch.log(w_h - 1.0))
    attn = attn.to(DEV).to(torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, T, d, generator=g).to(torch.bfloat16)
    cot = torch.randn(1, T, d, generator=g).to(torch.bfloat16)
    xr = x.to(DEV).requires_grad_(True)
    y = attn(xr, xr, xr)
    y.backward(cot.to(DEV))
    torch.cuda.synchronize()
    assert ms._lib.device_status() == 0

    # fp64 oracle on the same bf16 weights / inputs
    Wq, Wk, Wv, Wo = (getattr(attn, n).weight.detach().double().cpu()
                      for n in ("q_proj", "k_proj", "v_proj", "out_proj"))
    s_r = attn.s_r.detach().double().cpu()
    s_v = attn.s_v.detach().double().cpu()
    r, w = torch.exp(s_r) + 1.0, torch.exp(s_v) + 1.0
    xd, cd = x.double(), cot.double()
    q, k, v = ((xd @ W.T).view(1, T, H, 64) for W in (Wq, Wk, Wv))
    dcore = (cd @ Wo).view(1, T, H, 64)
    yc, dq, dk, dv, dr, dw = oracle.windowed_core_grads(q, k, v, r, w, dcore, chunk=256)
    ycf = yc.reshape(1, T, d)
    y_ref = ycf @ Wo.T
    dq2, dk2, dv2 = (t.reshape(T, d) for t in (dq, dk, dv))
    x2 = xd.reshape(T, d)
    dx_ref = dq2 @ Wq + dk2 @ Wk + dv2 @ Wv
    assert rel_err(y, y_ref) <= TOL
    assert rel_err(xr.grad[0], dx_ref) <= TOL
    assert rel_err(attn.out_proj.weight.grad, cd.reshape(T, d).T @ ycf.reshape(T, d)) <= TOL
    for name, dt in (("q_proj", dq2), ("k_proj", dk2), ("v_proj", dv2)):
        assert rel_err(getattr(attn, name).weight.grad, dt.T @ x2) <= TOL, name
    assert rel_err(attn.s_r.grad, dr * (r - 1.0)) <= TOL
    assert rel_err(attn.s_v.grad, dw * (w - 1.0)) <= TOL


def test_cfg4_long_context_first_and_last_rows(ms, oracle):
    T, H, D, win = 131072, 16, 64, 2048.0
    g = torch.Generator().manual_seed(4)
    basis = torch.randn(4, D, generator=g)
    q = _low_rank((1, T, H, D), basis, g).to(torch.bfloat16)
    k = _low_rank((1, T, H, D), basis, g).to(torch.bfloat16)
    v = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    r = torch.full((H,), 2.0)          # s_r = 0 at init
    w = torch.full((H,), win)
    with torch.no_grad():
        y = ms.screening_attention(q.to(DEV), k.to(DEV), v.to(DEV), r.to(DEV), w.to(DEV), True)
    torch.cuda.synchronize()
    assert ms._lib.device_status() == 0
    n, dmax = 4096, int(math.ceil(win)) - 1
    head = oracle.screening_core_windowed(q[:, :n].double(), k[:, :n].double(),
                                          v[:, :n].double(), r.double(), w.double(), True)
    lo = T - n - dmax
    tail = oracle.screening_core_windowed(q[:, T - n:].double(), k[:, lo:].double(),
                                          v[:, lo:].double(), r.double(), w.double(), True,
                                          q_offset=T - n - lo)
    assert rel_err(y[:, :n], head) <= TOL
    assert rel_err(y[:, T - n:], tail) <= TOL
    # a meaningful share of rows sees live (untrimmed) keys
    assert (head.abs().amax(-1) > 0).float().mean() > 0.5


@pytest.mark.parametrize("widen", [False, True])
def test_cfg5_decode_after_100k_prefix(ms, oracle, widen):
    B, H, D, T = 4, 16, 64, 100_001          # 100K-token prompt + the new token
    if widen:
        w = torch.full((H,), 4096.0)
    else:
        w = torch.exp(torch.linspace(0, math.log(255), H)) + 1.0   # w = 2..256 at init
    r = torch.full((H,), 2.0)
    g = torch.Generator().manual_seed(5 + int(widen))
    basis = torch.randn(4, D, generator=g)
    k = _low_rank((B, T, H, D), basis, g).to(torch.bfloat16)
    v = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16)
    q = _low_rank((B, H, D), basis, g).to(torch.bfloat16)
    cache = ms.PagedKVCache(1, B, H, D, max_len=T, max_window=float(w.max()),
                            dtype=torch.bfloat16, device=DEV, page_size=64)
    # fill the ring the way a long prefill followed by decode steps does:
    # chunks of at most `keep` tokens, wrapping the ring many times
    kd, vd = k.to(DEV), v.to(DEV)
    step = cache.keep
    for t0 in range(0, T, step):
        t1 = min(T, t0 + step)
        cache.append(0, kd[:, t0:t1], vd[:, t0:t1],
                     torch.full((B,), t0, dtype=torch.int32, device=DEV))
    y, _ = cache.decode(0, q.to(DEV), torch.full((B,), T, dtype=torch.int32, device=DEV),
                        r.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert ms._lib.device_status() == 0
    dmax = int(math.ceil(float(w.max()))) - 1
    lo = T - 1 - dmax
    ref = oracle.screening_core_windowed(q.unsqueeze(1).double(), k[:, lo:].double(),
                                         v[:, lo:].double(), r.double(), w.double(), True,
                                         q_offset=dmax)[:, 0]
    assert rel_err(y, ref) <= TOL
    assert (ref.abs().amax(-1) > 0).float().mean() > 0.5


def test_cfg2_bf16_training_step_vs_oracle(ms, oracle):
    """Loss and embedding gradients at 2e-2.  The s_r / s_v gradients at
    random init are sums of ~1e-6 that largely cancel, so bf16 autocast (the
    cuBLAS projections and bf16 activations, not only the attention kernels)
    moves them by a few per cent whatever computes the attention -- measured
    on seeds 0 and 1, per layer, this library 0.6-4 % and the reference's own
    dense attention under the same autocast 1-3 % (s_r), with either one the
    worse depending on the seed.  Each parameter group (s_r of all layers,
    s_v of all layers) is therefore held to 2e-2 or to three times the
    reference's own bf16 error on the same inputs, whichever is larger."""
    V, B, T = 50257, 16, 512
    torch.manual_seed(0)
    m = ms.MultiscreenLM(V, d_model=256, num_heads=4, num_layers=4, max_seq_len=T)
    om = oracle.OracleLM(V, d_model=256, num_heads=4, num_layers=4, max_seq_len=T,
                         windowed=True)
    om.load_state_dict(m.state_dict())
    ob = oracle.OracleLM(V, d_model=256, num_heads=4, num_layers=4, max_seq_len=T)
    ob.load_state_dict(m.state_dict())
    om = om.double()
    m, ob = m.to(DEV), ob.to(DEV)
    ids = torch.randint(0, V, (B, T), generator=torch.Generator().manual_seed(2))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(ids.to(DEV), labels=ids.to(DEV))
    out["loss"].backward()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        bout = ob(ids.to(DEV), labels=ids.to(DEV))
    bout["loss"].backward()
    torch.cuda.synchronize()
    assert ms._lib.device_status() == 0
    ref = om(ids, labels=ids)
    ref["loss"].backward()
    assert rel_err(out["loss"].float().view(1), ref["loss"].view(1)) <= TOL
    assert rel_err(m.token_emb.weight.grad, om.token_emb.weight.grad) <= TOL
    assert rel_err(m.pos_emb.weight.grad, om.pos_emb.weight.grad) <= TOL
    for name in ("s_r", "s_v"):
        def group(model):
            return torch.cat([getattr(b.attn, name).grad.double().cpu() for b in model.blocks])
        e_ours = rel_err(group(m), group(om))
        e_base = rel_err(group(ob), group(om))
        assert e_ours <= max(TOL, 3.0 * e_base), (name, e_ours, e_base)
