"""Module-, model- and decode-level parity on the GPU."""
import math

import pytest
import torch

from tests.conftest import rel_err
from tests.helpers import golden_module

MG = golden_module()
pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_cfg1_module_fp32_vs_reference(ms, golden):
    """cfg1: ScreeningAttention(512, 8), default init from seed 0, B=2, T=128,
    fp32 fwd+bwd, against the reference's recorded numbers."""
    rec = golden["cfg1"]
    attn, x, cot = MG.cfg1_inputs(ms.ScreeningAttention)
    attn = attn.to(DEV)
    xr = x.to(DEV).requires_grad_(True)
    out = attn(xr, xr, xr)
    (out * cot.to(DEV)).sum().backward()
    assert rel_err(out[:, ::8], rec["y_rows"]) <= 1e-4
    assert rel_err(xr.grad[:, ::8], rec["dx_rows"]) <= 1e-4
    probe = torch.randn(512, generator=torch.Generator().manual_seed(99)).to(DEV)
    for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
        gw = getattr(attn, name).weight.grad
        assert rel_err(gw @ probe, rec[f"{name}_grad_probe"]) <= 1e-4
    assert rel_err(attn.s_r.grad, rec["ds_r"]) <= 1e-4
    assert rel_err(attn.s_v.grad, rec["ds_v"]) <= 1e-4


@pytest.mark.parametrize("name", list(MG.LM_CASES))
def test_lm_fp32_vs_reference(ms, golden, name):
    rec = golden["lm"][name]
    spec = rec["spec"]
    m = ms.MultiscreenLM(spec["vocab"], spec["d_model"], spec["H"], spec["L"], spec["ffn"],
                         spec["max_seq_len"]).to(DEV)
    m.load_state_dict(rec["state"])
    g = torch.Generator().manual_seed(spec["seed"] + 1000)
    ids = torch.randint(0, spec["vocab"], (spec["B"], spec["T"]), generator=g)
    labels = ids.clone()
    labels[:, :3] = -100
    prompt = torch.randint(0, spec["vocab"], spec["prompt"], generator=g)
    out = m(ids.to(DEV), labels=labels.to(DEV))
    assert rel_err(out["logits"], rec["logits"]) <= 1e-4
    assert out["loss"].item() == pytest.approx(rec["loss"].item(), rel=1e-4)
    out["loss"].backward()
    for li, blk in enumerate(m.blocks):
        assert rel_err(blk.attn.s_r.grad, rec["s_r_grad"][li]) <= 1e-3
        assert rel_err(blk.attn.s_v.grad, rec["s_v_grad"][li]) <= 1e-3
    toks = m.generate(prompt.to(DEV), max_new_tokens=spec["new"], top_k=1)
    assert torch.equal(toks.cpu(), rec["tokens"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [16, 64, 128])
def test_decode_equals_forward_last_rows(ms, dtype, D):
    """screen_decode over the paged ring cache == rows of screen_fwd over the
    whole prefix, for every prefix length in a sweep."""
    B, T, H = 3, 300, 2
    g = torch.Generator(device=DEV).manual_seed(D)
    q = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    k = (q.float() + 0.6 * torch.randn(B, T, H, D, device=DEV, generator=g)).to(dtype)
    v = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    r = torch.tensor([1.1, 1.4], device=DEV)
    w = torch.tensor([37.5, 150.0], device=DEV)
    y_full = ms.screening_attention(q, k, v, r, w, True)
    cache = ms.PagedKVCache(1, B, H, D, max_len=T, max_window=150.0, dtype=dtype, device=DEV,
                            page_size=16)
    assert cache.pages_per_seq < cache.max_blocks  # the ring actually wraps
    for t in range(T):
        pos = torch.full((B,), t, dtype=torch.int32, device=DEV)
        cache.append(0, k[:, t:t + 1], v[:, t:t + 1], pos)
        y, _ = cache.decode(0, q[:, t], pos + 1, r, w)
        tol = 1e-4 if dtype == torch.float32 else 2e-2
        assert rel_err(y, y_full[:, t]) <= tol, t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D,page_size,splits", [(64, 64, None), (64, 24, 5), (32, 16, 3),
                                                (128, 64, 1), (16, 8, 7), (64, 64, 40)])
def test_decode_long_prefix_page_sizes_and_splits(ms, dtype, D, page_size, splits):
    """Decode of the newest token after a long prefix (the window wraps the
    ring several times), for page sizes that are and are not multiples of 32
    keys and for split counts that do not divide the window's pages."""
    B, T, H = 2, 1500, 3
    g = torch.Generator(device=DEV).manual_seed(1000 + D + page_size)
    q = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    k = (q.float() + 0.5 * torch.randn(B, T, H, D, device=DEV, generator=g)).to(dtype)
    v = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    r = torch.tensor([1.05, 1.3, 1.02], device=DEV)
    w = torch.tensor([700.0, 90.5, 333.0], device=DEV)
    y_full = ms.screening_attention(q, k, v, r, w, True)
    cache = ms.PagedKVCache(1, B, H, D, max_len=T, max_window=700.0, dtype=dtype, device=DEV,
                            page_size=page_size)
    if splits is not None:
        cache.num_splits = splits
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    step = 250
    for t0 in range(0, T, step):
        pos = torch.full((B,), t0, dtype=torch.int32, device=DEV)
        cache.append(0, k[:, t0:t0 + step], v[:, t0:t0 + step], pos)
        t = t0 + step - 1
        y, _ = cache.decode(0, q[:, t], torch.full((B,), t + 1, dtype=torch.int32, device=DEV),
                            r, w)
        assert rel_err(y, y_full[:, t]) <= tol, t
    assert ms._lib.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_generate_cuda_graph_matches_eager(ms, dtype):
    """The CUDA-graph decode loop of generate() gives the eager loop's tokens
    and the same last-step logits (one captured step replayed per token)."""
    torch.manual_seed(3)
    m = ms.MultiscreenLM(113, d_model=128, num_heads=2, num_layers=3, max_seq_len=160).to(DEV)
    with torch.no_grad():
        for blk in m.blocks:
            blk.attn.s_r.fill_(math.log(0.05))
            blk.attn.s_v.copy_(torch.tensor([2.5, 3.9]))
    m = m.to(dtype)
    prompt = torch.randint(0, 113, (3, 41), device=DEV,
                           generator=torch.Generator(device=DEV).manual_seed(5))
    # top_k=1 keeps every logit equal to the largest and samples among them
    # (multinomial, as the reference does): an exact bf16 tie is broken by
    # the generator, so both loops start from the same generator state
    torch.manual_seed(11)
    eager = m.generate(prompt, max_new_tokens=40, top_k=1, cuda_graph=False)
    torch.manual_seed(11)
    graph = m.generate(prompt, max_new_tokens=40, top_k=1, cuda_graph=True)
    assert torch.equal(eager, graph)
    # same prefix, one more step, both ways: identical logits
    cache_e = m.make_cache(3, 45)
    cache_g = m.make_cache(3, 45)
    st = m._decode_state()
    m.prefill(prompt, cache_e)
    m.prefill(prompt, cache_g)
    tok = eager[:, 41:42]
    le = m.decode_step(tok, 41, cache_e, st)
    g, g_tok, g_pos, g_logits = m._capture_decode(3, 41, cache_g, st)
    g_tok.copy_(tok)
    g_pos.fill_(41)
    g.replay()
    # the GEMM library may pick another algorithm under capture: compare with
    # the contract's tolerance rather than bitwise
    assert rel_err(g_logits, le) <= (1e-4 if dtype == torch.float32 else 2e-2)


def test_bf16_lm_generate_matches_full_recompute(ms):
    """KV-cached generate == the reference's recompute-everything loop run on
    the same (bf16) model with the same kernels, token for token."""
    torch.manual_seed(0)
    m = ms.MultiscreenLM(97, d_model=128, num_heads=2, num_layers=2, max_seq_len=128).to(DEV)
    with torch.no_grad():
        for blk in m.blocks:
            blk.attn.s_r.fill_(math.log(0.05))
            blk.attn.s_v.copy_(torch.tensor([2.0, 3.5]))
    m = m.to(torch.bfloat16)
    prompt = torch.randint(0, 97, (3, 30), device=DEV)
    fast = m.generate(prompt, max_new_tokens=12, top_k=1)
    ids = prompt
    for _ in range(12):
        logits = m(ids)["logits"][:, -1, :].float()
        ids = torch.cat([ids, logits.argmax(-1, keepdim=True)], 1)
    agree = (fast == ids).float().mean().item()
    assert agree >= 0.95, agree


def test_decoder_layer_cross_attention(ms, oracle):
    torch.manual_seed(1)
    layer = ms.MultiscreenDecoderLayer(64, 4).to(DEV)
    x = torch.randn(2, 12, 64, device=DEV, requires_grad=True)
    mem = torch.randn(2, 30, 64, device=DEV, requires_grad=True)
    mask = torch.zeros(2, 30, dtype=torch.bool, device=DEV)
    mask[1, 20:] = True
    out = layer(x, mem, memory_key_padding_mask=mask)
    out.sum().backward()
    assert out.shape == x.shape and mem.grad is not None
    # the cross-attention alone against the oracle module with the same weights
    o = oracle.OracleScreeningAttention(64, 4, causal=False)
    o.load_state_dict({k: v.cpu() for k, v in layer.cross_attn.state_dict().items()})
    h = torch.randn(2, 12, 64)
    ref = o(h, mem.detach().cpu(), mem.detach().cpu(), key_padding_mask=mask.cpu())
    got = layer.cross_attn(h.to(DEV), mem.detach(), mem.detach(), key_padding_mask=mask)
    assert rel_err(got, ref) <= 1e-4


def test_tanhnorm_module_grad(ms, oracle):
    x = torch.randn(37, 64, dtype=torch.float64) * 3
    x[3] = 0
    x[5] *= 1e-9
    xr = x.float().clone().requires_grad_(True)
    ref = oracle.tanh_norm(xr, 1e-8)
    dy = torch.randn_like(ref)
    ref.backward(dy)
    xc = x.float().to(DEV).requires_grad_(True)
    y = ms.TanhNorm()(xc)
    y.backward(dy.to(DEV))
    assert rel_err(y, ref) <= 1e-5
    assert rel_err(xc.grad, xr.grad) <= 1e-4


def test_packed_qkv_path_matches_separate_views(ms):
    """Self-attention routes through the packed (B,T,3,H,D) Function; its
    output and every gradient equal the three-view path's."""
    torch.manual_seed(3)
    attn = ms.ScreeningAttention(128, 2).to(DEV).to(torch.bfloat16)
    with torch.no_grad():
        attn.s_r.copy_(torch.log(torch.tensor([0.1, 0.4])))
    x = torch.randn(2, 200, 128, device=DEV, dtype=torch.bfloat16)
    x1 = x.clone().requires_grad_(True)
    y1 = attn(x1, x1, x1)                       # packed path
    y1.float().square().sum().backward()
    g1 = [p.grad.clone() for p in attn.parameters()]
    attn.zero_grad()
    x2 = x.clone().requires_grad_(True)
    y2 = attn(x2, x2.clone(), x2.clone())        # separate projections
    y2.float().square().sum().backward()
    g2 = [p.grad.clone() for p in attn.parameters()]
    assert rel_err(y1, y2) <= 1e-2
    assert rel_err(x1.grad, x2.grad) <= 2e-2
    for a, b in zip(g1, g2):
        assert rel_err(a, b) <= 2e-2
