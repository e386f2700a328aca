"""screen_head_params_fwd / _bwd: the module's r = exp(s_r) + 1 and
w = exp(s_v) + 1 (multiscreen/attention.py:164-165) in one launch each way,
against PyTorch's own ops on the same parameters."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H", [1, 16, 300])
def test_head_params_match_torch(ms, dtype, H):
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(H)
    s_r = (torch.randn(H, generator=g) - 1.0).to(dev, dtype).requires_grad_(True)
    s_v = (3.0 * torch.rand(H, generator=g) + 2.0).to(dev, dtype).requires_grad_(True)
    dr = torch.randn(H, generator=g).to(dev)
    dw = torch.randn(H, generator=g).to(dev)
    r, w = ms.functional.head_params(s_r, s_v)
    assert r.dtype == torch.float32 and w.dtype == torch.float32
    (r * dr).sum().add((w * dw).sum()).backward()
    got = (r.detach(), w.detach(), s_r.grad.clone(), s_v.grad.clone())
    s_r.grad = s_v.grad = None
    r0 = torch.exp(s_r.float()) + 1.0
    w0 = torch.exp(s_v.float()) + 1.0
    (r0 * dr).sum().add((w0 * dw).sum()).backward()
    ref = (r0.detach(), w0.detach(), s_r.grad, s_v.grad)
    # fp32 math on both sides; bf16 gradients carry one bf16 rounding
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    for name, a, b in zip(("r", "w", "ds_r", "ds_v"), got, ref):
        assert a.dtype == b.dtype, name
        err = ((a.float() - b.float()).abs() / b.float().abs().clamp_min(1e-30)).max().item()
        assert err <= (1e-6 if name in ("r", "w") else tol), (name, err)


def test_head_params_one_gradient_only(ms):
    dev = torch.device("cuda:0")
    s_r = torch.zeros(4, device=dev, requires_grad=True)
    s_v = torch.full((4,), 2.0, device=dev)
    r, w = ms.functional.head_params(s_r, s_v)
    (r.sum() + w.sum()).backward()
    assert torch.allclose(s_r.grad, torch.ones(4, device=dev))
    assert s_v.grad is None


def test_module_uses_the_fused_transform(ms):
    """ScreeningAttention's forward routes r, w through the fused transform
    and its s_r / s_v gradients equal the ones through PyTorch's ops."""
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    attn = ms.ScreeningAttention(128, 2).to(dev)
    with torch.no_grad():
        attn.s_r.copy_(torch.tensor([-1.0, 0.3]))
    x = torch.randn(2, 64, 128, device=dev)
    attn(x, x, x).square().sum().backward()
    g_fused = (attn.s_r.grad.clone(), attn.s_v.grad.clone())
    attn.zero_grad()
    q, k, v = attn._qkv(x, x, x)
    y = ms.functional.screening_attention(q, k, v, attn.sharpness(), attn.window(), causal=True)
    attn.out_proj(y.reshape(2, 64, 128)).square().sum().backward()
    for a, b in zip(g_fused, (attn.s_r.grad, attn.s_v.grad)):
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-7), (a, b)
