"""The RMSNorm in front of self-attention absorbed into the QKV GEMM
(ScreeningAttention.forward_rmsnormed): same output and gradients as running
nn.RMSNorm first and the attention on its output (multiscreen/layers.py:73-74),
for the block, the decoder layer and the KV-cached prefill."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("autocast", [False, True])
def test_block_absorbed_norm_matches_explicit_norm(ms, autocast):
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    blk = ms.MultiscreenBlock(128, 2).to(dev)
    with torch.no_grad():
        blk.norm1.weight.uniform_(0.5, 1.5)
        blk.attn.s_r.copy_(torch.tensor([-1.0, 0.2]))
    # residual-stream rows of very different scales: RMSNorm's rstd matters
    x = (torch.randn(2, 96, 128, device=dev) *
         torch.logspace(-2, 2, 96, device=dev).view(1, 96, 1)).requires_grad_(True)
    params = [x, blk.norm1.weight, blk.attn.q_proj.weight, blk.attn.v_proj.weight,
              blk.attn.s_r, blk.attn.s_v]

    def run(absorbed):
        for p in params:
            p.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            if absorbed:
                y = blk.attn.forward_rmsnormed(x, blk.norm1)
            else:
                n = blk.norm1(x)
                y = blk.attn(n, n, n)
        y.float().square().sum().backward()
        return [y.detach().float()] + [p.grad.clone() for p in params]

    got, ref = run(True), run(False)
    tol = 2e-2 if autocast else 1e-4
    names = ("y", "dx", "dnorm_w", "dWq", "dWv", "ds_r", "ds_v")
    for n, a, b in zip(names, got, ref):
        assert _rel(a, b) <= tol, (n, _rel(a, b))


def test_prefill_absorbed_norm_matches_forward(ms):
    dev = torch.device("cuda:0")
    torch.manual_seed(1)
    blk = ms.MultiscreenBlock(128, 2).to(dev).eval()
    with torch.no_grad():
        blk.norm1.weight.uniform_(0.5, 1.5)
    x = torch.randn(2, 80, 128, device=dev) * 3.0
    with torch.no_grad():
        a = blk.attn.prefill(x, None, 0, norm=blk.norm1)
        n = blk.norm1(x)
        b = blk.attn(n, n, n)
    assert _rel(a, b) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,D", [(768, 256), (3072, 1024), (5, 40)])
def test_col_scale_backward_matches_torch(ms, dtype, rows, D):
    dev = torch.device("cuda:0")
    g0 = torch.Generator().manual_seed(rows + D)
    w = torch.randn(rows, D, generator=g0).to(dev, dtype).requires_grad_(True)
    g = (torch.rand(D, generator=g0) + 0.5).to(dev, dtype).requires_grad_(True)
    dy = torch.randn(rows, D, generator=g0).to(dev, dtype)
    y = ms.functional.col_scale(w, g)
    y.backward(dy)
    got = (y.detach(), w.grad.clone(), g.grad.clone())
    w.grad = g.grad = None
    (w.float() * g.float()).backward(dy.float())
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    assert _rel(got[0], (w.float() * g.float()).detach()) <= tol
    assert _rel(got[1], w.grad) <= tol
    assert _rel(got[2], g.grad) <= tol
