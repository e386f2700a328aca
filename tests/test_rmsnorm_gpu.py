"""RMSNorm kernels (screen_rmsnorm_fwd / _bwd) against nn.RMSNorm in fp64:
the pre-norms of multiscreen/layers.py:60-76 and model.py:98.  fp32 rows and
weights within 1e-4 (output, dx, dw); a bf16 output (what autocast's next
Linear casts the fp32 result to) within one bf16 rounding (2e-2); bf16 rows
and weights within 2e-2."""
import importlib

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
FN = importlib.import_module("pytorch-implementation-of-screening-attention_b200.functional")
DEV = torch.device("cuda:0")


def _ref(x, w, eps, dy):
    xd = x.double().requires_grad_(True)
    wd = w.double().requires_grad_(True)
    y = torch.nn.functional.rms_norm(xd, (x.shape[-1],), wd, eps)
    y.backward(dy.double())
    return y.detach(), xd.grad, wd.grad


@pytest.mark.parametrize("x_dt,w_dt,y_dt,tol", [
    (torch.float32, torch.float32, torch.float32, 1e-4),
    (torch.float32, torch.float32, torch.bfloat16, 2e-2),
    (torch.bfloat16, torch.bfloat16, torch.bfloat16, 2e-2),
    (torch.float32, torch.bfloat16, torch.bfloat16, 2e-2),
])
@pytest.mark.parametrize("rows,D", [(1, 8), (37, 256), (8192, 256), (300, 1024), (5, 2048)])
def test_rmsnorm_matches_torch(ms, x_dt, w_dt, y_dt, tol, rows, D):
    g = torch.Generator(device=DEV).manual_seed(rows + D)
    x = (2.0 * torch.randn(rows, D, device=DEV, generator=g)).to(x_dt)
    w = (1.0 + 0.3 * torch.randn(D, device=DEV, generator=g)).to(w_dt)
    dy = torch.randn(rows, D, device=DEV, generator=g).to(y_dt)
    eps = 1.1920928955078125e-07
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    y = FN.RMSNormFn.apply(xr, wr, eps, y_dt)
    y.backward(dy)
    assert y.dtype == y_dt and xr.grad.dtype == x_dt and wr.grad.dtype == w_dt
    ry, rdx, rdw = _ref(x, w, eps, dy)
    assert rel_err(y, ry) <= tol
    assert rel_err(xr.grad, rdx) <= tol
    assert rel_err(wr.grad, rdw) <= tol


def test_rms_norm_module_path_and_determinism(ms):
    """functional.rms_norm over an nn.RMSNorm equals the module (fp32), and
    the weight gradient is bitwise the same on a second run."""
    norm = torch.nn.RMSNorm(256).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(256, device=DEV))
    x = torch.randn(4, 777, 256, device=DEV)
    grads = []
    for _ in range(2):
        norm.weight.grad = None
        xr = x.clone().requires_grad_(True)
        y = FN.rms_norm(norm, xr)
        y.square().sum().backward()
        grads.append(norm.weight.grad.clone())
    assert rel_err(y, norm(x)) <= 1e-5
    assert torch.equal(grads[0], grads[1])
