"""The chunked windowed gradient oracle (used by the full-size GPU parity
tests) equals the dense autograd oracle, which is itself pinned to the
reference's golden vectors."""
import pytest
import torch

from tests.conftest import rel_err


@pytest.mark.parametrize("causal,q_offset,Tq,Tk", [(True, 0, 150, 150), (False, 0, 90, 130),
                                                     (True, 40, 70, 110)])
def test_windowed_grads_equal_dense(oracle, causal, q_offset, Tq, Tk):
    g = torch.Generator().manual_seed(Tq + Tk)
    B, H, D = 2, 3, 16
    q = torch.randn(B, Tq, H, D, generator=g)
    k = q[:, :1].expand(B, Tk, H, D) * 0.3 + torch.randn(B, Tk, H, D, generator=g)
    v = torch.randn(B, Tk, H, D, generator=g)
    r = torch.tensor([1.05, 1.5, 2.0])
    w = torch.tensor([9.5, 33.0, 61.0])
    dy = torch.randn(B, Tq, H, D, generator=g)
    ref = oracle.param_grads_reference(q, k, v, r, w, causal, dy=dy, q_offset=q_offset)
    got = oracle.windowed_core_grads(q, k, v, r, w, dy, causal, q_offset=q_offset, chunk=32)
    for name, a, b in zip(("y", "dq", "dk", "dv", "dr", "dw"), got, ref):
        assert rel_err(a, b) <= 1e-10, name
