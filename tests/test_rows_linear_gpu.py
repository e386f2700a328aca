"""Few-row linear layer of the decode step (screen_rows_linear) against the
PyTorch ops it replaces (nn.RMSNorm -> nn.Linear -> nn.GELU -> residual add,
multiscreen/layers.py:60-76, model.py:97), and the fused decode step of
MultiscreenLM against the unfused one.  bf16 I/O: max |x - ref| / max |ref|
<= 2e-2."""
import importlib

import pytest
import torch
import torch.nn.functional as F

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
L = importlib.import_module("pytorch-implementation-of-screening-attention_b200._lib")


@pytest.mark.parametrize("M", [1, 3, 4, 8])
@pytest.mark.parametrize("N,K", [(1024, 1024), (3072, 1024), (4096, 1024), (1024, 4096),
                                 (50257, 256), (200, 72)])
@pytest.mark.parametrize("mode", ["plain", "norm_gelu", "residual"])
def test_rows_linear_matches_torch(cuda, M, N, K, mode):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn(K, device=cuda, generator=g)).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda, generator=g).to(torch.bfloat16)
    eps = torch.finfo(torch.bfloat16).eps
    if mode == "plain":
        got = L.rows_linear(x, W)
        ref = F.linear(x, W)
    elif mode == "norm_gelu":
        got = L.rows_linear(x, W, norm_w=nw, eps=eps, act=1)
        ref = F.gelu(F.linear(F.rms_norm(x, (K,), nw, eps), W))
    else:
        got = L.rows_linear(x, W, res=res)
        ref = res + F.linear(x, W)
    assert rel_err(got.float(), ref.float()) <= 2e-2


def test_fused_decode_step_matches_unfused(ms, cuda):
    torch.manual_seed(0)
    m = ms.MultiscreenLM(1000, d_model=256, num_heads=4, num_layers=3, max_seq_len=256)
    m = m.to(cuda).to(torch.bfloat16).eval()
    ids = torch.randint(0, 1000, (4, 97), device=cuda)
    with torch.no_grad():
        outs = []
        for fused in (True, False):
            cache = m.make_cache(4, 128)
            st = m._decode_state()
            m.prefill(ids[:, :-1], cache)
            if not fused:
                m._rows_fast = lambda x: False
            pos = torch.full((4,), 96, dtype=torch.int32, device=cuda)
            outs.append(m.decode_step(ids[:, -1:], pos, cache, st).float())
            if not fused:
                del m._rows_fast
        ref = m(ids)["logits"][:, -1].float()
    assert m._rows_fast(torch.zeros(4, 1, 256, device=cuda, dtype=torch.bfloat16))
    assert rel_err(outs[0], outs[1]) <= 2e-2
    assert rel_err(outs[0], ref) <= 2e-2
