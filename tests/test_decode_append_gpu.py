"""screen_decode_append (one new k / v row per sequence written by the
decode launch itself) == screen_kv_append followed by screen_decode, bit for
bit: the same output and the same cache contents, over a prefix that wraps
the paged ring, for one and several splits and the fallback page sizes."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D,page_size,splits", [(64, 64, None), (64, 24, 5), (32, 16, 3),
                                                (128, 64, 1), (16, 8, 7), (64, 16, 40)])
def test_decode_append_equals_append_then_decode(ms, dtype, D, page_size, splits):
    B, T, H = 3, 700, 2
    g = torch.Generator(device=DEV).manual_seed(7 * D + page_size)
    q = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    k = (q.float() + 0.5 * torch.randn(B, T, H, D, device=DEV, generator=g)).to(dtype)
    v = torch.randn(B, T, H, D, device=DEV, generator=g).to(dtype)
    r = torch.tensor([1.05, 1.3], device=DEV)
    w = torch.tensor([300.0, 41.5], device=DEV)
    caches = [ms.PagedKVCache(1, B, H, D, max_len=T, max_window=300.0, dtype=dtype, device=DEV,
                              page_size=page_size) for _ in range(2)]
    for c in caches:
        if splits is not None:
            c.num_splits = splits
    assert caches[0].pages_per_seq < caches[0].max_blocks   # the ring wraps
    for t in range(T):
        pos = torch.full((B,), t, dtype=torch.int32, device=DEV)
        caches[0].append(0, k[:, t:t + 1], v[:, t:t + 1], pos)
        y0, n0 = caches[0].decode(0, q[:, t], pos + 1, r, w)
        y1, n1 = caches[1].append_decode(0, k[:, t:t + 1], v[:, t:t + 1], pos, q[:, t], pos + 1,
                                         r, w)
        if t % 97 == 0 or t == T - 1:
            assert torch.equal(y0, y1), t
            assert torch.equal(n0, n1), t
            assert torch.equal(caches[0].k_pages[0], caches[1].k_pages[0]), t
            assert torch.equal(caches[0].v_pages[0], caches[1].v_pages[0]), t
    assert ms._lib.device_status() == 0


def test_decode_append_rejects_mismatched_requests(ms):
    c = ms.PagedKVCache(1, 2, 2, 64, max_len=64, max_window=16.0, dtype=torch.bfloat16,
                        device=DEV)
    k = torch.randn(2, 2, 2, 64, device=DEV, dtype=torch.bfloat16)   # two new rows
    q = torch.randn(2, 2, 64, device=DEV, dtype=torch.bfloat16)
    pos = torch.zeros(2, dtype=torch.int32, device=DEV)
    r = torch.ones(2, device=DEV) * 1.5
    with pytest.raises(ValueError):
        c.append_decode(0, k, k, pos, q, pos + 1, r, r)
