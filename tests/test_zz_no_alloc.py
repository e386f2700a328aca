"""screen_decode_noalloc: decode for callers that cannot allocate device
memory on their serving path (a fixed device-memory budget after start-up,
or a C/FFI caller without a device allocator).  It keeps its split-K
partials in a static 4 MiB device array instead of a caller workspace.

Called here through the C ABI (ctypes) and compared with screen_decode,
which takes a caller workspace, on two calls in a row.  This file is
collected last so that a run stopping at the first failure has run every
other test first; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _cache_with_tokens(ms, dtype, B, H, D, T, w_max, dev=DEV):
    g = torch.Generator(device=dev).manual_seed(11)
    cache = ms.PagedKVCache(1, B, H, D, max_len=T, max_window=w_max, dtype=dtype, device=dev,
                            page_size=16)
    k = torch.randn(B, T, H, D, device=dev, generator=g).to(dtype)
    v = torch.randn(B, T, H, D, device=dev, generator=g).to(dtype)
    cache.append(0, k, v, torch.zeros(B, dtype=torch.int32, device=dev))
    return cache, k


def _args(L, q, seq_lens, r, w, cache, y, no, num_splits, workspace=None):
    a = L.DecodeArgs(dtype=L._dtype_code(q), B=q.shape[0], H=q.shape[1], D=q.shape[2],
                     num_splits=num_splits, eps=1e-8, q=q.data_ptr(), q_sb=q.stride(0),
                     seq_lens=seq_lens.data_ptr(), r=r.data_ptr(), w=w.data_ptr(),
                     cache=L.kv_desc(cache.k_pages[0], cache.v_pages[0], cache.block_table),
                     y=y.data_ptr(), no=no.data_ptr())
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel()
    return a


def _compare_twice(ms, dtype, dev):
    """Two noalloc calls in a row on `dev`, each against screen_decode with a
    caller workspace on the same inputs."""
    L = ms._lib
    lib = L.load()
    B, H, D, T = 4, 3, 64, 200
    cache, k = _cache_with_tokens(ms, dtype, B, H, D, T, w_max=120.0, dev=dev)
    r = torch.tensor([1.05, 1.2, 1.6], device=dev)
    w = torch.tensor([7.5, 60.0, 120.0], device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for call, (t, splits) in enumerate([(150, 4), (199, 3)]):
        # the query of each call leans on a different cached key, so a stale
        # partial left by the first call would show in the second
        q = (k[:, t - 5] + 0.3 * torch.randn(B, H, D, device=dev, dtype=torch.float32)
             .to(dtype)).contiguous()
        seq_lens = torch.full((B,), t + 1, dtype=torch.int32, device=dev)
        y_ref = torch.empty(B, H, D, dtype=dtype, device=dev)
        no_ref = torch.empty(B, H, dtype=torch.float32, device=dev)
        ws = torch.empty(B * H * splits * D * 4 + 256, dtype=torch.uint8, device=dev)
        a_ref = _args(L, q, seq_lens, r, w, cache, y_ref, no_ref, splits, ws)
        assert lib.screen_decode(ctypes.byref(a_ref), ctypes.c_void_p(stream)) == 0
        y = torch.full((B, H, D), float("nan"), dtype=dtype, device=dev)
        no = torch.full((B, H), float("nan"), dtype=torch.float32, device=dev)
        a = _args(L, q, seq_lens, r, w, cache, y, no, splits)
        assert lib.screen_decode_noalloc(ctypes.byref(a), ctypes.c_void_p(stream)) == 0, call
        torch.cuda.synchronize(dev)
        assert torch.isfinite(y.float()).all()
        assert rel_err(y, y_ref) <= tol, call
        assert rel_err(no, no_ref) <= tol, call
        assert torch.count_nonzero(y_ref) > 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_decode_matches_workspace_decode_twice(ms, dtype):
    with torch.cuda.device(DEV):
        _compare_twice(ms, dtype, DEV)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs a second visible GPU")
def test_noalloc_decode_on_a_second_device(ms):
    """The scratch address and the decode kernel's shared-memory opt-in are
    per device: a process that decoded on cuda:0 must also decode on cuda:1."""
    with torch.cuda.device(DEV):
        _compare_twice(ms, torch.bfloat16, DEV)
    dev1 = torch.device("cuda:1")
    with torch.cuda.device(dev1):
        _compare_twice(ms, torch.bfloat16, dev1)


def test_noalloc_decode_rejects_requests_beyond_the_scratch(ms):
    L = ms._lib
    lib = L.load()
    B, H, D = 64, 16, 128
    cache, _ = _cache_with_tokens(ms, torch.bfloat16, 1, H, D, 16, w_max=16.0)
    q = torch.zeros(B, H, D, dtype=torch.bfloat16, device=DEV)
    seq_lens = torch.ones(B, dtype=torch.int32, device=DEV)
    r = torch.ones(H, device=DEV)
    w = torch.ones(H, device=DEV)
    y = torch.empty(B, H, D, dtype=torch.bfloat16, device=DEV)
    no = torch.empty(B, H, dtype=torch.float32, device=DEV)
    # 64 * 16 * 2 * 128 * 4 B = 1 MiB fits; 16 splits = 8 MiB does not
    a = _args(L, q, seq_lens, r, w, cache, y, no, num_splits=16)
    st = lib.screen_decode_noalloc(ctypes.byref(a), ctypes.c_void_p(0))
    assert st == -10
    assert "static scratch" in lib.screen_strerror(st).decode()
