"""The C-ABI library: it loads, exports every symbol include/*.h declares,
its argument structs match the ctypes mirrors, and argument validation
answers with status codes.  No kernel runs here (no GPU needed)."""
import ctypes
import re

import pytest

from tests.conftest import REPO


def header_symbols():
    text = "".join(p.read_text() for p in (REPO / "include").glob("*.h"))
    return sorted(set(re.findall(r"SCREEN_API\s+[\w\s\*]+?\b(screen_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(ms):
    lib = ms._lib.load()
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(ms._lib.EXPORTED)


def test_struct_sizes_and_version(ms):
    lib = ms._lib.load()
    assert lib.screen_version() == ms._lib.ABI_VERSION
    L = ms._lib
    mirrors = (L.FwdArgs, L.BwdArgs, L.KVCacheDesc, L.KVAppendArgs, L.DecodeArgs,
               L.RowsLinearArgs, L.XentArgs, L.RmsNormArgs)
    for i, st in enumerate(mirrors):
        assert lib.screen_sizeof_args(i) == ctypes.sizeof(st), st.__name__
    assert lib.screen_sizeof_args(len(mirrors)) == -1
    assert lib.screen_sizeof_args(99) == -1


def test_strerror_covers_codes(ms):
    lib = ms._lib.load()
    for code in range(0, -11, -1):
        assert lib.screen_strerror(code).decode() != "unknown status"
    assert lib.screen_strerror(-77).decode() == "unknown status"


def test_validation_before_any_launch(ms):
    """Bad requests are rejected before anything touches the device."""
    L = ms._lib
    lib = L.load()
    assert lib.screen_fwd(None, None) == -1
    a = L.FwdArgs(dtype=7, B=1, H=1, Tq=1, Tk=1, D=64)
    assert lib.screen_fwd(ctypes.byref(a), None) == -3          # dtype
    a = L.FwdArgs(dtype=L.BF16, B=1, H=1, Tq=1, Tk=1, D=48)
    assert lib.screen_fwd(ctypes.byref(a), None) == -2          # head dim
    a = L.FwdArgs(dtype=L.BF16, B=-1, H=1, Tq=1, Tk=1, D=64)
    assert lib.screen_fwd(ctypes.byref(a), None) == -1          # negative size
    a = L.FwdArgs(dtype=L.BF16, B=1, H=1, Tq=4, Tk=4, D=64)     # null buffers
    assert lib.screen_fwd(ctypes.byref(a), None) == -1
    a = L.FwdArgs(dtype=L.F32, B=1, H=1, Tq=4, Tk=4, D=64, q=8, k=16, v=32, nq=64, nk=64,
                  nv=64, y=64, no=128, r=256, w=512)            # misaligned q
    assert lib.screen_fwd(ctypes.byref(a), None) == -4
    a = L.FwdArgs(dtype=L.BF16, B=1, H=1, Tq=4, Tk=4, D=64, q=16, q_st=12, k=16, v=32, nq=64,
                  nk=64, nv=64, y=64, no=128, r=256, w=512)     # bf16 row stride not 16 B
    assert lib.screen_fwd(ctypes.byref(a), None) == -4
    b = L.BwdArgs(dtype=L.F32, B=1, H=1, Tq=4, Tk=4, D=64)
    assert lib.screen_bwd(ctypes.byref(b), None) == -1
    assert lib.screen_bwd_workspace_size(ctypes.byref(b)) > 0
    d = L.DecodeArgs(dtype=L.BF16, B=1, H=1, D=64, num_splits=0)
    assert lib.screen_decode(ctypes.byref(d), None) == -1
    d.num_splits = 2
    assert lib.screen_decode_workspace_size(ctypes.byref(d)) >= 2 * 64 * 4
    assert lib.screen_tanhnorm_fwd(7, 4, 24, 1e-8, None, None, None) == -3
    assert lib.screen_tanhnorm_fwd(L.F32, 4, 0, 1e-8, None, None, None) == -1
    assert lib.screen_tanhnorm_fwd(L.F32, 0, 64, 1e-8, None, None, None) == 0
    # per-head parameter transforms
    assert lib.screen_head_params_fwd(7, 4, None, None, None, None, None) == -3
    assert lib.screen_head_params_fwd(L.BF16, -1, None, None, None, None, None) == -1
    assert lib.screen_head_params_fwd(L.BF16, 0, None, None, None, None, None) == 0
    assert lib.screen_head_params_fwd(L.F32, 4, None, None, None, None, None) == -1
    assert lib.screen_head_params_bwd(L.F32, 4, None, None, None, None, None, None, None) == 0
    assert lib.screen_head_params_bwd(L.F32, 4, 256, 256, 512, None, None, None, None) == -1
    # folded-norm column scale backward
    assert lib.screen_col_scale_bwd(7, 4, 8, None, None, None, None, None, None) == -3
    assert lib.screen_col_scale_bwd(L.F32, 4, 0, None, None, None, None, None, None) == -1
    assert lib.screen_col_scale_bwd(L.F32, 4, 8, None, None, None, None, None, None) == 0
    assert lib.screen_col_scale_bwd(L.F32, 4, 8, None, None, None, 256, None, None) == -1
