"""ctypes binding of libscreening_b200.so (include/screening_b200.h).

Torch is used here only for device memory and the current stream: every
call passes raw device pointers, sizes and a cudaStream_t through the C ABI.
There is no CPU fallback -- a missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

# the in-tree build (built by _build.py / __graft_entry__.build())
LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libscreening_b200.so"

F32, BF16 = 0, 1
_DTYPES = {torch.float32: F32, torch.bfloat16: BF16}


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int32), ("B", c_int32), ("H", c_int32), ("Tq", c_int32), ("Tk", c_int32),
        ("D", c_int32), ("causal", c_int32), ("norms_given", c_int32),
        ("q_offset", c_int64), ("eps", c_float), ("stages", c_int32),
        ("q", c_void_p), ("q_sb", c_int64), ("q_st", c_int64),
        ("k", c_void_p), ("k_sb", c_int64), ("k_st", c_int64),
        ("v", c_void_p), ("v_sb", c_int64), ("v_st", c_int64),
        ("r", c_void_p), ("w", c_void_p), ("key_padding_mask", c_void_p), ("kpm_sb", c_int64),
        ("nq", c_void_p), ("nk", c_void_p), ("nv", c_void_p),
        ("y", c_void_p), ("no", c_void_p), ("tile_stats", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dropout_threshold", ctypes.c_uint32), ("_pad1", ctypes.c_uint32),
        ("dropout_seed", ctypes.c_uint64),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int32), ("B", c_int32), ("H", c_int32), ("Tq", c_int32), ("Tk", c_int32),
        ("D", c_int32), ("causal", c_int32), ("stages", c_int32),
        ("q_offset", c_int64), ("eps", c_float), ("_pad0", c_int32),
        ("q", c_void_p), ("q_sb", c_int64), ("q_st", c_int64),
        ("k", c_void_p), ("k_sb", c_int64), ("k_st", c_int64),
        ("v", c_void_p), ("v_sb", c_int64), ("v_st", c_int64),
        ("nq", c_void_p), ("nk", c_void_p), ("nv", c_void_p),
        ("y", c_void_p), ("no", c_void_p),
        ("dy", c_void_p), ("dy_sb", c_int64), ("dy_st", c_int64),
        ("r", c_void_p), ("w", c_void_p), ("key_padding_mask", c_void_p), ("kpm_sb", c_int64),
        ("dq", c_void_p), ("dq_sb", c_int64), ("dq_st", c_int64),
        ("dk", c_void_p), ("dk_sb", c_int64), ("dk_st", c_int64),
        ("dv", c_void_p), ("dv_sb", c_int64), ("dv_st", c_int64),
        ("dr", c_void_p), ("dw", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("dropout_threshold", ctypes.c_uint32), ("_pad1", ctypes.c_uint32),
        ("dropout_seed", ctypes.c_uint64),
    ]


class RowsLinearArgs(ctypes.Structure):
    _fields_ = [
        ("M", c_int32), ("N", c_int32), ("K", c_int32), ("act", c_int32),
        ("norm_eps", c_float), ("_pad0", c_int32),
        ("x", c_void_p), ("x_stride", c_int64), ("norm_w", c_void_p), ("W", c_void_p),
        ("res", c_void_p), ("res_stride", c_int64), ("y", c_void_p), ("y_stride", c_int64),
    ]


class XentArgs(ctypes.Structure):
    _fields_ = [
        ("rows", c_int64), ("V", c_int32), ("ignore_index", c_int32),
        ("logits", c_void_p), ("ld", c_int64), ("labels", c_void_p),
        ("lse", c_void_p), ("loss", c_void_p), ("dlogits", c_void_p), ("dld", c_int64),
        ("dscale", c_void_p),
    ]


class RmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("rows", c_int64), ("D", c_int32), ("x_dtype", c_int32), ("w_dtype", c_int32),
        ("y_dtype", c_int32), ("eps", c_float),
        ("x", c_void_p), ("w", c_void_p), ("y", c_void_p), ("rstd", c_void_p),
        ("dy", c_void_p), ("dx", c_void_p), ("dw", c_void_p), ("partials", c_void_p),
    ]


class KVCacheDesc(ctypes.Structure):
    _fields_ = [
        ("k_pages", c_void_p), ("v_pages", c_void_p), ("block_table", c_void_p),
        ("num_pages", c_int32), ("page_size", c_int32), ("max_blocks", c_int32),
        ("_pad0", c_int32),
    ]


class KVAppendArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int32), ("B", c_int32), ("H", c_int32), ("D", c_int32), ("n_new", c_int32),
        ("eps", c_float),
        ("k", c_void_p), ("k_sb", c_int64), ("k_st", c_int64),
        ("v", c_void_p), ("v_sb", c_int64), ("v_st", c_int64),
        ("positions", c_void_p), ("cache", KVCacheDesc),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int32), ("B", c_int32), ("H", c_int32), ("D", c_int32),
        ("num_splits", c_int32), ("eps", c_float),
        ("q", c_void_p), ("q_sb", c_int64), ("seq_lens", c_void_p),
        ("r", c_void_p), ("w", c_void_p), ("cache", KVCacheDesc),
        ("y", c_void_p), ("no", c_void_p), ("workspace", c_void_p),
        ("workspace_bytes", c_size_t),
    ]


EXPORTED = (
    "screen_fwd", "screen_bwd", "screen_bwd_workspace_size", "screen_kv_append",
    "screen_decode", "screen_decode_workspace_size", "screen_tanhnorm_fwd",
    "screen_tanhnorm_bwd", "screen_strerror", "screen_version", "screen_sizeof_args",
    "screen_last_cuda_error", "screen_decode_noalloc", "screen_fwd_workspace_size",
    "screen_device_status", "screen_dropout_bits", "screen_rows_linear",
    "screen_cross_entropy_fwd", "screen_cross_entropy_bwd", "screen_rmsnorm_partials",
    "screen_rmsnorm_fwd", "screen_rmsnorm_bwd", "screen_head_params_fwd",
    "screen_head_params_bwd", "screen_col_scale_bwd", "screen_decode_append",
)
ABI_VERSION = 5

_lib = None


def load() -> ctypes.CDLL:
    """Load the library once, bind signatures and check the ABI."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built; run __graft_entry__.build() (nvcc, sm_100a) first")
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.POINTER
    lib.screen_fwd.argtypes = [P(FwdArgs), c_void_p]
    lib.screen_bwd.argtypes = [P(BwdArgs), c_void_p]
    lib.screen_fwd_workspace_size.argtypes = [P(FwdArgs)]
    lib.screen_fwd_workspace_size.restype = c_size_t
    lib.screen_device_status.argtypes = [ctypes.c_int]
    lib.screen_bwd_workspace_size.argtypes = [P(BwdArgs)]
    lib.screen_bwd_workspace_size.restype = c_size_t
    lib.screen_kv_append.argtypes = [P(KVAppendArgs), c_void_p]
    lib.screen_decode.argtypes = [P(DecodeArgs), c_void_p]
    lib.screen_decode_workspace_size.argtypes = [P(DecodeArgs)]
    lib.screen_decode_workspace_size.restype = c_size_t
    lib.screen_decode_noalloc.argtypes = [P(DecodeArgs), c_void_p]
    lib.screen_tanhnorm_fwd.argtypes = [c_int32, c_int64, c_int32, c_float, c_void_p, c_void_p,
                                        c_void_p]
    lib.screen_tanhnorm_bwd.argtypes = [c_int32, c_int64, c_int32, c_float, c_void_p, c_void_p,
                                        c_void_p, c_void_p]
    lib.screen_rows_linear.argtypes = [P(RowsLinearArgs), c_void_p]
    lib.screen_cross_entropy_fwd.argtypes = [P(XentArgs), c_void_p]
    lib.screen_cross_entropy_bwd.argtypes = [P(XentArgs), c_void_p]
    lib.screen_rmsnorm_partials.argtypes = [c_int64]
    lib.screen_rmsnorm_partials.restype = c_int64
    lib.screen_rmsnorm_fwd.argtypes = [P(RmsNormArgs), c_void_p]
    lib.screen_rmsnorm_bwd.argtypes = [P(RmsNormArgs), c_void_p]
    lib.screen_head_params_fwd.argtypes = [c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p]
    lib.screen_head_params_bwd.argtypes = [c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_void_p, c_void_p]
    lib.screen_col_scale_bwd.argtypes = [c_int32, c_int64, c_int32, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p]
    lib.screen_decode_append.argtypes = [P(KVAppendArgs), P(DecodeArgs), c_void_p]
    lib.screen_dropout_bits.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_uint32]
    lib.screen_dropout_bits.restype = ctypes.c_uint32
    lib.screen_strerror.argtypes = [ctypes.c_int]
    lib.screen_strerror.restype = ctypes.c_char_p
    lib.screen_last_cuda_error.restype = ctypes.c_char_p
    lib.screen_sizeof_args.argtypes = [ctypes.c_int]
    lib.screen_sizeof_args.restype = c_int64
    if lib.screen_version() != ABI_VERSION:
        raise RuntimeError("libscreening_b200.so ABI version mismatch; rebuild it")
    for i, st in enumerate((FwdArgs, BwdArgs, KVCacheDesc, KVAppendArgs, DecodeArgs,
                            RowsLinearArgs, XentArgs, RmsNormArgs)):
        if lib.screen_sizeof_args(i) != ctypes.sizeof(st):
            raise RuntimeError(f"struct {st.__name__} size differs from the C header; rebuild")
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != 0:
        lib = load()
        msg = lib.screen_strerror(status).decode()
        detail = lib.screen_last_cuda_error().decode()
        raise RuntimeError(f"screening kernel error {status}: {msg}" + (f" ({detail})" if detail else ""))


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _DTYPES:
        raise TypeError(f"screening kernels take float32 or bfloat16, got {t.dtype}")
    return _DTYPES[t.dtype]


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("screening attention runs on CUDA tensors only (no CPU path)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _bthd(x: torch.Tensor) -> torch.Tensor:
    """A (B,T,H,D) view the kernels can read in place: unit D stride, stride D
    over H, 16-byte aligned base and batch/time strides; else a contiguous copy."""
    B, T, H, D = x.shape
    vec = 16 // x.element_size()
    if x.stride(3) != 1 or x.stride(2) != D or x.stride(0) % vec or x.stride(1) % vec or \
            x.data_ptr() % 16:
        x = x.contiguous()
    return x


def _kpm(mask):
    if mask is None:
        return None
    return mask.to(torch.bool).contiguous().view(torch.uint8)


def rows_linear(x, W, norm_w=None, eps=1e-6, act=0, res=None):
    """act(RMSNorm(x) W^T) + res for few rows (decode step): x (M, K) bf16 with
    M <= 8, W (N, K) bf16 contiguous, norm_w (K,) bf16 or None, res (M, N)
    bf16 or None; act 0 none, 1 GELU (erf).  Returns (M, N) bf16."""
    _require_cuda(x, W, norm_w, res)
    lib = load()
    M, K = x.shape
    N = W.shape[0]
    if x.stride(1) != 1 or not W.is_contiguous() or W.shape[1] != K:
        raise ValueError("rows_linear: x rows and W must be contiguous over K")
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    a = RowsLinearArgs(M=M, N=N, K=K, act=int(act), norm_eps=float(eps),
                       x=_ptr(x), x_stride=x.stride(0), norm_w=_ptr(norm_w), W=_ptr(W),
                       res=_ptr(res), res_stride=0 if res is None else res.stride(0),
                       y=_ptr(y), y_stride=y.stride(0))
    if res is not None and res.stride(1) != 1:
        raise ValueError("rows_linear: res must be contiguous over N")
    _check(lib.screen_rows_linear(ctypes.byref(a), _stream(x.device)))
    return y


def cross_entropy_fwd(logits, labels, ignore_index=-100):
    """Per-row (lse, loss) of bf16 logits (N, V) (V % 8 == 0) against int64
    labels (N,); loss is 0 for ignored labels."""
    _require_cuda(logits, labels)
    N, V = logits.shape
    lse = torch.empty(N, dtype=torch.float32, device=logits.device)
    loss = torch.empty(N, dtype=torch.float32, device=logits.device)
    a = XentArgs(rows=N, V=V, ignore_index=int(ignore_index), logits=_ptr(logits),
                 ld=logits.stride(0), labels=_ptr(labels), lse=_ptr(lse), loss=_ptr(loss))
    _check(load().screen_cross_entropy_fwd(ctypes.byref(a), _stream(logits.device)))
    return lse, loss


def rmsnorm_fwd(x, w, eps, out_dtype):
    """RMSNorm rows of x (.., D) with weight w (D,): returns (y, rstd); y in
    out_dtype (bf16, or x's dtype), rstd (rows,) fp32."""
    _require_cuda(x, w)
    D = x.shape[-1]
    rows = x.numel() // D
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    a = RmsNormArgs(rows=rows, D=D, x_dtype=_dtype_code(x), w_dtype=_dtype_code(w),
                    y_dtype=_dtype_code(y), eps=float(eps), x=_ptr(x), w=_ptr(w), y=_ptr(y),
                    rstd=_ptr(rstd))
    _check(load().screen_rmsnorm_fwd(ctypes.byref(a), _stream(x.device)))
    return y, rstd


def rmsnorm_bwd(x, w, rstd, dy):
    """Gradients (dx in x's dtype, dw in w's dtype) of rmsnorm_fwd for dy."""
    D = x.shape[-1]
    rows = x.numel() // D
    lib = load()
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    part = torch.empty(int(lib.screen_rmsnorm_partials(rows)), D, dtype=torch.float32,
                       device=x.device)
    a = RmsNormArgs(rows=rows, D=D, x_dtype=_dtype_code(x), w_dtype=_dtype_code(w),
                    y_dtype=_dtype_code(dy), x=_ptr(x), w=_ptr(w), rstd=_ptr(rstd),
                    dy=_ptr(dy), dx=_ptr(dx), dw=_ptr(dw), partials=_ptr(part))
    _check(lib.screen_rmsnorm_bwd(ctypes.byref(a), _stream(x.device)))
    return dx, dw


def cross_entropy_bwd(logits, labels, lse, dscale, ignore_index=-100):
    """dlogits (N, V) bf16 = (softmax - onehot) * dscale (a device scalar)."""
    N, V = logits.shape
    dl = torch.empty_like(logits)
    a = XentArgs(rows=N, V=V, ignore_index=int(ignore_index), logits=_ptr(logits),
                 ld=logits.stride(0), labels=_ptr(labels), lse=_ptr(lse),
                 dlogits=_ptr(dl), dld=dl.stride(0), dscale=_ptr(dscale))
    _check(load().screen_cross_entropy_bwd(ctypes.byref(a), _stream(logits.device)))
    return dl


def dropout_threshold(p: float) -> int:
    """The kernels' 32-bit drop threshold for probability p (0 <= p < 1): a
    score is dropped iff its counter bits are below it."""
    if not 0.0 <= p < 1.0:
        raise ValueError(f"dropout probability {p} outside [0, 1)")
    return min(int(p * 4294967296.0), 4294967295)


def dropout_bits(seed: int, bh: int, i: int, j: int) -> int:
    """Counter bits of score (bh, query i, key j) for `seed` (the library's
    screen_dropout_bits)."""
    return int(load().screen_dropout_bits(seed & (2**64 - 1), bh, i, j))


def screen_fwd(q, k, v, r, w, causal=True, key_padding_mask=None, eps=1e-8, q_offset=0,
               tile_stats=None, norms=None, stages=0, dropout=None):
    """Fused forward on raw projections q (B,Tq,H,D), k/v (B,Tk,H,D) (any
    batch/time strides); r, w (H,).  Returns (y, no, nq, nk, nv, q, k, v)
    where q, k, v are the (possibly re-laid-out) inputs the kernel read --
    the tensors to keep for the backward.  `norms` = (nq, nk, nv) skips the
    norm pass.  `dropout` = (threshold, seed) drops alpha (attention.py:190)."""
    _require_cuda(q, k, v, r, w, key_padding_mask)
    lib = load()
    q, k, v = _bthd(q), _bthd(k), _bthd(v)
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    dt = _dtype_code(q)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share a dtype")
    if k.shape[0] != B or k.shape[2:] != q.shape[2:] or v.shape != k.shape:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
    r = r.detach().contiguous().float()
    w = w.detach().contiguous().float()
    kpm = _kpm(key_padding_mask)
    dev = q.device
    if norms is None:
        nq = torch.empty((B, Tq, H), dtype=torch.float32, device=dev)
        nk = torch.empty((B, Tk, H), dtype=torch.float32, device=dev)
        nv = torch.empty((B, Tk, H), dtype=torch.float32, device=dev)
    else:
        nq, nk, nv = (t.contiguous() for t in norms)
    y = torch.empty((B, Tq, H, D), dtype=q.dtype, device=dev)
    no = torch.empty((B, Tq, H), dtype=torch.float32, device=dev)
    a = FwdArgs(dtype=dt, B=B, H=H, Tq=Tq, Tk=Tk, D=D, causal=int(bool(causal)),
                norms_given=int(norms is not None), q_offset=int(q_offset), eps=float(eps),
                stages=int(stages),
                q=_ptr(q), q_sb=q.stride(0), q_st=q.stride(1),
                k=_ptr(k), k_sb=k.stride(0), k_st=k.stride(1),
                v=_ptr(v), v_sb=v.stride(0), v_st=v.stride(1),
                r=_ptr(r), w=_ptr(w), key_padding_mask=_ptr(kpm),
                kpm_sb=0 if kpm is None else kpm.stride(0),
                nq=_ptr(nq), nk=_ptr(nk), nv=_ptr(nv), y=_ptr(y), no=_ptr(no),
                tile_stats=_ptr(tile_stats))
    if dropout is not None:
        a.dropout_threshold, a.dropout_seed = int(dropout[0]), int(dropout[1]) & (2**64 - 1)
    nbytes = int(lib.screen_fwd_workspace_size(ctypes.byref(a)))
    ws = None
    if nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = nbytes
    _check(lib.screen_fwd(ctypes.byref(a), _stream(dev)))
    return y, no, nq, nk, nv, q, k, v


def device_status(clear: bool = True) -> int:
    """0, or the status code a kernel left after giving up a bounded wait."""
    return int(load().screen_device_status(int(clear)))


def row_norms(x, eps=1e-8):
    """max(|x|, eps) per row of a (B,T,H,D) tensor -> (B,T,H) float32."""
    _require_cuda(x)
    lib = load()
    x = _bthd(x)
    B, T, H, D = x.shape
    nx = torch.empty((B, T, H), dtype=torch.float32, device=x.device)
    nv = torch.empty_like(nx)
    a = FwdArgs(dtype=_dtype_code(x), B=B, H=H, Tq=0, Tk=T, D=D, causal=1, eps=float(eps),
                stages=1, k=_ptr(x), k_sb=x.stride(0), k_st=x.stride(1),
                v=_ptr(x), v_sb=x.stride(0), v_st=x.stride(1), nk=_ptr(nx), nv=_ptr(nv))
    _check(lib.screen_fwd(ctypes.byref(a), _stream(x.device)))
    return nx


# screen_bwd stage flag (include/screening_b200.h): fixed-order dq.  Set
# whenever torch.use_deterministic_algorithms(True) is in effect.
SCREEN_BWD_DETERMINISTIC = 16


def screen_bwd(q, k, v, nq, nk, nv, y, no, dy, r, w, causal=True, key_padding_mask=None,
               eps=1e-8, q_offset=0, out=None, stages=0, dropout=None):
    """Backward of screen_fwd.  Returns dq, dk, dv ((B,T,H,D); written into
    `out` = (dq, dk, dv) views when given) and dr, dw (H,) float32.
    `dropout` must be the (threshold, seed) the forward used."""
    _require_cuda(dy)
    lib = load()
    dy = _bthd(dy.to(y.dtype))
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    dev = q.device
    r = r.detach().contiguous().float()
    w = w.detach().contiguous().float()
    kpm = _kpm(key_padding_mask)
    if out is None:
        dq = torch.empty((B, Tq, H, D), dtype=q.dtype, device=dev)
        dk = torch.empty((B, Tk, H, D), dtype=q.dtype, device=dev)
        dv = torch.empty((B, Tk, H, D), dtype=q.dtype, device=dev)
    else:
        dq, dk, dv = out
    dr = torch.empty(H, dtype=torch.float32, device=dev)
    dw = torch.empty(H, dtype=torch.float32, device=dev)
    a = BwdArgs(dtype=_dtype_code(q), B=B, H=H, Tq=Tq, Tk=Tk, D=D, causal=int(bool(causal)),
                stages=int(stages) | (SCREEN_BWD_DETERMINISTIC
                                      if torch.are_deterministic_algorithms_enabled() else 0),
                q_offset=int(q_offset), eps=float(eps),
                q=_ptr(q), q_sb=q.stride(0), q_st=q.stride(1),
                k=_ptr(k), k_sb=k.stride(0), k_st=k.stride(1),
                v=_ptr(v), v_sb=v.stride(0), v_st=v.stride(1),
                nq=_ptr(nq), nk=_ptr(nk), nv=_ptr(nv), y=_ptr(y), no=_ptr(no),
                dy=_ptr(dy), dy_sb=dy.stride(0), dy_st=dy.stride(1),
                r=_ptr(r), w=_ptr(w), key_padding_mask=_ptr(kpm),
                kpm_sb=0 if kpm is None else kpm.stride(0),
                dq=_ptr(dq), dq_sb=dq.stride(0), dq_st=dq.stride(1),
                dk=_ptr(dk), dk_sb=dk.stride(0), dk_st=dk.stride(1),
                dv=_ptr(dv), dv_sb=dv.stride(0), dv_st=dv.stride(1),
                dr=_ptr(dr), dw=_ptr(dw))
    if dropout is not None:
        a.dropout_threshold, a.dropout_seed = int(dropout[0]), int(dropout[1]) & (2**64 - 1)
    nbytes = lib.screen_bwd_workspace_size(ctypes.byref(a))
    ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    _check(lib.screen_bwd(ctypes.byref(a), _stream(dev)))
    return dq, dk, dv, dr, dw


def kv_desc(k_pages, v_pages, block_table) -> KVCacheDesc:
    return KVCacheDesc(k_pages=_ptr(k_pages), v_pages=_ptr(v_pages),
                       block_table=_ptr(block_table), num_pages=k_pages.shape[0],
                       page_size=k_pages.shape[2], max_blocks=block_table.shape[1])


def screen_kv_append(k, v, positions, k_pages, v_pages, block_table, eps=1e-8):
    """Normalise raw k, v (B,n,H,D) and write them into the paged cache at
    positions[b] + (0..n-1)."""
    _require_cuda(k, v, positions, k_pages, v_pages, block_table)
    lib = load()
    k, v = _bthd(k), _bthd(v)
    B, n, H, D = k.shape
    if k_pages.dtype != k.dtype:
        raise TypeError("cache dtype must match k/v")
    a = KVAppendArgs(dtype=_dtype_code(k), B=B, H=H, D=D, n_new=n, eps=float(eps),
                     k=_ptr(k), k_sb=k.stride(0), k_st=k.stride(1),
                     v=_ptr(v), v_sb=v.stride(0), v_st=v.stride(1),
                     positions=_ptr(positions), cache=kv_desc(k_pages, v_pages, block_table))
    _check(lib.screen_kv_append(ctypes.byref(a), _stream(k.device)))


def screen_decode(q, seq_lens, r, w, k_pages, v_pages, block_table, eps=1e-8, num_splits=1,
                  workspace=None):
    """One causal query per (b, h): q (B,H,D) raw.  Returns y (B,H,D), no (B,H)."""
    _require_cuda(q, seq_lens, r, w, k_pages, v_pages, block_table)
    lib = load()
    if q.stride(-1) != 1 or q.stride(-2) != q.shape[-1] or q.stride(0) % 4 or q.data_ptr() % 16:
        q = q.contiguous()
    B, H, D = q.shape
    dev = q.device
    y = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    no = torch.empty((B, H), dtype=torch.float32, device=dev)
    a = DecodeArgs(dtype=_dtype_code(q), B=B, H=H, D=D, num_splits=int(num_splits), eps=float(eps),
                   q=_ptr(q), q_sb=q.stride(0), seq_lens=_ptr(seq_lens), r=_ptr(r), w=_ptr(w),
                   cache=kv_desc(k_pages, v_pages, block_table), y=_ptr(y), no=_ptr(no))
    need = int(lib.screen_decode_workspace_size(ctypes.byref(a)))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    a.workspace = workspace.data_ptr()
    a.workspace_bytes = workspace.numel()
    _check(lib.screen_decode(ctypes.byref(a), _stream(dev)))
    return y, no


def screen_decode_append(k, v, positions, q, seq_lens, r, w, k_pages, v_pages, block_table,
                         eps=1e-8, num_splits=1, workspace=None):
    """screen_kv_append of one new raw k, v row per sequence (B,1,H,D) at
    positions[b], then screen_decode of q (B,H,D) over the same cache, in one
    launch.  Returns y (B,H,D), no (B,H)."""
    _require_cuda(k, v, positions, q, seq_lens, r, w, k_pages, v_pages, block_table)
    lib = load()
    k, v = _bthd(k), _bthd(v)
    if k.shape[1] != 1:
        raise ValueError("screen_decode_append appends one row per sequence")
    if k_pages.dtype != k.dtype or q.dtype != k.dtype:
        raise TypeError("cache dtype must match q / k / v")
    if q.stride(-1) != 1 or q.stride(-2) != q.shape[-1] or q.stride(0) % 4 or q.data_ptr() % 16:
        q = q.contiguous()
    B, H, D = q.shape
    dev = q.device
    cache = kv_desc(k_pages, v_pages, block_table)
    ap = KVAppendArgs(dtype=_dtype_code(k), B=B, H=H, D=D, n_new=1, eps=float(eps),
                      k=_ptr(k), k_sb=k.stride(0), k_st=k.stride(1),
                      v=_ptr(v), v_sb=v.stride(0), v_st=v.stride(1),
                      positions=_ptr(positions), cache=cache)
    y = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    no = torch.empty((B, H), dtype=torch.float32, device=dev)
    a = DecodeArgs(dtype=_dtype_code(q), B=B, H=H, D=D, num_splits=int(num_splits), eps=float(eps),
                   q=_ptr(q), q_sb=q.stride(0), seq_lens=_ptr(seq_lens), r=_ptr(r), w=_ptr(w),
                   cache=cache, y=_ptr(y), no=_ptr(no))
    need = int(lib.screen_decode_workspace_size(ctypes.byref(a)))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    a.workspace = workspace.data_ptr()
    a.workspace_bytes = workspace.numel()
    _check(lib.screen_decode_append(ctypes.byref(ap), ctypes.byref(a), _stream(dev)))
    return y, no


def screen_tanhnorm(x, eps=1e-8):
    _require_cuda(x)
    lib = load()
    xc = x.contiguous()
    y = torch.empty_like(xc)
    D = xc.shape[-1]
    _check(lib.screen_tanhnorm_fwd(_dtype_code(xc), xc.numel() // max(D, 1), D, float(eps),
                                   _ptr(xc), _ptr(y), _stream(x.device)))
    return y


def screen_tanhnorm_backward(x, dy, eps=1e-8):
    _require_cuda(x, dy)
    lib = load()
    xc = x.contiguous()
    dyc = dy.to(x.dtype).contiguous()
    dx = torch.empty_like(xc)
    D = xc.shape[-1]
    _check(lib.screen_tanhnorm_bwd(_dtype_code(xc), xc.numel() // max(D, 1), D, float(eps),
                                   _ptr(xc), _ptr(dyc), _ptr(dx), _stream(x.device)))
    return dx


def head_params_fwd(s_r, s_v):
    """(r, w) = (exp(s_r) + 1, exp(s_v) + 1) as fp32 (H,) tensors, one launch."""
    _require_cuda(s_r, s_v)
    lib = load()
    sr, sv = s_r.contiguous(), s_v.to(s_r.dtype).contiguous()
    H = sr.numel()
    r = torch.empty(H, dtype=torch.float32, device=sr.device)
    w = torch.empty(H, dtype=torch.float32, device=sr.device)
    _check(lib.screen_head_params_fwd(_dtype_code(sr), H, _ptr(sr), _ptr(sv), _ptr(r), _ptr(w),
                                      _stream(sr.device)))
    return r, w


def head_params_bwd(s_r, s_v, dr, dw):
    """(ds_r, ds_v) = (dr exp(s_r), dw exp(s_v)) in the parameters' dtype; a
    None gradient in gives None out."""
    _require_cuda(s_r, s_v)
    lib = load()
    sr, sv = s_r.contiguous(), s_v.to(s_r.dtype).contiguous()
    H = sr.numel()
    drc = None if dr is None else dr.float().contiguous()
    dwc = None if dw is None else dw.float().contiguous()
    ds_r = None if drc is None else torch.empty_like(sr)
    ds_v = None if dwc is None else torch.empty_like(sr)
    _check(lib.screen_head_params_bwd(_dtype_code(sr), H, _ptr(sr), _ptr(sv), _ptr(drc),
                                      _ptr(dwc), _ptr(ds_r), _ptr(ds_v), _stream(sr.device)))
    return ds_r, ds_v


def col_scale_bwd(dy, w, g, need_dw=True, need_dg=True):
    """Gradients of W diag(g) (W: rows x D, g: D) for dy: (dW, dg) in the
    common dtype of the three (None where not needed)."""
    _require_cuda(dy, w, g)
    lib = load()
    dt = w.dtype
    dyc, wc, gc = dy.to(dt).contiguous(), w.contiguous(), g.to(dt).contiguous()
    D = wc.shape[-1]
    rows = wc.numel() // D
    dw = torch.empty_like(wc) if need_dw else None
    dg = torch.empty(D, dtype=dt, device=wc.device) if need_dg else None
    _check(lib.screen_col_scale_bwd(_dtype_code(wc), rows, D, _ptr(dyc), _ptr(wc), _ptr(gc),
                                    _ptr(dw), _ptr(dg), _stream(wc.device)))
    return dw, dg
