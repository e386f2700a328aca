"""Autograd entry points over the C-ABI kernels.

`screening_attention(q, k, v, r, w, ...)` is the op-level drop-in for the
reference's `_ScreeningFunc.apply(q, k, v, r, w, causal)`
(multiscreen/attention_triton.py:24-48) with three differences that make it
the whole of multiscreen/attention.py:156-196 instead of its middle:
  * q, k, v are the RAW projections in (B, T, H, D) layout -- unit
    normalisation happens inside the kernel, and their gradients flow back
    through the normalisation Jacobian;
  * the output is post-TanhNorm (B, T_q, H, D), ready for out_proj;
  * r and w receive gradients (the Triton wrapper returns None for them,
    attention_triton.py:44), so s_r and s_v train.
"""
from __future__ import annotations

import torch

from . import _lib


def _dropout_args(p: float, seed: int | None):
    """(threshold, seed) for the kernels, None without dropout.  Without an
    explicit seed one is drawn from torch's default CPU generator, so
    torch.manual_seed makes the masks reproducible."""
    if p <= 0.0:
        return None
    if seed is None:
        seed = int(torch.randint(0, 2**62, (1,)).item())
    return (_lib.dropout_threshold(p), int(seed))


class HeadParamsFn(torch.autograd.Function):
    """(s_r, s_v) -> (r, w) = (exp(s_r) + 1, exp(s_v) + 1) as fp32, the
    module's parameter transforms (multiscreen/attention.py:164-165), forward
    and backward one launch each instead of a cast, an exp and an add per
    parameter."""

    @staticmethod
    def forward(ctx, s_r, s_v):
        r, w = _lib.head_params_fwd(s_r, s_v)
        ctx.save_for_backward(s_r, s_v)
        return r, w

    @staticmethod
    def backward(ctx, dr, dw):
        s_r, s_v = ctx.saved_tensors
        ds_r, ds_v = _lib.head_params_bwd(s_r, s_v, dr if ctx.needs_input_grad[0] else None,
                                          dw if ctx.needs_input_grad[1] else None)
        return ds_r, ds_v


def head_params(s_r: torch.Tensor, s_v: torch.Tensor):
    """(r, w) for the kernels from the module's s_r, s_v (H,) parameters."""
    if s_r.is_cuda and s_v.is_cuda and s_r.dtype == s_v.dtype and \
            s_r.dtype in (torch.float32, torch.bfloat16):
        return HeadParamsFn.apply(s_r, s_v)
    return torch.exp(s_r.float()) + 1.0, torch.exp(s_v.float()) + 1.0


class ColScaleFn(torch.autograd.Function):
    """W diag(g) with its backward in one launch (dW = dY diag(g) and the
    column sums dg = sum_o dY W): the RMSNorm weight g folded into the QKV
    projection.  PyTorch's own backward of the broadcast product reduces the
    columns with a two-CTA kernel (tens of microseconds per layer)."""

    @staticmethod
    def forward(ctx, w, g):
        ctx.save_for_backward(w, g)
        return w * g

    @staticmethod
    def backward(ctx, dy):
        w, g = ctx.saved_tensors
        dw, dg = _lib.col_scale_bwd(dy, w, g, ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        if dw is not None and dw.dtype != w.dtype:
            dw = dw.to(w.dtype)
        if dg is not None and dg.dtype != g.dtype:
            dg = dg.to(g.dtype)
        return dw, dg


def col_scale(w: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """w * g (g over the last dimension of w)."""
    if w.is_cuda and g.is_cuda and w.dtype == g.dtype and w.dtype in (torch.float32,
                                                                     torch.bfloat16) \
            and w.dim() == 2 and g.dim() == 1 and w.shape[1] == g.shape[0]:
        return ColScaleFn.apply(w, g)
    return w * g


class ScreenFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, r, w, causal, key_padding_mask, eps, q_offset, dropout=None):
        y, no, nq, nk, nv, qq, kk, vv = _lib.screen_fwd(q, k, v, r, w, causal, key_padding_mask,
                                                        eps, q_offset, dropout=dropout)
        ctx.save_for_backward(qq, kk, vv, nq, nk, nv, y, no, r, w, key_padding_mask)
        ctx.causal, ctx.eps, ctx.q_offset, ctx.dropout = causal, eps, q_offset, dropout
        ctx.has_kpm = key_padding_mask is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        q, k, v, nq, nk, nv, y, no, r, w, kpm = ctx.saved_tensors
        dq, dk, dv, dr, dw = _lib.screen_bwd(q, k, v, nq, nk, nv, y, no, dy, r, w, ctx.causal,
                                             kpm if ctx.has_kpm else None, ctx.eps, ctx.q_offset,
                                             dropout=ctx.dropout)
        return (dq, dk, dv, dr.to(r.dtype) if ctx.needs_input_grad[3] else None,
                dw.to(w.dtype) if ctx.needs_input_grad[4] else None, None, None, None, None,
                None)


def screening_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r: torch.Tensor,
                        w: torch.Tensor, causal: bool = True,
                        key_padding_mask: torch.Tensor | None = None, eps: float = 1e-8,
                        q_offset: int = 0, dropout_p: float = 0.0,
                        dropout_seed: int | None = None) -> torch.Tensor:
    """y = TanhNorm(screen(q^, k^, v^; r, w)) on raw (B,T,H,D) projections.

    float32 and bfloat16 run natively; float16 inputs are computed in float32
    and cast back.  r, w are (H,) tensors (any float dtype; math in float32).
    dropout_p > 0 drops alpha as nn.Dropout does (attention.py:190): each score
    is zeroed with probability p, kept ones scaled by 1 / (1 - p); the mask is
    a counter-based hash of (dropout_seed, b*H+h, i, j), regenerated in the
    backward (see _lib.dropout_bits).
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("screening_attention runs on CUDA tensors only (no CPU path)")
    if dropout_p >= 1.0:
        # every alpha dropped: y = TanhNorm(0) = 0 (nn.Dropout(1.0) zeroes all)
        B, Tq, H, D = q.shape
        return (q * 0).reshape(B, Tq, H, D)
    out_dtype = q.dtype
    if q.dtype == torch.float16:
        q, k, v = q.float(), k.float(), v.float()
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    rf, wf = r.float(), w.float()
    y = ScreenFn.apply(q, k, v, rf, wf, bool(causal), key_padding_mask, float(eps), int(q_offset),
                       _dropout_args(float(dropout_p), dropout_seed))
    return y if y.dtype == out_dtype else y.to(out_dtype)


class ScreenPackedFn(torch.autograd.Function):
    """Self-attention on a packed (B, T, 3, H, D) QKV projection: the kernels
    read q, k, v as strided views and the backward writes dq, dk, dv straight
    into one packed gradient, so no per-view gradient assembly follows."""

    @staticmethod
    def forward(ctx, qkv, r, w, causal, key_padding_mask, eps, dropout=None):
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        y, no, nq, nk, nv, qq, kk, vv = _lib.screen_fwd(q, k, v, r, w, causal, key_padding_mask,
                                                        eps, 0, dropout=dropout)
        ctx.save_for_backward(qkv, nq, nk, nv, y, no, r, w, key_padding_mask)
        ctx.causal, ctx.eps, ctx.dropout = causal, eps, dropout
        ctx.has_kpm = key_padding_mask is not None
        ctx.views_ok = qq.data_ptr() == q.data_ptr() and kk.data_ptr() == k.data_ptr()
        return y

    @staticmethod
    def backward(ctx, dy):
        qkv, nq, nk, nv, y, no, r, w, kpm = ctx.saved_tensors
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        dqkv = torch.empty_like(qkv)
        out = (dqkv[:, :, 0], dqkv[:, :, 1], dqkv[:, :, 2])
        _, _, _, dr, dw = _lib.screen_bwd(q, k, v, nq, nk, nv, y, no, dy, r, w, ctx.causal,
                                          kpm if ctx.has_kpm else None, ctx.eps, 0, out=out,
                                          dropout=ctx.dropout)
        return (dqkv, dr.to(r.dtype) if ctx.needs_input_grad[1] else None,
                dw.to(w.dtype) if ctx.needs_input_grad[2] else None, None, None, None, None)


def screening_attention_packed(qkv: torch.Tensor, r: torch.Tensor, w: torch.Tensor,
                               causal: bool = True,
                               key_padding_mask: torch.Tensor | None = None,
                               eps: float = 1e-8, dropout_p: float = 0.0,
                               dropout_seed: int | None = None) -> torch.Tensor:
    """screening_attention for self-attention with q, k, v packed as one
    contiguous (B, T, 3, H, D) projection output (the fused QKV GEMM)."""
    if not qkv.is_cuda:
        raise RuntimeError("screening_attention runs on CUDA tensors only (no CPU path)")
    if qkv.dtype == torch.float16 or not qkv.is_contiguous() or dropout_p >= 1.0:
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        return screening_attention(q, k, v, r, w, causal, key_padding_mask, eps,
                                   dropout_p=dropout_p, dropout_seed=dropout_seed)
    return ScreenPackedFn.apply(qkv, r.float(), w.float(), bool(causal), key_padding_mask,
                                float(eps), _dropout_args(float(dropout_p), dropout_seed))


class CrossEntropyFn(torch.autograd.Function):
    """Mean cross-entropy of bf16 logits rows with ignore_index (the LM loss,
    multiscreen/model.py:103-107) in one pass forward and one backward, with
    no fp32 copy of the logits; the mean and its scale stay on the device."""

    @staticmethod
    def forward(ctx, logits, labels, ignore_index):
        lse, loss = _lib.cross_entropy_fwd(logits, labels, ignore_index)
        # rows whose label is outside [0, V) get loss 0 in the kernel (which
        # flags them in screen_device_status); they stay out of the mean too
        V = logits.shape[1]
        count = ((labels != ignore_index) & (labels >= 0) & (labels < V)).sum().to(torch.float32)
        ctx.save_for_backward(logits, labels, lse, count)
        ctx.ignore_index = ignore_index
        return loss.sum() / count

    @staticmethod
    def backward(ctx, dmean):
        logits, labels, lse, count = ctx.saved_tensors
        dscale = (dmean.float() / count).reshape(1).contiguous()
        dl = _lib.cross_entropy_bwd(logits, labels, lse, dscale, ctx.ignore_index)
        return dl, None, None


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor,
                  ignore_index: int = -100) -> torch.Tensor:
    """F.cross_entropy(logits, labels, ignore_index) (mean) for (N, V) logits;
    bf16 CUDA logits with V % 8 == 0 run the fused kernels."""
    if (logits.is_cuda and logits.dtype == torch.bfloat16 and logits.dim() == 2 and
            logits.shape[1] % 8 == 0 and logits.stride(1) == 1 and logits.stride(0) % 8 == 0 and
            logits.data_ptr() % 16 == 0):
        return CrossEntropyFn.apply(logits, labels.reshape(-1).long().contiguous(),
                                    int(ignore_index))
    return torch.nn.functional.cross_entropy(logits, labels, ignore_index=ignore_index)


class TanhNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):
        ctx.save_for_backward(x)
        ctx.eps = eps
        return _lib.screen_tanhnorm(x, eps)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return _lib.screen_tanhnorm_backward(x, dy, ctx.eps), None


def tanh_norm(x: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """TanhNorm over the last dim (multiscreen/norm.py:23-25) on CUDA."""
    if not x.is_cuda:
        raise RuntimeError("tanh_norm runs on CUDA tensors only (no CPU path)")
    out_dtype = x.dtype
    xx = x.float() if x.dtype == torch.float16 else x
    y = TanhNormFn.apply(xx, float(eps))
    return y if y.dtype == out_dtype else y.to(out_dtype)


def rms_eps(norm: torch.nn.RMSNorm, x: torch.Tensor) -> float:
    """nn.RMSNorm's eps.  None means the machine epsilon of the type torch
    computes in, float32 for bf16 / fp16 / fp32 inputs (not the input
    dtype's: bf16's would be 2^-7)."""
    if norm.eps is not None:
        return float(norm.eps)
    return float(torch.finfo(torch.float64 if x.dtype == torch.float64 else torch.float32).eps)


class RMSNormFn(torch.autograd.Function):
    """RMSNorm forward / backward on the library's kernels (fp32 math; the
    weight gradient summed in a fixed order)."""

    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype):
        y, rstd = _lib.rmsnorm_fwd(x, weight, eps, out_dtype)
        ctx.save_for_backward(x, weight, rstd)
        ctx.out_dtype = out_dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dx, dw = _lib.rmsnorm_bwd(x, weight, rstd, dy.to(ctx.out_dtype).contiguous())
        return dx, dw, None, None


def rms_norm(norm: torch.nn.RMSNorm, x: torch.Tensor) -> torch.Tensor:
    """`norm(x)` for the blocks' pre-norms (nn.RMSNorm over the last dim).
    On CUDA with fp32 / bf16 rows of a length that is a multiple of 8 (up to
    2048) it runs the fused kernels; under bf16 autocast it returns the bf16
    row the next Linear would cast the fp32 result to (the same rounding).
    Other cases (CPU tensors, fp16, other shapes) call the module."""
    w = norm.weight
    D = x.shape[-1]
    if not (x.is_cuda and w is not None and x.dtype in (torch.float32, torch.bfloat16) and
            w.dtype in (torch.float32, torch.bfloat16) and D % 8 == 0 and D <= 2048 and
            tuple(norm.normalized_shape) == (D,) and x.is_contiguous() and
            x.data_ptr() % 16 == 0):
        return norm(x)
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        out_dtype = torch.bfloat16
    else:
        out_dtype = torch.promote_types(x.dtype, w.dtype)
        if out_dtype != x.dtype:
            return norm(x)
    return RMSNormFn.apply(x, w, rms_eps(norm, x), out_dtype)
