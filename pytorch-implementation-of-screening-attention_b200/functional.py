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


class ScreenFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, r, w, causal, key_padding_mask, eps, q_offset):
        y, no, nq, nk, nv, qq, kk, vv = _lib.screen_fwd(q, k, v, r, w, causal, key_padding_mask,
                                                        eps, q_offset)
        ctx.save_for_backward(qq, kk, vv, nq, nk, nv, y, no, r, w, key_padding_mask)
        ctx.causal, ctx.eps, ctx.q_offset = causal, eps, q_offset
        ctx.has_kpm = key_padding_mask is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        q, k, v, nq, nk, nv, y, no, r, w, kpm = ctx.saved_tensors
        dq, dk, dv, dr, dw = _lib.screen_bwd(q, k, v, nq, nk, nv, y, no, dy, r, w, ctx.causal,
                                             kpm if ctx.has_kpm else None, ctx.eps, ctx.q_offset)
        return (dq, dk, dv, dr.to(r.dtype) if ctx.needs_input_grad[3] else None,
                dw.to(w.dtype) if ctx.needs_input_grad[4] else None, None, None, None, None)


def screening_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r: torch.Tensor,
                        w: torch.Tensor, causal: bool = True,
                        key_padding_mask: torch.Tensor | None = None, eps: float = 1e-8,
                        q_offset: int = 0) -> torch.Tensor:
    """y = TanhNorm(screen(q^, k^, v^; r, w)) on raw (B,T,H,D) projections.

    float32 and bfloat16 run natively; float16 inputs are computed in float32
    and cast back.  r, w are (H,) tensors (any float dtype; math in float32).
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("screening_attention runs on CUDA tensors only (no CPU path)")
    out_dtype = q.dtype
    if q.dtype == torch.float16:
        q, k, v = q.float(), k.float(), v.float()
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    rf, wf = r.float(), w.float()
    y = ScreenFn.apply(q, k, v, rf, wf, bool(causal), key_padding_mask, float(eps), int(q_offset))
    return y if y.dtype == out_dtype else y.to(out_dtype)


class ScreenPackedFn(torch.autograd.Function):
    """Self-attention on a packed (B, T, 3, H, D) QKV projection: the kernels
    read q, k, v as strided views and the backward writes dq, dk, dv straight
    into one packed gradient, so no per-view gradient assembly follows."""

    @staticmethod
    def forward(ctx, qkv, r, w, causal, key_padding_mask, eps):
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        y, no, nq, nk, nv, qq, kk, vv = _lib.screen_fwd(q, k, v, r, w, causal, key_padding_mask,
                                                        eps, 0)
        ctx.save_for_backward(qkv, nq, nk, nv, y, no, r, w, key_padding_mask)
        ctx.causal, ctx.eps = causal, eps
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
                                          kpm if ctx.has_kpm else None, ctx.eps, 0, out=out)
        return (dqkv, dr.to(r.dtype) if ctx.needs_input_grad[1] else None,
                dw.to(w.dtype) if ctx.needs_input_grad[2] else None, None, None, None)


def screening_attention_packed(qkv: torch.Tensor, r: torch.Tensor, w: torch.Tensor,
                               causal: bool = True,
                               key_padding_mask: torch.Tensor | None = None,
                               eps: float = 1e-8) -> torch.Tensor:
    """screening_attention for self-attention with q, k, v packed as one
    contiguous (B, T, 3, H, D) projection output (the fused QKV GEMM)."""
    if not qkv.is_cuda:
        raise RuntimeError("screening_attention runs on CUDA tensors only (no CPU path)")
    if qkv.dtype == torch.float16 or not qkv.is_contiguous():
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        return screening_attention(q, k, v, r, w, causal, key_padding_mask, eps)
    return ScreenPackedFn.apply(qkv, r.float(), w.float(), bool(causal), key_padding_mask,
                                float(eps))


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
