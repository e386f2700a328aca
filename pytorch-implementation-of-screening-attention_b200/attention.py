"""ScreeningAttention on the B200 kernels -- drop-in for
multiscreen/attention.py:23-200.

Same constructor, forward signature, parameter names and initialisation
(q/k/v/out_proj bias-free Linear; s_v = linspace(0, ln 255, H) so w = 2..256;
s_r = 0 so r = 2; attention.py:52-66), so reference checkpoints load
unchanged.  Everything between the projections and out_proj
(attention.py:156-196) runs in one fused CUDA forward and one fused CUDA
backward (functional.screening_attention).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .functional import col_scale, head_params, screening_attention, screening_attention_packed
from .norm import TanhNorm
from .sequence_parallel import current_shard, screening_attention_sharded


class ScreeningAttention(nn.Module):
    """Multi-head Screening Attention.

    Args match the reference: d_model, num_heads, dropout (on alpha, applied
    in training mode as nn.Dropout does, attention.py:190; the fused kernels
    draw the mask from a counter-based hash seeded from torch's default
    generator, so it is not bit-identical to torch's dropout), causal, eps.
    """

    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.0, causal: bool = True,
                 eps: float = 1e-8):
        super().__init__()
        assert d_model % num_heads == 0, "d_model must be divisible by num_heads"
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.causal = causal
        self.eps = eps
        self.q_proj = nn.Linear(d_model, d_model, bias=False)
        self.k_proj = nn.Linear(d_model, d_model, bias=False)
        self.v_proj = nn.Linear(d_model, d_model, bias=False)
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.s_v = nn.Parameter(torch.linspace(0, math.log(255), num_heads))   # log(w - 1)
        self.s_r = nn.Parameter(torch.zeros(num_heads))                         # log(r - 1)
        self.attn_dropout = nn.Dropout(dropout)
        self.tahn_norm = TanhNorm(eps=eps)  # attribute name kept from the reference

    # ------------------------------------------------------------------
    def window(self) -> torch.Tensor:
        """w = exp(s_v) + 1 (attention.py:164), float32."""
        return torch.exp(self.s_v.float()) + 1.0

    def sharpness(self) -> torch.Tensor:
        """r = exp(s_r) + 1 (attention.py:165), float32."""
        return torch.exp(self.s_r.float()) + 1.0

    def _head_params(self):
        """(r, w) as above, both transforms in one launch (and one in the
        backward) on CUDA."""
        return head_params(self.s_r, self.s_v)

    def _wqkv(self, gamma: torch.Tensor | None = None) -> torch.Tensor:
        """[W_q; W_k; W_v] (3 d_model, d_model), its input columns scaled by
        `gamma` (an RMSNorm weight absorbed into the projections) if given."""
        wqkv = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0)
        return wqkv if gamma is None else col_scale(wqkv, gamma)

    def _qkv(self, query, key, value, gamma: torch.Tensor | None = None):
        B, Tq, _ = query.shape
        Tk = key.shape[1]
        H, D = self.num_heads, self.head_dim
        if query is key and key is value:
            # self-attention: one GEMM for the three projections; q, k, v are
            # strided (B,T,H,D) views the kernel reads in place
            qkv = F.linear(query, self._wqkv(gamma)).view(B, Tq, 3, H, D)
            return qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        if gamma is not None:
            raise ValueError("an absorbed RMSNorm applies to self-attention only")
        q = self.q_proj(query).view(B, Tq, H, D)
        k = self.k_proj(key).view(B, Tk, H, D)
        v = self.v_proj(value).view(B, Tk, H, D)
        return q, k, v

    def _dropout_p(self) -> float:
        """Attention dropout probability of this call (0 outside training)."""
        return float(self.attn_dropout.p) if self.training else 0.0

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                key_padding_mask: torch.Tensor | None = None) -> torch.Tensor:
        """query (B,T_q,d_model), key/value (B,T_k,d_model),
        key_padding_mask (B,T_k) bool, True = ignore.  Returns (B,T_q,d_model)."""
        if query is key and key is value:
            return self._self_attention(query, None, key_padding_mask)
        p = self._dropout_p()
        B, Tq, _ = query.shape
        q, k, v = self._qkv(query, key, value)
        y = screening_attention(q, k, v, *self._head_params(), causal=self.causal,
                                key_padding_mask=key_padding_mask, eps=self.eps,
                                dropout_p=p)
        return self.out_proj(y.reshape(B, Tq, self.d_model))

    def forward_rmsnormed(self, x: torch.Tensor, norm: nn.RMSNorm,
                          key_padding_mask: torch.Tensor | None = None) -> torch.Tensor:
        """self.forward(n, n, n) with n = norm(x) (the pre-norm blocks'
        `self.attn(self.norm1(x), ...)`, multiscreen/layers.py:73-74), with the
        RMSNorm absorbed into the QKV GEMM instead of run as a pass over x.

        RMSNorm multiplies token t's row by rstd_t > 0 and every feature c by
        weight_c.  rstd_t scales q_t, k_t and v_t of every head alike, and
        the unit normalisation of each head's rows (attention.py:156-158)
        divides it out again, so the output only depends on x diag(weight):
        q, k, v = x (W diag(weight))^T give the same attention, and the same
        gradients for x, weight and W (the loss does not depend on rstd).
        The one difference is the eps clamp of that normalisation: a head row
        whose norm falls below eps (1e-8) is scaled differently."""
        return self._self_attention(x, norm.weight, key_padding_mask)

    def _self_attention(self, x, gamma, key_padding_mask):
        p = self._dropout_p()
        B, Tq, _ = x.shape
        shard = current_shard() if self.causal else None
        if shard is not None:
            if p > 0:
                raise NotImplementedError(
                    "attention dropout with a sequence-sharded input is not implemented")
            # causal self-attention of one block of a sequence-sharded input:
            # the K/V halo before the block comes from the previous ranks
            q, k, v = self._qkv(x, x, x, gamma)
            y = screening_attention_sharded(q, k, v, *self._head_params(),
                                            key_padding_mask=key_padding_mask, eps=self.eps,
                                            shard=shard)
        else:
            # one GEMM for the three projections; the kernels read q, k, v in
            # place and write their gradients into one buffer
            H, D = self.num_heads, self.head_dim
            qkv = F.linear(x, self._wqkv(gamma)).view(B, Tq, 3, H, D)
            y = screening_attention_packed(qkv, *self._head_params(),
                                           causal=self.causal,
                                           key_padding_mask=key_padding_mask, eps=self.eps,
                                           dropout_p=p)
        return self.out_proj(y.reshape(B, Tq, self.d_model))

    # ------------------------------------------------------------------
    # KV-cached inference (used by MultiscreenLM.generate)
    # ------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, x: torch.Tensor, cache, layer: int,
                norm: nn.RMSNorm | None = None) -> torch.Tensor:
        """Causal self-attention over a whole prompt x (B,T,d) that also
        writes the prompt's last `cache.keep` unit keys/values into `cache`
        (cache None: attention only).  Inside sequence_parallel(), x is this
        rank's block of a sharded prompt.  With `norm`, the attention is that
        of norm(x), the RMSNorm absorbed as in forward_rmsnormed (the cache
        holds unit rows, which the RMSNorm's row scale does not change)."""
        B, T, _ = x.shape
        q, k, v = self._qkv(x, x, x, None if norm is None else norm.weight)
        shard = current_shard()
        if cache is not None:
            if shard is not None and shard.world > 1:
                raise NotImplementedError("a KV cache fill from a sequence-sharded prefill")
            keep = min(T, cache.keep)
            if keep > 0:
                pos = torch.full((B,), T - keep, dtype=torch.int32, device=x.device)
                cache.append(layer, k[:, T - keep:], v[:, T - keep:], pos, eps=self.eps)
        if shard is not None:
            y = screening_attention_sharded(q, k, v, *self._head_params(),
                                            eps=self.eps, shard=shard)
        else:
            y = screening_attention(q, k, v, *self._head_params(), causal=True,
                                    eps=self.eps)
        return self.out_proj(y.reshape(B, T, self.d_model))

    @torch.no_grad()
    def decode_step(self, x: torch.Tensor, cache, layer: int, positions: torch.Tensor,
                    seq_lens: torch.Tensor, wqkv: torch.Tensor | None = None,
                    r: torch.Tensor | None = None, w: torch.Tensor | None = None) -> torch.Tensor:
        """One new token per sequence: x (B,1,d) at `positions` (B,) int32.
        Appends its unit k/v to the cache and attends over the cached window."""
        B = x.shape[0]
        if wqkv is None:
            wqkv = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0)
        y = self.decode_attend(F.linear(x, wqkv), cache, layer, positions, seq_lens, r, w)
        return self.out_proj(y.reshape(B, 1, self.d_model))

    def decode_attend(self, qkv: torch.Tensor, cache, layer: int, positions: torch.Tensor,
                      seq_lens: torch.Tensor, r: torch.Tensor | None = None,
                      w: torch.Tensor | None = None) -> torch.Tensor:
        """The attention of decode_step between the QKV projection (qkv: B
        rows of 3*d_model) and out_proj: appends the unit k/v rows to the
        cache, attends over the cached window; returns (B, d_model)."""
        B = qkv.shape[0]
        H, D = self.num_heads, self.head_dim
        qkv = qkv.reshape(B, 1, 3, H, D)
        # the new token's unit k / v rows are written by the decode launch itself
        y, _ = cache.append_decode(layer, qkv[:, :, 1], qkv[:, :, 2], positions, qkv[:, 0, 0],
                                   seq_lens, self.sharpness() if r is None else r,
                                   self.window() if w is None else w, eps=self.eps)
        return y.reshape(B, self.d_model)
