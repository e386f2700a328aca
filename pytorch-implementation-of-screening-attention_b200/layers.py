"""Pre-norm blocks around ScreeningAttention -- drop-ins for
multiscreen/layers.py:15-144 (same constructor arguments, submodule names
and therefore state_dict keys).  The FFN and the residuals stay in
PyTorch; the attention and the RMSNorms (functional.rms_norm, over the
nn.RMSNorm modules' weights) run on the library's kernels, except the norm
in front of each self-attention, which the attention absorbs into its QKV
GEMM (ScreeningAttention.forward_rmsnormed: the unit normalisation of q, k,
v divides out its per-token scale)."""
from __future__ import annotations

import torch
import torch.nn as nn

from .attention import ScreeningAttention
from .functional import rms_norm


def _ffn(d_model: int, ffn_dim: int, dropout: float) -> nn.Sequential:
    return nn.Sequential(
        nn.Linear(d_model, ffn_dim, bias=False),
        nn.GELU(),
        nn.Dropout(dropout),
        nn.Linear(ffn_dim, d_model, bias=False),
        nn.Dropout(dropout),
    )


class MultiscreenBlock(nn.Module):
    """x = x + ScreeningAttn(RMSNorm(x)); x = x + FFN(RMSNorm(x))  (layers.py:60-76)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int | None = None,
                 dropout: float = 0.0, causal: bool = True):
        super().__init__()
        ffn_dim = ffn_dim or 4 * d_model
        self.norm1 = nn.RMSNorm(d_model)
        self.norm2 = nn.RMSNorm(d_model)
        self.attn = ScreeningAttention(d_model=d_model, num_heads=num_heads, dropout=dropout,
                                       causal=causal)
        self.ffn = _ffn(d_model, ffn_dim, dropout)

    def forward(self, x: torch.Tensor, key_padding_mask: torch.Tensor | None = None) -> torch.Tensor:
        # self.attn(norm1(x), ...) with the RMSNorm absorbed into the QKV GEMM
        x = x + self.attn.forward_rmsnormed(x, self.norm1, key_padding_mask=key_padding_mask)
        x = x + self.ffn(rms_norm(self.norm2, x))
        return x


class MultiscreenDecoderLayer(nn.Module):
    """Self (causal) + cross (non-causal, T_q != T_k) screening attention and
    FFN, pre-norm (layers.py:79-144)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int | None = None,
                 dropout: float = 0.0):
        super().__init__()
        ffn_dim = ffn_dim or 4 * d_model
        self.norm1 = nn.RMSNorm(d_model)
        self.norm2 = nn.RMSNorm(d_model)
        self.norm3 = nn.RMSNorm(d_model)
        self.self_attn = ScreeningAttention(d_model=d_model, num_heads=num_heads, dropout=dropout,
                                            causal=True)
        self.cross_attn = ScreeningAttention(d_model=d_model, num_heads=num_heads,
                                             dropout=dropout, causal=False)
        self.ffn = _ffn(d_model, ffn_dim, dropout)

    def forward(self, x: torch.Tensor, memory: torch.Tensor,
                tgt_key_padding_mask: torch.Tensor | None = None,
                memory_key_padding_mask: torch.Tensor | None = None) -> torch.Tensor:
        x = x + self.self_attn.forward_rmsnormed(x, self.norm1,
                                                 key_padding_mask=tgt_key_padding_mask)
        normed = rms_norm(self.norm2, x)
        x = x + self.cross_attn(normed, memory, memory, key_padding_mask=memory_key_padding_mask)
        x = x + self.ffn(rms_norm(self.norm3, x))
        return x
