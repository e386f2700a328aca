"""TanhNorm (multiscreen/norm.py:8-25) on the CUDA kernel."""
import torch
import torch.nn as nn

from .functional import tanh_norm


class TanhNorm(nn.Module):
    """TanhNorm(x) = tanh(|x|) / max(|x|, eps) * x over the last dim.

    Same constructor and (parameter-free) state as the reference module.
    Inside ScreeningAttention it is fused into the attention kernel's
    epilogue; this stand-alone module runs its own row kernel.
    """

    def __init__(self, eps: float = 1e-8):
        super().__init__()
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return tanh_norm(x, self.eps)
