"""Paged K/V cache for KV-cached generation.

Pages are [num_pages, H, page_size, D] tensors of UNIT key/value rows per
layer; a block table [B, max_blocks] maps each sequence's logical block to a
physical page.  Because the softmask is exactly zero beyond the window
(multiscreen/attention.py:117-118), no key older than t - (ceil(max w) - 1)
is ever read again, so each sequence only owns `pages_per_seq` pages used as
a ring: logical block lb lives in page b * pages_per_seq + lb % pages_per_seq.
With pages_per_seq >= ceil(keep / page_size) + 1 every block inside the
window maps to a distinct page, and the table never changes after set-up.
"""
from __future__ import annotations

import math

import torch

from . import _lib


class PagedKVCache:
    def __init__(self, num_layers: int, batch: int, num_heads: int, head_dim: int, max_len: int,
                 max_window: float, dtype: torch.dtype, device: torch.device,
                 page_size: int = 64):
        self.num_layers, self.batch = num_layers, batch
        self.num_heads, self.head_dim = num_heads, head_dim
        self.page_size = page_size
        dmax = max(0, int(math.ceil(max_window)) - 1)
        # keys a decode step can still see: positions t - dmax .. t
        self.keep = min(max_len, dmax + 1)
        self.max_blocks = max(1, math.ceil(max_len / page_size))
        self.pages_per_seq = min(self.max_blocks, math.ceil(self.keep / page_size) + 1)
        num_pages = batch * self.pages_per_seq
        self.k_pages = [torch.zeros(num_pages, num_heads, page_size, head_dim, dtype=dtype,
                                    device=device) for _ in range(num_layers)]
        self.v_pages = [torch.zeros_like(p) for p in self.k_pages]
        lb = torch.arange(self.max_blocks, dtype=torch.int32)
        table = (torch.arange(batch, dtype=torch.int32).unsqueeze(1) * self.pages_per_seq
                 + (lb % self.pages_per_seq).unsqueeze(0))
        self.block_table = table.to(device)
        self._workspace = None
        # split each (b, h) window into runs of whole pages: at least one
        # wave of CTAs (148 SMs x 3 resident decode CTAs), and about
        # sqrt(pages) splits for long windows -- measured on B200 at 32K and
        # 100K keys per window, fewer splits leave a wave tail, more pay the
        # per-CTA pipeline fill; the split partials are summed
        # short windows (<= 512 keys: the w <= 256 of a model at init) take
        # one split per (b, h), which applies TanhNorm itself: a finishing
        # launch costs more than the few pages it would spread
        pages = math.ceil(self.keep / page_size)
        fill = math.ceil(148 * 3 / max(1, batch * num_heads))
        if self.keep <= 512:
            self.num_splits = 1
        else:
            self.num_splits = max(1, min(256, pages, max(fill, round(1.1 * math.sqrt(pages)))))

    def nbytes(self) -> int:
        return sum(p.numel() * p.element_size() for p in self.k_pages + self.v_pages)

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
               eps: float = 1e-8) -> None:
        """Write unit rows of raw k, v (B,n,H,D) at positions[b] + (0..n-1)."""
        dt = self.k_pages[layer].dtype
        _lib.screen_kv_append(k.to(dt), v.to(dt), positions, self.k_pages[layer],
                              self.v_pages[layer], self.block_table, eps)

    def append_decode(self, layer: int, k: torch.Tensor, v: torch.Tensor,
                      positions: torch.Tensor, q: torch.Tensor, seq_lens: torch.Tensor,
                      r: torch.Tensor, w: torch.Tensor, eps: float = 1e-8):
        """append(layer, k, v, positions) of one new row per sequence, then
        decode(layer, q, ...), in one launch."""
        dt = self.k_pages[layer].dtype
        if self._workspace is None:
            need = self.batch * self.num_heads * self.num_splits * self.head_dim * 4
            self._workspace = torch.empty(need + 256, dtype=torch.uint8, device=q.device)
        return _lib.screen_decode_append(k.to(dt), v.to(dt), positions, q.to(dt), seq_lens, r, w,
                                         self.k_pages[layer], self.v_pages[layer],
                                         self.block_table, eps, self.num_splits, self._workspace)

    def decode(self, layer: int, q: torch.Tensor, seq_lens: torch.Tensor, r: torch.Tensor,
               w: torch.Tensor, eps: float = 1e-8):
        """Screening decode of raw q (B,H,D) for the newest token of each sequence."""
        if self._workspace is None:
            need = self.batch * self.num_heads * self.num_splits * self.head_dim * 4
            self._workspace = torch.empty(need + 256, dtype=torch.uint8, device=q.device)
        return _lib.screen_decode(q.to(self.k_pages[layer].dtype), seq_lens, r, w, self.k_pages[layer], self.v_pages[layer],
                                  self.block_table, eps, self.num_splits, self._workspace)
