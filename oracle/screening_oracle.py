"""CPU oracle for Screening Attention -- TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU, fp32/fp64) restatement of the reference package
`multiscreen` (ibusan100/PyTorch-implementation-of-Screening-Attention),
used as the checker for the CUDA path.  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may import it; the product never does.

Pinned: tests/test_oracle_golden.py checks every function here against
golden vectors produced by the reference itself (tests/golden/make_golden.py
imports the reference package and records its outputs and gradients).

Citations are path:line inside the reference project.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


# ---------------------------------------------------------------------------
# Functional core on raw projections laid out (B, T, H, D)
# ---------------------------------------------------------------------------
def unit_rows(x: torch.Tensor, eps: float) -> torch.Tensor:
    """F.normalize(x, dim=-1, eps) -- multiscreen/attention.py:156-158."""
    return x / x.norm(dim=-1, keepdim=True).clamp_min(eps)


def tanh_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    """TanhNorm -- multiscreen/norm.py:23-25."""
    n = x.norm(dim=-1, keepdim=True).clamp(min=eps)
    return (torch.tanh(n) / n) * x


def softmask(T_q: int, T_k: int, w: torch.Tensor, causal: bool, q_offset: int = 0,
             q_start: int = 0, k_start: int = 0) -> torch.Tensor:
    """(H, T_q, T_k) distance-aware cosine softmask.

    causal:     multiscreen/attention.py:92-119 (rel = j - i, -w < rel <= 0)
    non-causal: multiscreen/attention.py:174-183 (rel = |j - i| < w)
    q_offset shifts query i to key-axis position i + q_offset (0 in the
    reference); q_start/k_start select a sub-block of a larger matrix.
    """
    i_idx = torch.arange(q_start, q_start + T_q, device=w.device).unsqueeze(1) + q_offset
    j_idx = torch.arange(k_start, k_start + T_k, device=w.device).unsqueeze(0)
    rel = (j_idx - i_idx).to(w.dtype)
    wv = w.view(-1, 1, 1)
    if causal:
        cos_mask = 0.5 * (torch.cos(math.pi * rel.unsqueeze(0) / wv) + 1.0)
        in_window = (rel.unsqueeze(0) > -wv) & (rel.unsqueeze(0) <= 0)
        return cos_mask * in_window.to(w.dtype)
    rel = rel.abs()
    cos_mask = 0.5 * (torch.cos(math.pi * rel.unsqueeze(0) / wv) + 1.0)
    return cos_mask * (rel.unsqueeze(0) < wv).to(w.dtype)


def screening_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r: torch.Tensor,
                   w: torch.Tensor, causal: bool = True,
                   key_padding_mask: torch.Tensor | None = None, eps: float = 1e-8,
                   q_offset: int = 0) -> torch.Tensor:
    """Dense screening attention + TanhNorm on raw (B,T,H,D) projections.

    Returns y (B, T_q, H, D).  Follows multiscreen/attention.py:156-196:
    normalise (:156-158), sim (:161), trim-and-square (:75-90, :168),
    softmask (:170-184), key padding (:186-188), alpha @ v (:193),
    TanhNorm (:196).
    """
    qh = unit_rows(q.transpose(1, 2), eps)   # (B,H,Tq,D)
    kh = unit_rows(k.transpose(1, 2), eps)
    vh = unit_rows(v.transpose(1, 2), eps)
    sim = torch.matmul(qh, kh.transpose(-2, -1))
    rr = r.view(1, -1, 1, 1)
    alpha = F.relu(1.0 - rr * (1.0 - sim)).pow(2)
    alpha = alpha * softmask(q.shape[1], k.shape[1], w, causal, q_offset).unsqueeze(0)
    if key_padding_mask is not None:
        alpha = alpha.masked_fill(key_padding_mask.unsqueeze(1).unsqueeze(2), 0.0)
    out = torch.matmul(alpha, vh)
    return tanh_norm(out, eps).transpose(1, 2)


# ---------------------------------------------------------------------------
# Attention dropout (multiscreen/attention.py:68,190 applies nn.Dropout to
# alpha).  torch's dropout mask cannot be reproduced bit for bit, so the CUDA
# path draws its mask from a counter-based hash instead; this restates that
# hash (the library's screen_dropout_bits) so that parity tests can apply the
# very same mask here.
# ---------------------------------------------------------------------------
_M32 = 0xFFFFFFFF


def _mul32(x: torch.Tensor, c: int) -> torch.Tensor:
    """(x * c) mod 2^32 for int64 tensors holding uint32 values (split so no
    product leaves int64)."""
    lo = x * (c & 0xFFFF)
    hi = ((x * (c >> 16)) & 0xFFFF) << 16
    return (lo + hi) & _M32


def _mix32(x: torch.Tensor) -> torch.Tensor:
    """lowbias32 finalizer: x ^= x>>16; x *= 0x7feb352d; x ^= x>>15;
    x *= 0x846ca68b; x ^= x>>16 (all mod 2^32)."""
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    return x ^ (x >> 16)


def dropout_bits(seed: int, bh: torch.Tensor, i: torch.Tensor, j: torch.Tensor) -> torch.Tensor:
    """Counter bits of scores (bh, query i, key j), broadcast over the three
    int64 index tensors: k = mix(seed_lo ^ mix(seed_hi ^ bh * 0x9E3779B1)),
    row = mix(k ^ i * 0x85EBCA77), bits = mix(row ^ j * 0xC2B2AE3D)."""
    lo, hi = seed & _M32, (seed >> 32) & _M32
    k = _mix32(lo ^ _mix32(hi ^ _mul32(bh.long(), 0x9E3779B1)))
    row = _mix32(k ^ _mul32(i.long(), 0x85EBCA77))
    return _mix32(row ^ _mul32(j.long(), 0xC2B2AE3D))


def dropout_keep(seed: int, threshold: int, B: int, H: int, i: torch.Tensor,
                 j: torch.Tensor) -> torch.Tensor:
    """(B, H, len(i), len(j)) float mask: 2^32 / (2^32 - threshold) where the
    score is kept (bits >= threshold), 0 where dropped."""
    bh = torch.arange(B * H).view(B, H, 1, 1)
    bits = dropout_bits(seed, bh, i.view(1, 1, -1, 1), j.view(1, 1, 1, -1))
    scale = 4294967296.0 / (4294967296.0 - threshold)
    return (bits >= threshold).double() * scale


def screening_core_windowed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, r: torch.Tensor,
                            w: torch.Tensor, causal: bool = True,
                            key_padding_mask: torch.Tensor | None = None, eps: float = 1e-8,
                            q_offset: int = 0, chunk: int = 256,
                            dropout: tuple[int, int] | None = None) -> torch.Tensor:
    """Same result as screening_core, evaluated per block of `chunk` queries
    against only the keys inside the largest window (the softmask of
    multiscreen/attention.py:118 is exactly zero for |i - j| >= w), so large T
    never builds a T x T matrix.  dropout = (threshold, seed) applies the
    CUDA path's dropout mask to alpha (attention.py:190)."""
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    dmax = int(math.ceil(float(w.detach().max()))) - 1 if H > 0 else -1
    kh = unit_rows(k.transpose(1, 2), eps)
    vh = unit_rows(v.transpose(1, 2), eps)
    outs = []
    for i0 in range(0, Tq, chunk):
        i1 = min(Tq, i0 + chunk)
        p0, p1 = i0 + q_offset, i1 - 1 + q_offset
        lo = max(0, p0 - dmax)
        hi = min(Tk - 1, p1 if causal else p1 + dmax)
        qh = unit_rows(q[:, i0:i1].transpose(1, 2), eps)
        if hi < lo or dmax < 0:
            outs.append(torch.zeros(B, H, i1 - i0, D, dtype=q.dtype))
            continue
        sim = torch.matmul(qh, kh[:, :, lo:hi + 1].transpose(-2, -1))
        alpha = F.relu(1.0 - r.view(1, -1, 1, 1) * (1.0 - sim)).pow(2)
        m = softmask(i1 - i0, hi - lo + 1, w, causal, q_offset, q_start=i0, k_start=lo)
        alpha = alpha * m.unsqueeze(0)
        if key_padding_mask is not None:
            alpha = alpha.masked_fill(key_padding_mask[:, lo:hi + 1].unsqueeze(1).unsqueeze(2), 0.0)
        if dropout is not None and dropout[0] > 0:
            keep = dropout_keep(dropout[1], dropout[0], B, H, torch.arange(i0, i1),
                                torch.arange(lo, hi + 1))
            alpha = alpha * keep.to(alpha.dtype)
        outs.append(torch.matmul(alpha, vh[:, :, lo:hi + 1]))
    out = torch.cat(outs, dim=2) if outs else torch.zeros(B, H, 0, D, dtype=q.dtype)
    return tanh_norm(out, eps).transpose(1, 2)


# ---------------------------------------------------------------------------
# Modules mirroring the reference's (same ctor args and parameter names)
# ---------------------------------------------------------------------------
class OracleScreeningAttention(nn.Module):
    """multiscreen/attention.py:23-200 restated; parameter names and init
    (q/k/v/out_proj bias-free Linear, s_v = linspace(0, ln 255, H), s_r = 0)
    as in attention.py:52-66."""

    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.0, causal: bool = True,
                 eps: float = 1e-8, windowed: bool = False):
        super().__init__()
        assert d_model % num_heads == 0
        self.d_model, self.num_heads = d_model, num_heads
        self.head_dim = d_model // num_heads
        self.causal, self.eps, self.windowed = causal, eps, windowed
        self.q_proj = nn.Linear(d_model, d_model, bias=False)
        self.k_proj = nn.Linear(d_model, d_model, bias=False)
        self.v_proj = nn.Linear(d_model, d_model, bias=False)
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.s_v = nn.Parameter(torch.linspace(0, math.log(255), num_heads))
        self.s_r = nn.Parameter(torch.zeros(num_heads))

    def forward(self, query, key, value, key_padding_mask=None):
        B, Tq, _ = query.shape
        Tk = key.shape[1]
        H, D = self.num_heads, self.head_dim
        q = self.q_proj(query).view(B, Tq, H, D)
        k = self.k_proj(key).view(B, Tk, H, D)
        v = self.v_proj(value).view(B, Tk, H, D)
        w = torch.exp(self.s_v) + 1.0   # attention.py:164
        r = torch.exp(self.s_r) + 1.0   # attention.py:165
        core = screening_core_windowed if self.windowed else screening_core
        y = core(q, k, v, r, w, self.causal, key_padding_mask, self.eps)
        return self.out_proj(y.reshape(B, Tq, self.d_model))


class OracleBlock(nn.Module):
    """multiscreen/layers.py:15-76 (pre-norm block)."""

    def __init__(self, d_model, num_heads, ffn_dim=None, dropout=0.0, causal=True, windowed=False):
        super().__init__()
        ffn_dim = ffn_dim or 4 * d_model
        self.norm1 = nn.RMSNorm(d_model)
        self.norm2 = nn.RMSNorm(d_model)
        self.attn = OracleScreeningAttention(d_model, num_heads, dropout, causal, windowed=windowed)
        self.ffn = nn.Sequential(nn.Linear(d_model, ffn_dim, bias=False), nn.GELU(),
                                 nn.Dropout(dropout), nn.Linear(ffn_dim, d_model, bias=False),
                                 nn.Dropout(dropout))

    def forward(self, x, key_padding_mask=None):
        h = self.norm1(x)
        x = x + self.attn(h, h, h, key_padding_mask=key_padding_mask)
        return x + self.ffn(self.norm2(x))


class OracleLM(nn.Module):
    """multiscreen/model.py:12-141, including the recompute-everything
    generate() (model.py:111-141)."""

    def __init__(self, vocab_size, d_model=512, num_heads=8, num_layers=6, ffn_dim=None,
                 max_seq_len=2048, dropout=0.0, tie_weights=True, windowed=False):
        super().__init__()
        self.token_emb = nn.Embedding(vocab_size, d_model)
        self.pos_emb = nn.Embedding(max_seq_len, d_model)
        self.blocks = nn.ModuleList([OracleBlock(d_model, num_heads, ffn_dim, dropout, True,
                                                 windowed) for _ in range(num_layers)])
        self.norm = nn.RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.token_emb.weight

    def forward(self, input_ids, key_padding_mask=None, labels=None):
        B, T = input_ids.shape
        pos = torch.arange(T, device=input_ids.device).unsqueeze(0)
        x = self.token_emb(input_ids) + self.pos_emb(pos)
        for blk in self.blocks:
            x = blk(x, key_padding_mask=key_padding_mask)
        logits = self.lm_head(self.norm(x))
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.view(-1, logits.size(-1)), labels.view(-1),
                                          ignore_index=-100)
        return out

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=100, temperature=1.0, top_k=None):
        self.eval()
        for _ in range(max_new_tokens):
            logits = self(input_ids)["logits"][:, -1, :] / temperature
            if top_k is not None:
                values, _ = torch.topk(logits, top_k)
                logits[logits < values[:, -1:]] = float("-inf")
            nxt = torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)
            input_ids = torch.cat([input_ids, nxt], dim=1)
        return input_ids


def param_grads_reference(q, k, v, r, w, causal=True, key_padding_mask=None, eps=1e-8,
                          dy=None, q_offset=0, dtype=torch.float64):
    """Run screening_core under autograd (CPU, `dtype`) and return
    (y, dq, dk, dv, dr, dw) for the cotangent dy (default: ones)."""
    q = q.detach().to(dtype).requires_grad_(True)
    k = k.detach().to(dtype).requires_grad_(True)
    v = v.detach().to(dtype).requires_grad_(True)
    r = r.detach().to(dtype).requires_grad_(True)
    w = w.detach().to(dtype).requires_grad_(True)
    y = screening_core(q, k, v, r, w, causal, key_padding_mask, eps, q_offset)
    g = torch.ones_like(y) if dy is None else dy.to(dtype)
    y.backward(g)
    return y.detach(), q.grad, k.grad, v.grad, r.grad, w.grad


def windowed_core_grads(q, k, v, r, w, dy, causal=True, q_offset=0, eps=1e-8, chunk=256,
                        dtype=torch.float64):
    """(y, dq, dk, dv, dr, dw) of screening_core for the cotangent dy, with
    bounded memory at long T: the loss sum(y * dy) is a sum over query rows,
    and row i depends on q_i and on the keys inside its window only
    (multiscreen/attention.py:156-196, mask exactly zero outside the window,
    attention.py:117-118), so each block of `chunk` query rows runs forward
    and backward on its own against its key range and the gradients of k, v,
    r and w are summed over the blocks.  Inputs (B, T, H, D) on the CPU."""
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    dmax = int(math.ceil(float(w.detach().max()))) - 1 if H > 0 else -1
    qd, kd, vd, dyd = (t.detach().to(dtype) for t in (q, k, v, dy))
    rd = r.detach().to(dtype).requires_grad_(True)
    wd = w.detach().to(dtype).requires_grad_(True)
    y = torch.zeros(B, Tq, H, D, dtype=dtype)
    dq = torch.zeros_like(qd)
    dk = torch.zeros_like(kd)
    dv = torch.zeros_like(vd)
    for i0 in range(0, Tq, chunk):
        i1 = min(Tq, i0 + chunk)
        p0, p1 = i0 + q_offset, i1 - 1 + q_offset
        lo = max(0, p0 - dmax)
        hi = min(Tk - 1, p1 if causal else p1 + dmax)
        if hi < lo or dmax < 0:
            continue
        qc = qd[:, i0:i1].clone().requires_grad_(True)
        kc = kd[:, lo:hi + 1].clone().requires_grad_(True)
        vc = vd[:, lo:hi + 1].clone().requires_grad_(True)
        # the block's query i sits at key-axis position i + q_offset, i.e.
        # (i - i0) + (p0 - lo) inside the key slice
        yc = screening_core(qc, kc, vc, rd, wd, causal, None, eps, q_offset=p0 - lo)
        yc.backward(dyd[:, i0:i1])
        y[:, i0:i1] = yc.detach()
        dq[:, i0:i1] = qc.grad
        dk[:, lo:hi + 1] += kc.grad
        dv[:, lo:hi + 1] += vc.grad
    dr = rd.grad if rd.grad is not None else torch.zeros_like(rd)
    dw = wd.grad if wd.grad is not None else torch.zeros_like(wd)
    return y, dq, dk, dv, dr.detach(), dw.detach()
