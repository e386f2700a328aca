"""MultiscreenLM on the B200 kernels -- drop-in for multiscreen/model.py:12-141.

forward() keeps the reference signature and result dict.  generate() keeps
the reference signature and sampling (temperature, top-k, softmax,
multinomial; model.py:131-140) but replaces the full-prefix recompute per
token (model.py:133) by one prefill pass plus a KV-cached single-token decode
per step, computing logits for the last position only.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .functional import cross_entropy, rms_eps, rms_norm
from .kv_cache import PagedKVCache
from .layers import MultiscreenBlock
from .sequence_parallel import current_shard


def _sharded_mean_ce(logits, labels, shard):
    """Mean cross-entropy over the tokens of all ranks (model.py:103-107 on the
    whole sequence).  Its value is the global mean on every rank; its gradient
    is this rank's tokens' share only, so summing the parameter gradients over
    the ranks (as data parallelism does) gives the full gradient."""
    import torch.distributed as dist
    lg = logits.reshape(-1, logits.size(-1))
    if lg.dtype in (torch.float16, torch.bfloat16):
        lg = lg.float()
    s = F.cross_entropy(lg, labels.reshape(-1), ignore_index=-100, reduction="sum")
    tot = torch.stack([s.detach(), (labels != -100).sum().to(s.dtype)])
    dist.all_reduce(tot, group=shard.group)
    return (s + (tot[0] - s.detach())) / tot[1]


_rms_eps = rms_eps


class MultiscreenLM(nn.Module):
    def __init__(self, vocab_size: int, d_model: int = 512, num_heads: int = 8,
                 num_layers: int = 6, ffn_dim: int | None = None, max_seq_len: int = 2048,
                 dropout: float = 0.0, tie_weights: bool = True):
        super().__init__()
        self.d_model = d_model
        self.token_emb = nn.Embedding(vocab_size, d_model)
        self.pos_emb = nn.Embedding(max_seq_len, d_model)
        self.emb_dropout = nn.Dropout(dropout)
        self.blocks = nn.ModuleList([
            MultiscreenBlock(d_model=d_model, num_heads=num_heads, ffn_dim=ffn_dim,
                             dropout=dropout, causal=True)
            for _ in range(num_layers)
        ])
        self.norm = nn.RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.token_emb.weight
        self._init_weights()

    def _init_weights(self):
        """model.py:62-69: N(0, 0.02) for embeddings and every Linear."""
        nn.init.normal_(self.token_emb.weight, std=0.02)
        nn.init.normal_(self.pos_emb.weight, std=0.02)
        for module in self.modules():
            if isinstance(module, nn.Linear):
                nn.init.normal_(module.weight, std=0.02)

    def forward(self, input_ids: torch.Tensor, key_padding_mask: torch.Tensor | None = None,
                labels: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        B, T = input_ids.shape
        shard = current_shard()
        off = shard.start if shard is not None else 0
        positions = torch.arange(off, off + T, device=input_ids.device).unsqueeze(0)
        x = self.emb_dropout(self.token_emb(input_ids) + self.pos_emb(positions))
        for block in self.blocks:
            x = block(x, key_padding_mask=key_padding_mask)
        x = rms_norm(self.norm, x)
        logits, lpad = self._lm_logits(x)
        result = {"logits": logits}
        if labels is not None:
            # model.py:103-107 on the padded logits (pad columns are -inf)
            if shard is None or shard.world == 1:
                result["loss"] = cross_entropy(lpad.reshape(-1, lpad.size(-1)),
                                               labels.reshape(-1), ignore_index=-100)
            else:
                result["loss"] = _sharded_mean_ce(lpad, labels, shard)
        return result

    # ------------------------------------------------------------------
    def _lm_logits(self, x: torch.Tensor):
        """lm_head(x) over all positions.  The vocabulary (50257 for GPT-2) is
        padded to a multiple of 64 for the GEMM: with an odd leading dimension
        cuBLAS falls back to unaligned kernels several times slower.  The pad
        columns get logit -inf (zero weight rows, -inf bias), so softmax and
        cross-entropy over the padded logits equal those over the real ones.
        Returns (logits (..., V) -- a view --, padded logits (..., Vp))."""
        W = self.lm_head.weight
        V = W.shape[0]
        pad = (-V) % 64
        if pad == 0 or not x.is_cuda:
            lg = self.lm_head(x)
            return lg, lg
        if torch.is_autocast_enabled("cuda"):
            W = W.to(torch.get_autocast_dtype("cuda"))
        Wp = F.pad(W, (0, 0, 0, pad))
        bias = torch.zeros(V + pad, dtype=Wp.dtype, device=x.device)
        bias[V:] = float("-inf")
        lp = F.linear(x, Wp, bias)
        return lp[..., :V], lp

    def _max_window(self) -> float:
        ws = torch.cat([blk.attn.window().detach() for blk in self.blocks])
        return float(ws.max()) if ws.numel() else 0.0

    def make_cache(self, batch: int, max_len: int, dtype: torch.dtype | None = None,
                   page_size: int = 64) -> PagedKVCache:
        a0 = self.blocks[0].attn
        dt = dtype or self.token_emb.weight.dtype
        if dt not in (torch.float32, torch.bfloat16):
            dt = torch.float32
        return PagedKVCache(len(self.blocks), batch, a0.num_heads, a0.head_dim, max_len,
                            self._max_window(), dt, self.token_emb.weight.device, page_size)

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, cache: PagedKVCache | None) -> torch.Tensor:
        """Run the prompt once, fill `cache` (if given), return the logits of
        the last position (B,V).  Inside sequence_parallel(), input_ids is this
        rank's block of the prompt and the logits are those of the block's last
        position (the prompt's last on the last rank)."""
        B, T = input_ids.shape
        shard = current_shard()
        off = shard.start if shard is not None else 0
        positions = torch.arange(off, off + T, device=input_ids.device).unsqueeze(0)
        x = self.emb_dropout(self.token_emb(input_ids) + self.pos_emb(positions))
        for li, blk in enumerate(self.blocks):
            x = x + blk.attn.prefill(x, cache, li, norm=blk.norm1)
            x = x + blk.ffn(rms_norm(blk.norm2, x))
        return self.lm_head(rms_norm(self.norm, x[:, -1:].contiguous()))[:, -1]

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, position, cache: PagedKVCache,
                    state: dict | None = None) -> torch.Tensor:
        """tokens (B,1) at absolute `position` (an int, or an int32 (B,) device
        tensor); returns logits (B,V).  With a tensor position the step has no
        host-side dependence on the position, so it can be captured once in a
        CUDA graph and replayed for every generated token."""
        B = tokens.shape[0]
        dev = tokens.device
        if state is None:
            state = self._decode_state()
        if isinstance(position, torch.Tensor):
            pos_t = position
        else:
            pos_t = torch.full((B,), position, dtype=torch.int32, device=dev)
        x = self.token_emb(tokens) + self.pos_emb(pos_t.long()).unsqueeze(1)
        seq_lens = pos_t + 1
        if self._rows_fast(x):
            # few tokens: every linear layer is one bandwidth-bound pass over
            # its weights with RMSNorm, GELU and the residual add fused in
            d = self.d_model
            h = x.reshape(B, d)
            for li, blk in enumerate(self.blocks):
                wqkv, r, w = state["layers"][li]
                qkv = _lib.rows_linear(h, wqkv, norm_w=blk.norm1.weight, eps=_rms_eps(blk.norm1, h))
                y = blk.attn.decode_attend(qkv, cache, li, pos_t, seq_lens, r, w)
                h = _lib.rows_linear(y, blk.attn.out_proj.weight, res=h)
                u = _lib.rows_linear(h, blk.ffn[0].weight, norm_w=blk.norm2.weight,
                                     eps=_rms_eps(blk.norm2, h), act=1)
                h = _lib.rows_linear(u, blk.ffn[3].weight, res=h)
            return _lib.rows_linear(h, self.lm_head.weight, norm_w=self.norm.weight,
                                    eps=_rms_eps(self.norm, h))
        for li, blk in enumerate(self.blocks):
            wqkv, r, w = state["layers"][li]
            x = x + blk.attn.decode_step(blk.norm1(x), cache, li, pos_t, seq_lens, wqkv, r, w)
            x = x + blk.ffn(blk.norm2(x))
        return self.lm_head(self.norm(x))[:, -1]

    def _rows_fast(self, x: torch.Tensor) -> bool:
        """The fused few-row decode path applies: bf16 CUDA weights and
        activations, at most 8 tokens, feature sizes multiples of 8, exact
        GELU FFN without bias, RMSNorm with an affine weight."""
        if not (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[0] <= 8):
            return False
        if self.lm_head.weight.dtype != torch.bfloat16 or self.d_model % 8:
            return False
        for blk in self.blocks:
            f = blk.ffn
            if not (isinstance(f[0], nn.Linear) and isinstance(f[1], nn.GELU) and
                    f[1].approximate == "none" and f[0].bias is None and f[3].bias is None and
                    f[0].out_features % 8 == 0 and blk.norm1.weight is not None and
                    blk.norm2.weight is not None and blk.attn.out_proj.bias is None):
                return False
        return self.norm.weight is not None

    @torch.no_grad()
    def _capture_decode(self, batch: int, first_position: int, cache: PagedKVCache,
                        state: dict):
        """One decode step (every layer + lm_head) captured in a CUDA graph with
        static inputs `tokens` (B,1) and `pos` (B,) int32.  The warm-up steps
        run at `first_position`, whose cache slot the first real step
        overwrites before reading it."""
        dev = self.token_emb.weight.device
        tokens = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        pos = torch.full((batch,), first_position, dtype=torch.int32, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                self.decode_step(tokens, pos, cache, state)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits = self.decode_step(tokens, pos, cache, state)
        return graph, tokens, pos, logits

    def _decode_state(self) -> dict:
        layers = []
        for blk in self.blocks:
            a = blk.attn
            wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)
            layers.append((wqkv, a.sharpness().contiguous(), a.window().contiguous()))
        return {"layers": layers}

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100,
                 temperature: float = 1.0, top_k: int | None = None,
                 cuda_graph: bool = True) -> torch.Tensor:
        """(B,T) prompt -> (B, T + max_new_tokens), sampling as model.py:134-140.
        On CUDA the per-token decode step is one CUDA-graph replay
        (`cuda_graph=False`: eager launches, same numbers)."""
        self.eval()
        if max_new_tokens <= 0:
            return input_ids
        B, T0 = input_ids.shape
        if T0 + max_new_tokens - 1 > self.pos_emb.num_embeddings:
            # the reference fails the same way inside pos_emb (model.py:90-92)
            raise IndexError("index out of range in self: prompt + new tokens exceed max_seq_len")
        cache = self.make_cache(B, T0 + max_new_tokens)
        state = self._decode_state()
        logits = self.prefill(input_ids, cache)
        graph = None
        if cuda_graph and input_ids.is_cuda and max_new_tokens > 1:
            graph, g_tok, g_pos, g_logits = self._capture_decode(B, T0, cache, state)
        for step in range(max_new_tokens):
            logits = logits / temperature
            if top_k is not None:
                values, _ = torch.topk(logits, top_k)
                logits[logits < values[:, -1:]] = float("-inf")
            probs = F.softmax(logits, dim=-1)
            next_token = torch.multinomial(probs, num_samples=1)
            input_ids = torch.cat([input_ids, next_token], dim=1)
            if step + 1 < max_new_tokens:
                if graph is not None:
                    g_tok.copy_(next_token)
                    g_pos.fill_(T0 + step)
                    graph.replay()
                    logits = g_logits.clone()
                else:
                    logits = self.decode_step(next_token, T0 + step, cache, state)
        return input_ids
