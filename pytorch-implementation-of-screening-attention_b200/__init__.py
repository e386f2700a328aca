"""B200-native Screening Attention ("Screening Is Enough", arXiv:2604.01178).

Drop-in for the `multiscreen` package's public API (multiscreen/__init__.py:
ScreeningAttention, MultiscreenBlock, MultiscreenDecoderLayer, MultiscreenLM,
TanhNorm) with the attention hot path in hand-written sm_100a CUDA behind a
C ABI (include/screening_b200.h).  The directory name is not a Python
identifier, so import it with importlib; on import it also registers itself
as `screening_b200`:

    import importlib
    ms = importlib.import_module("pytorch-implementation-of-screening-attention_b200")
    attn = ms.ScreeningAttention(512, 8).cuda()
"""
import sys as _sys

from .attention import ScreeningAttention
from .functional import ScreenFn, ScreenPackedFn, screening_attention, screening_attention_packed, tanh_norm
from .kv_cache import PagedKVCache
from .layers import MultiscreenBlock, MultiscreenDecoderLayer
from .model import MultiscreenLM
from .norm import TanhNorm
from .sequence_parallel import (SequenceShard, current_shard, screening_attention_sharded,
                                sequence_parallel, shard_timeline, shard_timeline_summary)
from . import _lib

_sys.modules.setdefault("screening_b200", _sys.modules[__name__])

__all__ = [
    "ScreeningAttention",
    "MultiscreenBlock",
    "MultiscreenDecoderLayer",
    "MultiscreenLM",
    "TanhNorm",
    "ScreenFn",
    "screening_attention",
    "tanh_norm",
    "PagedKVCache",
    "sequence_parallel",
    "shard_timeline",
    "shard_timeline_summary",
    "screening_attention_sharded",
    "SequenceShard",
]

__version__ = "0.1.0"
