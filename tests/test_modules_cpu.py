"""Host-side module behaviour that needs no GPU: constructors, parameter
names and init identical to the reference (so checkpoints load), and no
silent CPU fallback."""
import math

import pytest
import torch

from tests.helpers import golden_module

MG = golden_module()


def test_state_dict_keys_match_reference_layout(ms, oracle):
    a = ms.ScreeningAttention(64, 4)
    o = oracle.OracleScreeningAttention(64, 4)
    assert list(a.state_dict()) == list(o.state_dict())
    torch.testing.assert_close(a.s_v, torch.linspace(0, math.log(255), 4))
    assert torch.all(a.s_r == 0)
    assert hasattr(a, "tahn_norm")


def test_same_seed_same_init_as_reference_construction(ms, oracle, golden):
    """ScreeningAttention(512, 8) under manual_seed(0) draws the reference's
    weights (the cfg1 fixture's checksum)."""
    attn, x, _ = MG.cfg1_inputs(ms.ScreeningAttention)
    assert sum(MG.checksum(p) for p in attn.parameters()) == pytest.approx(
        golden["cfg1"]["w_checksum"], rel=1e-9)


def test_lm_loads_reference_state_dict(ms, golden):
    rec = golden["lm"]["lm_d16"]
    spec = rec["spec"]
    m = ms.MultiscreenLM(spec["vocab"], spec["d_model"], spec["H"], spec["L"], spec["ffn"],
                         spec["max_seq_len"])
    missing, unexpected = m.load_state_dict(rec["state"], strict=True)
    assert not missing and not unexpected
    assert m.lm_head.weight is m.token_emb.weight


def test_decoder_layer_names(ms):
    layer = ms.MultiscreenDecoderLayer(64, 4)
    keys = set(layer.state_dict())
    assert {"self_attn.s_v", "cross_attn.s_r", "norm3.weight", "ffn.3.weight"} <= keys
    assert layer.cross_attn.causal is False


def test_cpu_tensors_raise_instead_of_falling_back(ms):
    a = ms.ScreeningAttention(64, 4)
    x = torch.randn(1, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        a(x, x, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        ms.TanhNorm()(torch.randn(2, 8))


def test_dropout_training_is_refused(ms):
    a = ms.ScreeningAttention(64, 4, dropout=0.1).train()
    x = torch.randn(1, 8, 64)
    with pytest.raises(NotImplementedError):
        a(x, x, x)


def test_kv_cache_ring_layout(ms):
    c = ms.PagedKVCache(2, 3, 4, 16, max_len=1000, max_window=100.0, dtype=torch.float32,
                        device=torch.device("cpu"), page_size=32)
    assert c.keep == 100
    assert c.pages_per_seq == math.ceil(100 / 32) + 1
    t = c.block_table
    # any `keep` consecutive positions map to distinct pages of the sequence's own set
    for b in range(3):
        for start in range(0, 1000 - c.keep, 7):
            blocks = range(start // 32, (start + c.keep - 1) // 32 + 1)
            pages = [int(t[b, lb]) for lb in blocks]
            assert len(set(pages)) == len(pages)
            assert all(b * c.pages_per_seq <= p < (b + 1) * c.pages_per_seq for p in pages)
