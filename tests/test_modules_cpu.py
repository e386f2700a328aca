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


def test_dropout_only_in_training(ms):
    a = ms.ScreeningAttention(64, 4, dropout=0.25)
    assert a.train()._dropout_p() == 0.25
    assert a.eval()._dropout_p() == 0.0
    assert ms.ScreeningAttention(64, 4).train()._dropout_p() == 0.0


def test_dropout_bits_oracle_matches_library(ms, oracle):
    """The oracle's restatement of the counter-based dropout hash equals the
    library's screen_dropout_bits (host function, no GPU needed)."""
    from importlib import import_module
    lib = import_module("pytorch-implementation-of-screening-attention_b200._lib")
    g = torch.Generator().manual_seed(3)
    seeds = [0, 1, 2**32 - 1, 2**32, 0x0123456789ABCDEF, 2**64 - 1]
    idx = torch.randint(0, 2**31 - 1, (40, 3), generator=g)
    idx[:4] = torch.tensor([[0, 0, 0], [1, 2, 3], [2**31 - 2, 2**31 - 2, 2**31 - 2], [7, 0, 9]])
    for seed in seeds:
        bits = oracle.dropout_bits(seed, idx[:, 0], idx[:, 1], idx[:, 2])
        for (bh, i, j), got in zip(idx.tolist(), bits.tolist()):
            assert got == lib.dropout_bits(seed, bh, i, j)


def test_dropout_mask_statistics(oracle):
    """Drop rate equals p; masks of neighbouring scores, rows and seeds are
    uncorrelated (Bernoulli statistics on 2^20 scores, 5-sigma bounds)."""
    from importlib import import_module
    lib = import_module("pytorch-implementation-of-screening-attention_b200._lib")
    n = 1024
    i = torch.arange(n)
    j = torch.arange(n)
    for p in (0.1, 0.5, 0.9):
        thr = lib.dropout_threshold(p)
        keep = oracle.dropout_keep(1234, thr, 1, 1, i, j)[0, 0] > 0
        rate = 1.0 - keep.double().mean().item()
        sd = math.sqrt(p * (1 - p) / (n * n))
        assert abs(rate - p) < 5 * sd, (p, rate)
        k = keep.double() - keep.double().mean()
        den = (k * k).mean().item()
        for a, b in ((k[:, 1:], k[:, :-1]), (k[1:, :], k[:-1, :])):
            corr = (a * b).mean().item() / den
            assert abs(corr) < 5 / n, corr
    k1 = oracle.dropout_keep(1, lib.dropout_threshold(0.5), 2, 3, i[:256], j[:256]) > 0
    k2 = oracle.dropout_keep(2, lib.dropout_threshold(0.5), 2, 3, i[:256], j[:256]) > 0
    agree = (k1 == k2).double().mean().item()
    assert abs(agree - 0.5) < 5 * math.sqrt(0.25 / k1.numel())
    # different (b, h) planes of one seed differ too
    assert (k1[0, 0] != k1[1, 2]).any()


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


def test_head_params_and_col_scale_host_forms(ms):
    """The module's r / w transforms and the folded norm weight give the
    reference's formulas (attention.py:164-165; RMSNorm weight times the
    projection's columns) when no kernel can run (CPU parameters)."""
    a = ms.ScreeningAttention(64, 4)
    with torch.no_grad():
        a.s_r.copy_(torch.tensor([-1.0, 0.0, 0.5, 2.0]))
    r, w = a._head_params()
    torch.testing.assert_close(r, torch.exp(a.s_r) + 1.0)
    torch.testing.assert_close(w, torch.exp(a.s_v) + 1.0)
    torch.testing.assert_close(r, a.sharpness())
    g = torch.rand(64) + 0.5
    wq = a._wqkv(g)
    ref = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0) * g
    torch.testing.assert_close(wq, ref)
    assert a._wqkv().shape == (192, 64)


def test_absorbed_norm_rejects_cross_attention(ms):
    a = ms.ScreeningAttention(64, 4)
    x, m = torch.randn(1, 3, 64), torch.randn(1, 5, 64)
    with pytest.raises(ValueError):
        a._qkv(x, m, m, torch.ones(64))
