"""Pin the CPU oracle (oracle/screening_oracle.py) to the reference's own
outputs recorded in tests/golden/golden.pt by tests/golden/make_golden.py."""
import math

import pytest
import torch

from tests.conftest import rel_err
from tests.helpers import golden_module

MG = golden_module()


def _core_case(oracle, rec):
    spec = rec["spec"]
    inp = MG.case_inputs(spec)
    chk = MG.checksum(inp["q"]) + MG.checksum(inp["k"]) + MG.checksum(inp["v"])
    assert chk == pytest.approx(rec["in_checksum"], rel=1e-9)
    B, Tq, Tk, H, D = spec["B"], spec["Tq"], spec["Tk"], spec["H"], spec["D"]
    q = inp["q"].view(B, Tq, H, D).clone().requires_grad_(True)
    k = inp["k"].view(B, Tk, H, D).clone().requires_grad_(True)
    v = inp["v"].view(B, Tk, H, D).clone().requires_grad_(True)
    s_r = inp["s_r"].clone().requires_grad_(True)
    s_v = inp["s_v"].clone().requires_grad_(True)
    r = torch.exp(s_r) + 1.0
    w = torch.exp(s_v) + 1.0
    return inp, (q, k, v, s_r, s_v, r, w)


@pytest.mark.parametrize("name", list(MG.ATTN_CASES))
@pytest.mark.parametrize("windowed", [False, True])
def test_core_matches_reference(oracle, golden, name, windowed):
    rec = golden["attention"][name]
    spec = rec["spec"]
    inp, (q, k, v, s_r, s_v, r, w) = _core_case(oracle, rec)
    if windowed:
        y = oracle.screening_core_windowed(q, k, v, r, w, spec["causal"], inp["kpm"], 1e-8,
                                           chunk=16)
    else:
        y = oracle.screening_core(q, k, v, r, w, spec["causal"], inp["kpm"], 1e-8)
    y = y.reshape(spec["B"], spec["Tq"], -1)
    (y * inp["cot"]).sum().backward()
    assert rel_err(y, rec["y"]) < 1e-5
    assert rel_err(q.grad.reshape_as(rec["dq"]), rec["dq"]) < 1e-4
    assert rel_err(k.grad.reshape_as(rec["dk"]), rec["dk"]) < 1e-4
    assert rel_err(v.grad.reshape_as(rec["dv"]), rec["dv"]) < 1e-4
    torch.testing.assert_close(s_r.grad, rec["ds_r"], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(s_v.grad, rec["ds_v"], rtol=1e-4, atol=1e-6)


def test_cfg1_module_matches_reference(oracle, golden):
    rec = golden["cfg1"]
    attn, x, cot = MG.cfg1_inputs(oracle.OracleScreeningAttention)
    assert MG.checksum(x) == pytest.approx(rec["x_checksum"], rel=1e-9)
    assert sum(MG.checksum(p) for p in attn.parameters()) == pytest.approx(rec["w_checksum"],
                                                                          rel=1e-9)
    xr = x.clone().requires_grad_(True)
    out = attn(xr, xr, xr)
    (out * cot).sum().backward()
    assert rel_err(out[:, ::8], rec["y_rows"]) < 1e-5
    assert rel_err(xr.grad[:, ::8], rec["dx_rows"]) < 1e-4
    probe = torch.randn(rec["spec"]["d_model"], generator=torch.Generator().manual_seed(99))
    for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
        gw = getattr(attn, name).weight.grad
        assert rel_err(gw @ probe, rec[f"{name}_grad_probe"]) < 1e-4
        assert gw.norm().item() == pytest.approx(rec[f"{name}_grad_norm"].item(), rel=1e-4)
    torch.testing.assert_close(attn.s_r.grad, rec["ds_r"], rtol=1e-3, atol=1e-7)
    torch.testing.assert_close(attn.s_v.grad, rec["ds_v"], rtol=1e-3, atol=1e-7)


@pytest.mark.parametrize("name", list(MG.LM_CASES))
def test_lm_matches_reference(oracle, golden, name):
    rec = golden["lm"][name]
    spec = rec["spec"]
    model = oracle.OracleLM(spec["vocab"], spec["d_model"], spec["H"], spec["L"], spec["ffn"],
                            spec["max_seq_len"])
    model.load_state_dict(rec["state"])
    ids, labels, prompt = _ids(spec)
    out = model(ids, labels=labels)
    assert rel_err(out["logits"], rec["logits"]) < 1e-5
    assert out["loss"].item() == pytest.approx(rec["loss"].item(), rel=1e-5)
    out["loss"].backward()
    for li, blk in enumerate(model.blocks):
        torch.testing.assert_close(blk.attn.s_r.grad, rec["s_r_grad"][li], rtol=1e-3, atol=1e-8)
        torch.testing.assert_close(blk.attn.s_v.grad, rec["s_v_grad"][li], rtol=1e-3, atol=1e-8)
    toks = model.generate(prompt, max_new_tokens=spec["new"], top_k=1)
    assert torch.equal(toks, rec["tokens"])


def _ids(spec):
    """The id/label/prompt tensors of make_golden.lm_inputs (same generator)."""
    g = torch.Generator().manual_seed(spec["seed"] + 1000)
    ids = torch.randint(0, spec["vocab"], (spec["B"], spec["T"]), generator=g)
    labels = ids.clone()
    labels[:, :3] = -100
    prompt = torch.randint(0, spec["vocab"], spec["prompt"], generator=g)
    return ids, labels, prompt


@pytest.mark.parametrize("causal", [True, False])
def test_windowed_equals_dense_larger(oracle, causal):
    g = torch.Generator().manual_seed(5)
    B, T, H, D = 1, 300, 3, 16
    q = torch.randn(B, T, H, D, generator=g)
    k = q + 0.5 * torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    r = torch.tensor([1.1, 1.5, 2.0])
    w = torch.tensor([5.5, 40.0, 130.0])
    a = oracle.screening_core(q, k, v, r, w, causal)
    b = oracle.screening_core_windowed(q, k, v, r, w, causal, chunk=64)
    assert rel_err(b, a) < 1e-6


def test_q_offset_is_a_shifted_slice(oracle):
    """Queries at key-axis offset o over all keys equal the last rows of the
    full self-attention -- the identity sequence-sharded prefill relies on."""
    g = torch.Generator().manual_seed(6)
    B, T, H, D = 1, 64, 2, 16
    x = torch.randn(B, T, H, D, generator=g)
    k = x + 0.3 * torch.randn(B, T, H, D, generator=g)
    v = torch.randn(B, T, H, D, generator=g)
    r = torch.tensor([1.2, 1.6])
    w = torch.tensor([9.0, 30.0])
    full = oracle.screening_core(x, k, v, r, w, True)
    part = oracle.screening_core(x[:, 40:], k, v, r, w, True, q_offset=40)
    assert rel_err(part, full[:, 40:]) < 1e-6
