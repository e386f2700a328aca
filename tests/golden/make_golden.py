"""Generate golden vectors from the reference `multiscreen` package.

Run once in a checkout that has the reference source tree:

    python tests/golden/make_golden.py --reference <path to the reference repo>

It imports the reference's own ScreeningAttention / MultiscreenLM
(multiscreen/attention.py, multiscreen/model.py), runs seeded cases on CPU in
fp32 and writes tests/golden/golden.pt: inputs are regenerated from their
seeds by the tests (a checksum guards the regeneration), outputs and
gradients are stored.  The reference itself never runs at test time.

Attention cases use identity projections (q_proj = k_proj = v_proj =
out_proj = I), so the module output is exactly the screening core
y = TanhNorm(alpha v^) on the raw inputs and the input gradients are the
core's dq, dk, dv.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def case_inputs(spec: dict) -> dict:
    """Seeded inputs of an attention case.  Shared with the tests."""
    g = torch.Generator().manual_seed(spec["seed"])
    B, Tq, Tk, H, D = spec["B"], spec["Tq"], spec["Tk"], spec["H"], spec["D"]
    q = torch.randn(B, Tq, H * D, generator=g)
    k = torch.randn(B, Tk, H * D, generator=g)
    v = torch.randn(B, Tk, H * D, generator=g)
    corr = spec.get("corr", 0.0)
    if corr:
        # keys close to queries -> many scores clear the trim threshold
        n = min(Tq, Tk)
        k[:, :n] = q[:, :n] + corr * k[:, :n]
    for (b, t) in spec.get("zero_q_rows", []):
        q[b, t] = 0.0
    for (b, t) in spec.get("zero_k_rows", []):
        k[b, t] = 0.0
        v[b, t] = 0.0
    s_v = torch.tensor(spec["s_v"], dtype=torch.float32)
    s_r = torch.tensor(spec["s_r"], dtype=torch.float32)
    kpm = None
    if spec.get("kpm"):
        kpm = torch.zeros(B, Tk, dtype=torch.bool)
        for (b, lo, hi) in spec["kpm"]:
            kpm[b, lo:hi] = True
    cot = torch.randn(B, Tq, H * D, generator=g)
    return dict(q=q, k=k, v=v, s_v=s_v, s_r=s_r, kpm=kpm, cot=cot)


def checksum(t: torch.Tensor) -> float:
    return float(t.detach().double().abs().sum())


ATTN_CASES = {
    "causal_d16": dict(seed=1, B=2, Tq=48, Tk=48, H=4, D=16, causal=True,
                       s_v=[0.0, 1.5, 3.0, math.log(255)], s_r=[0.0, -1.0, -2.0, 0.5]),
    "causal_d64_ragged": dict(seed=2, B=2, Tq=70, Tk=70, H=2, D=64, causal=True, corr=0.6,
                              s_v=[math.log(19.0), math.log(80.0)], s_r=[math.log(0.2), 0.0]),
    "causal_d32_corr": dict(seed=3, B=1, Tq=40, Tk=40, H=2, D=32, causal=True, corr=0.3,
                            s_v=[math.log(7.5), math.log(500.0)], s_r=[-3.0, 0.3]),
    "noncausal_cross": dict(seed=4, B=2, Tq=8, Tk=20, H=4, D=16, causal=False, corr=0.5,
                            s_v=[0.0, 1.0, 2.0, 3.0], s_r=[-1.0, -1.0, -2.0, 0.0]),
    "noncausal_self_d64": dict(seed=5, B=1, Tq=36, Tk=36, H=2, D=64, causal=False, corr=0.5,
                               s_v=[math.log(9.0), math.log(40.0)], s_r=[math.log(0.3), -2.0]),
    "key_padding": dict(seed=6, B=2, Tq=33, Tk=33, H=2, D=16, causal=True, corr=0.5,
                        s_v=[math.log(15.0), math.log(60.0)], s_r=[-1.0, -2.0],
                        kpm=[(0, 28, 33), (1, 0, 33)]),
    "zero_rows_eps": dict(seed=7, B=1, Tq=24, Tk=24, H=2, D=16, causal=True, corr=0.5,
                          s_v=[math.log(5.0), math.log(30.0)], s_r=[-1.5, -0.5],
                          zero_q_rows=[(0, 3), (0, 10)], zero_k_rows=[(0, 5)]),
    "window_extremes": dict(seed=8, B=1, Tq=40, Tk=40, H=3, D=16, causal=True, corr=0.5,
                            s_v=[-9.0, math.log(1000.0), math.log(0.5)],
                            s_r=[-6.0, -1.0, -1.0]),
}

# cfg1 of the benchmark list: ScreeningAttention(512, 8) default init, B=2, T=128
CFG1 = dict(seed=0, B=2, T=128, d_model=512, H=8)

LM_CASES = {
    "lm_d16": dict(seed=11, vocab=50, d_model=64, H=4, L=2, ffn=64, max_seq_len=32, B=2, T=16,
                   prompt=(1, 4), new=8),
    "lm_d64": dict(seed=12, vocab=67, d_model=128, H=2, L=1, ffn=128, max_seq_len=48, B=2, T=40,
                   prompt=(2, 12), new=10),
}


def run_attention_case(ms, spec: dict) -> dict:
    inp = case_inputs(spec)
    H, D = spec["H"], spec["D"]
    d = H * D
    attn = ms.ScreeningAttention(d_model=d, num_heads=H, causal=spec["causal"])
    with torch.no_grad():
        for lin in (attn.q_proj, attn.k_proj, attn.v_proj, attn.out_proj):
            lin.weight.copy_(torch.eye(d))
        attn.s_v.copy_(inp["s_v"])
        attn.s_r.copy_(inp["s_r"])
    q = inp["q"].clone().requires_grad_(True)
    k = inp["k"].clone().requires_grad_(True)
    v = inp["v"].clone().requires_grad_(True)
    out = attn(q, k, v, key_padding_mask=inp["kpm"])
    (out * inp["cot"]).sum().backward()
    return dict(spec=spec, in_checksum=checksum(inp["q"]) + checksum(inp["k"]) + checksum(inp["v"]),
                y=out.detach(), dq=q.grad, dk=k.grad, dv=v.grad,
                ds_r=attn.s_r.grad.clone(), ds_v=attn.s_v.grad.clone())


def cfg1_inputs(ms_attention_cls, spec=CFG1):
    """Module + input + cotangent of cfg1 from the seed (module built first,
    exactly as `torch.manual_seed(seed); Cls(512, 8)`)."""
    torch.manual_seed(spec["seed"])
    attn = ms_attention_cls(spec["d_model"], spec["H"])
    x = torch.randn(spec["B"], spec["T"], spec["d_model"])
    cot = torch.randn(spec["B"], spec["T"], spec["d_model"])
    return attn, x, cot


def run_cfg1(ms) -> dict:
    attn, x, cot = cfg1_inputs(ms.ScreeningAttention)
    xr = x.clone().requires_grad_(True)
    out = attn(xr, xr, xr)
    (out * cot).sum().backward()
    g = torch.Generator().manual_seed(99)
    probe = torch.randn(CFG1["d_model"], generator=g)
    res = dict(spec=CFG1, x_checksum=checksum(x),
               w_checksum=sum(checksum(p) for p in attn.parameters()),
               y_rows=out.detach()[:, ::8].clone(), dx_rows=xr.grad[:, ::8].clone(),
               ds_r=attn.s_r.grad.clone(), ds_v=attn.s_v.grad.clone(), probe_seed=99)
    for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
        gw = getattr(attn, name).weight.grad
        res[f"{name}_grad_probe"] = gw @ probe
        res[f"{name}_grad_norm"] = gw.norm()
    return res


def lm_inputs(ms_lm_cls, spec):
    torch.manual_seed(spec["seed"])
    model = ms_lm_cls(vocab_size=spec["vocab"], d_model=spec["d_model"], num_heads=spec["H"],
                      num_layers=spec["L"], ffn_dim=spec["ffn"], max_seq_len=spec["max_seq_len"])
    g = torch.Generator().manual_seed(spec["seed"] + 1000)
    ids = torch.randint(0, spec["vocab"], (spec["B"], spec["T"]), generator=g)
    labels = ids.clone()
    labels[:, :3] = -100
    prompt = torch.randint(0, spec["vocab"], spec["prompt"], generator=g)
    return model, ids, labels, prompt


def run_lm_case(ms, spec) -> dict:
    model, ids, labels, prompt = lm_inputs(ms.MultiscreenLM, spec)
    # the LM's own _init_weights re-inits every Linear with N(0, 0.02), which
    # leaves nearly every score trimmed; sharpen r and widen w so attention
    # actually contributes in this fixture
    with torch.no_grad():
        for blk in model.blocks:
            blk.attn.s_r.fill_(math.log(0.05))
            blk.attn.s_v.copy_(torch.linspace(1.0, math.log(40.0), spec["H"]))
    state = {k: v.clone() for k, v in model.state_dict().items()}
    out = model(ids, labels=labels)
    out["loss"].backward()
    tokens = model.generate(prompt, max_new_tokens=spec["new"], top_k=1)
    return dict(spec=spec, state=state, logits=out["logits"].detach(), loss=out["loss"].detach(),
                tokens=tokens, s_r_grad=[b.attn.s_r.grad.clone() for b in model.blocks],
                s_v_grad=[b.attn.s_v.grad.clone() for b in model.blocks])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference repository")
    ap.add_argument("--out", default=str(HERE / "golden.pt"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.dont_write_bytecode = True
    import multiscreen as ms  # noqa: E402  (the reference package)

    torch.set_num_threads(4)
    data = {"attention": {}, "lm": {}, "torch_version": torch.__version__}
    for name, spec in ATTN_CASES.items():
        data["attention"][name] = run_attention_case(ms, spec)
    data["cfg1"] = run_cfg1(ms)
    for name, spec in LM_CASES.items():
        data["lm"][name] = run_lm_case(ms, spec)
    torch.save(data, args.out)
    print(f"wrote {args.out} ({Path(args.out).stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
