"""Benchmark: Screening Attention fwd+bwd on B200.

Headline workload (cfg3): isolated ScreeningAttention, d_model=1024, 16
heads x 64, causal, global batch 8, T=4096, bf16, x ~ N(0,1), r_h ~ U[1,2],
w_h ~ U[256,4096] (seeded).  One step = module forward + backward (q/k/v/out
projections on cuBLAS, the screening core on this repo's kernels).  With N
GPUs the global batch of 8 is split over the ranks (8/N sequences each:
strong scaling, batch sharding) and the projection-weight gradients are
averaged over NCCL as data-parallel training does (the out_proj bucket on a
side stream during the screening backward); the whole step is one CUDA
graph.  A weak-scaling run (8 sequences per rank) is reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload cfg3|decode|prefill|lm|generate]

Prints one JSON line (rank 0).  At one GPU the cfg3 line also carries
sub-records measured in the same run: the decode kernel's HBM fraction at a
100K-key window, attention-only fwd+bwd at T=32K and 128K, the cfg2 training
step, the cfg4 prefill, the cfg5 decode step and the reference's own Triton
kernels at cfg3 shapes.  `--impl reference` times the reference algorithm's CPU
implementation (the windowed restatement of multiscreen/attention.py in the
oracle, fp32, all host threads) on a bounded sample of the same workload
(one of the 8 sequences, all 16 heads, per step).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = "pytorch-implementation-of-screening-attention_b200"

D_MODEL, HEADS, HEAD_DIM, BATCH, SEQ = 1024, 16, 64, 8, 4096
METRIC = "screening-attn fwd+bwd tokens/s (ScreeningAttention d=1024 H=16 D=64 causal T=4096, bf16)"
WORKLOAD = ("cfg3: isolated ScreeningAttention d_model=1024, 16 heads x 64, causal, global batch 8 "
            "split over the GPUs, T=4096, bf16, r~U[1,2], w~U[256,4096], fwd+bwd")
# this repo's kernels launched per cfg3 step: forward (r / w transforms,
# prep, k meta, CTA order, attention), backward (TanhNorm-grad prologue, aux
# norms, CTA order, fused attention, dq finalize, dr/dw reduction, r / w
# gradients)
LAUNCHES_PER_STEP = 12
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def head_params(seed=0):
    g = torch.Generator().manual_seed(seed)
    r = 1.0 + torch.rand(HEADS, generator=g)
    w = 256.0 + (4096.0 - 256.0) * torch.rand(HEADS, generator=g)
    return r, w


def windowed_pairs(w: torch.Tensor, T: int, causal=True) -> float:
    """sum over heads of #(i, j) with j in the causal window of i."""
    tot = 0
    for wh in w.tolist():
        d = max(-1, math.ceil(wh) - 1)
        n = d + 1
        if n >= T:
            tot += T * (T + 1) // 2
        else:
            tot += n * (n + 1) // 2 + (T - n) * n
    return float(tot)


def bwd_executed_tiles(w: torch.Tensor, T: int) -> int:
    """Tiles of 128 keys x 64 queries the fused causal backward runs per
    sequence: each key tile [j0, j0 + 127] walks the 64-query tiles from the
    one holding j0 to the one holding min(T - 1, j0 + 127 + ceil(w) - 1)."""
    tot = 0
    for wh in w.tolist():
        dmax = math.ceil(wh) - 1
        if dmax < 0:
            continue
        for j0 in range(0, T, 128):
            ihi = min(T - 1, j0 + 127 + dmax)
            tot += ihi // 64 - j0 // 64 + 1
    return tot


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[3]) if v.lower() == "active"})
        loaded = [r[0] for r in rows if r[2] > 200.0] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


def finish_distributed(dist):
    """End a multi-rank run: wait for the device and the other ranks, then
    leave without tearing down the NCCL communicators -- a process group
    destroyed while CUDA graphs that captured its collectives are alive can
    block at exit."""
    torch.cuda.synchronize()
    dist.barrier()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


class NullClock:
    """Stand-in for ClockSampler inside sub-records (the outer line samples)."""

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        pass

    def summary(self):
        return None


def cpu_reference_sample(threads: int | None = None):
    """Oracle fwd+bwd of one sequence (B=1, T=4096, 16 heads) in fp32 on the
    host; returns (seconds, tokens, threads)."""
    from oracle import screening_oracle as oracle
    nt = threads or os.cpu_count() or 1
    torch.set_num_threads(nt)
    torch.manual_seed(0)
    m = oracle.OracleScreeningAttention(D_MODEL, HEADS, windowed=True)
    r, w = head_params()
    with torch.no_grad():
        m.s_r.copy_(torch.log(r - 1.0))
        m.s_v.copy_(torch.log(w - 1.0))
    x = torch.randn(1, SEQ, D_MODEL, generator=torch.Generator().manual_seed(1))
    x.requires_grad_(True)
    cot = torch.randn(1, SEQ, D_MODEL, generator=torch.Generator().manual_seed(2))
    t0 = time.perf_counter()
    y = m(x, x, x)
    y.backward(cot)
    return time.perf_counter() - t0, SEQ, nt


def run_reference(args, rank):
    if rank != 0:
        return
    times = []
    for i in range(args.warmup + args.steps):
        dt, toks, nt = cpu_reference_sample()
        if i >= args.warmup:
            times.append(dt)
    per = sum(times) / len(times)
    val = SEQ / per
    sample = (f"windowed CPU restatement of multiscreen/attention.py (oracle), fp32: 1 sequence x "
              f"T={SEQ} x {HEADS} heads per step = 1/{BATCH} of the cfg3 batch")
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "seq_len": SEQ, "global_batch": BATCH},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": nt, "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure_decode(dev, window: int, steps: int, warmup: int, splits: int = 0, seed: int = 7,
                   clk=None) -> dict:
    """Decode-kernel roofline: one new token per sequence, B=4 sequences per
    GPU (cfg5: batch 32 over 8 GPUs), 16 heads x 64, bf16 paged cache with
    `window` cached keys in every head's window (the cfg5 prompt is 100K
    tokens; at random init w <= 256, so the window is widened here to make
    the kernel's HBM stream measurable).  Algorithmic bytes per launch =
    keys in window x (K + V rows) + query + output."""
    import importlib
    ms = importlib.import_module(PKG)
    B, H, D = 4, HEADS, HEAD_DIM
    T = window + 1
    cache = ms.PagedKVCache(1, B, H, D, max_len=T, max_window=float(T), dtype=torch.bfloat16,
                            device=dev, page_size=64)
    if splits > 0:
        cache.num_splits = splits
    g = torch.Generator(device=dev).manual_seed(seed)
    for pg in (cache.k_pages[0], cache.v_pages[0]):
        pg.copy_(torch.nn.functional.normalize(
            torch.randn(pg.shape, device=dev, generator=g), dim=-1).to(torch.bfloat16))
    q = torch.randn(B, H, D, device=dev, generator=g).to(torch.bfloat16)
    seq = torch.full((B,), T, dtype=torch.int32, device=dev)
    r = torch.full((H,), 1.02, device=dev)
    w = torch.full((H,), float(T + 1), device=dev)
    # inputs several times larger than L2 need no flush (and a 256 MiB write
    # flush would leave L2 full of dirty lines the kernel then writes back)
    window_bytes = B * H * T * D * 2 * 2
    need_flush = window_bytes < 4 * 126 * 1024 * 1024
    flush = torch.empty(256 * 1024 * 1024 // 4 if need_flush else 1, dtype=torch.float32,
                        device=dev)
    for _ in range(warmup):
        cache.decode(0, q, seq, r, w)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    if clk is not None:
        clk.__enter__()
    for a, b in evs:
        if need_flush:
            flush.zero_()
        a.record()
        cache.decode(0, q, seq, r, w)
        b.record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.__exit__(None, None, None)
    ms_per = statistics.median(a.elapsed_time(b) for a, b in evs)
    keys = B * H * T
    alg_bytes = keys * D * 2 * 2 + 2 * B * H * D * 2
    gbs = alg_bytes / (ms_per / 1e3) / 1e9
    pk, kind = peaks()
    peak = float(pk["hbm_gbs"])
    return {"workload": f"cfg5 decode kernel: B=4/GPU, H=16, D=64, {T} keys per (b,h) window, "
                        f"num_splits={cache.num_splits}",
            "l2": ("flushed (256 MiB write) between launches" if need_flush else
                   f"inputs larger than L2 ({window_bytes / 2**30:.2f} GiB of K/V read per "
                   "launch), no flush"),
            "ms": ms_per, "gbs": gbs, "peak_gbs": peak, "frac": gbs / peak, "peak_kind": kind,
            "bytes_per_launch": alg_bytes, "tokens_per_s_attention_only": B / (ms_per / 1e3)}


def run_decode(args, rank, world):
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    clk = ClockSampler(local)
    d = measure_decode(dev, args.decode_window, args.steps, args.warmup, args.decode_splits,
                       seed=7 + rank, clk=clk)
    if rank == 0:
        print(json.dumps({
            "metric": "screening decode attention, paged bf16 KV, HBM bandwidth",
            "value": d["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": d["ms"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": d["workload"], "l2": d["l2"]},
            "roofline": {"bound": "hbm", "kernel": "decode_bulk+finish", "achieved": d["gbs"],
                         "peak": d["peak_gbs"], "unit": "GB/s", "frac": d["frac"],
                         "peak_kind": d["peak_kind"], "traffic": None},
            "tokens_per_s_attention_only": d["tokens_per_s_attention_only"],
            "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
        }), flush=True)


PREFILL = dict(vocab=50257, d_model=1024, heads=16, layers=12, window=2048.0)


def prefill_flops(T: int, n_layers: int, d_model: int, H: int, D: int, window: float,
                  ffn: int) -> dict:
    """Forward FLOPs of a prefill over T tokens: the windowed attention pairs
    (2 GEMMs of 2*D flops per (i, j) pair) and the dense GEMMs of every block
    (QKV 3d^2, out d^2, FFN 2*d*ffn; 2 flops/MAC) plus the last position's
    lm_head."""
    n = max(0, math.ceil(window) - 1) + 1
    pairs = (T * (T + 1) // 2) if n >= T else (n * (n + 1) // 2 + (T - n) * n)
    attn = n_layers * H * pairs * 2 * (2 * D)
    gemm = n_layers * T * 2 * (4 * d_model * d_model + 2 * d_model * ffn)
    return {"attention": float(attn), "gemm": float(gemm), "total": float(attn + gemm)}


def cpu_prefill_sample(T_sample: int = 4096):
    """One oracle MultiscreenBlock (windowed restatement, fp32, all host
    threads) over T_sample tokens, no_grad; returns (seconds, threads).  The
    whole prefill is this x layers x (T / T_sample): the windowed attention
    and the GEMMs are both linear in T at a fixed window."""
    from oracle import screening_oracle as oracle
    nt = os.cpu_count() or 1
    torch.set_num_threads(nt)
    torch.manual_seed(0)
    d, H = PREFILL["d_model"], PREFILL["heads"]
    blk = oracle.OracleBlock(d, H, windowed=True)
    with torch.no_grad():
        blk.attn.s_v.fill_(math.log(PREFILL["window"] - 1.0))
        for mod in blk.modules():
            if isinstance(mod, torch.nn.Linear):
                torch.nn.init.normal_(mod.weight, std=0.02)
    x = torch.randn(1, T_sample, d, generator=torch.Generator().manual_seed(1)) * 0.02
    with torch.no_grad():
        blk(x)
        t0 = time.perf_counter()
        blk(x)
        dt = time.perf_counter() - t0
    return dt, nt


def run_prefill(args, rank, world, sub=False):
    """cfg4: long-context prefill of MultiscreenLM(50257, 1024, 16, 12) over
    T = --prefill-len tokens (batch 1, bf16, w = 2048 in every head, random
    init), sequence-sharded over the ranks (T / world tokens each, K/V halo of
    2047 rows per layer by NCCL P2P).  A step is the forward of every block
    and the last position's logits (MultiscreenLM.prefill without a cache).
    Strong scaling: T is fixed as the rank count grows."""
    import importlib
    ms = importlib.import_module(PKG)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    T = args.prefill_len
    if T % world:
        raise SystemExit(f"--prefill-len {T} is not divisible by {world} ranks")
    Lb = T // world
    cfg = PREFILL
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or sub):
        dt, nt = cpu_prefill_sample()
        per_tok = dt / 4096 * cfg["layers"]
        cpu = {"value": 1.0 / per_tok, "unit": "tokens/s", "cores": nt, "kind": "port",
               "sample": f"one oracle MultiscreenBlock (windowed, fp32, no_grad) over 4096 "
                         f"tokens in {dt:.2f} s, x {cfg['layers']} layers, linear in T"}
    torch.manual_seed(0)
    model = ms.MultiscreenLM(cfg["vocab"], d_model=cfg["d_model"], num_heads=cfg["heads"],
                             num_layers=cfg["layers"], max_seq_len=T)
    with torch.no_grad():
        for blk in model.blocks:
            blk.attn.s_v.fill_(math.log(cfg["window"] - 1.0))
    model = model.to(dev).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1234)
    ids_host = torch.randint(0, cfg["vocab"], (1, T), generator=g)
    ids_local_host = ids_host[:, rank * Lb:(rank + 1) * Lb].contiguous().pin_memory()
    ids = ids_local_host.to(dev)
    ctx = (lambda: ms.sequence_parallel(Lb)) if dist is not None else contextlib.nullcontext

    def step(inp):
        with torch.no_grad(), ctx():
            return model.prefill(inp, None)

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    if args.profile_only:
        step(ids)
        torch.cuda.synchronize()
        return
    clk = NullClock() if sub else ClockSampler(local)
    clk.__enter__()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        a.record()
        step(ids)
        b.record()
    torch.cuda.synchronize()
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    # one more step with CUDA events around each layer's sharded attention:
    # interior rows (overlapping the halo exchange), the stream's stall for
    # the halo (wait + assembly), boundary rows
    overlap = None
    if dist is not None:
        with ms.shard_timeline() as tl:
            step(ids)
        torch.cuda.synchronize()
        ov = ms.shard_timeline_summary(tl)
        keys = ["interior_ms", "halo_stall_ms", "boundary_ms"]
        t = torch.tensor([ov.get(k_, 0.0) for k_ in keys], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        overlap = {"per_layer_max_over_ranks": dict(zip(keys, (float(x_) for x_ in t.tolist()))),
                   "layers": ov.get("calls", 0),
                   "note": "CUDA events on each rank's stream; halo_stall = time the stream "
                           "waited for the K/V halo after its interior rows were done"}
    # end to end: ids from pinned host memory, last logits back to the host
    logit_host = torch.empty(1, cfg["vocab"], dtype=torch.bfloat16).pin_memory()
    ids_dev = torch.empty_like(ids)
    e2e = []
    for i in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ids_dev.copy_(ids_local_host, non_blocking=True)
        lg = step(ids_dev)
        logit_host.copy_(lg, non_blocking=True)
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e)
    if dist is not None:
        t = torch.tensor([total_ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = (float(x) for x in t.tolist())
    ms_per = total_ms / args.steps
    e2e_per = e2e_ms / args.steps
    ffn = 4 * cfg["d_model"]
    fl = prefill_flops(T, cfg["layers"], cfg["d_model"], cfg["heads"], HEAD_DIM, cfg["window"],
                       ffn)
    pk, kind = peaks()
    peak = float(pk.get("bf16_tflops_sustained", pk["bf16_tflops"]))
    tf = fl["total"] / (ms_per / 1e3) / 1e12
    if sub:
        return {"workload": f"cfg4: MultiscreenLM(50257, 1024, 16, 12) prefill, batch 1, T={T}, "
                            "w=2048, random init, no_grad, last-position logits, one GPU",
                "ms_per_step": ms_per, "tokens_per_s": T / (ms_per / 1e3),
                "e2e_tokens_per_s": T / (e2e_per / 1e3), "tflops": tf,
                "frac_of_sustained_peak": tf / peak,
                "flops_basis": "windowed attention pairs + dense block GEMMs"}
    if rank == 0:
        print(json.dumps({
            "metric": "long-context prefill tokens/s (MultiscreenLM 1024x16x12, T=131072, w=2048)",
            "value": T / (ms_per / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg4 prefill: MultiscreenLM(50257, 1024, 16, 12), batch 1, "
                                   f"T={T}, w=2048, random init, no_grad, last-position logits",
                       "seq_len": T, "global_batch": 1,
                       "parallelism": f"sequence-sharded x{world}, K/V halo 2047 rows/layer "
                                      f"by NCCL P2P",
                       "l2": f"inputs larger than L2 (activations of {Lb} tokens x 1024 bf16 "
                             f"per layer plus 12 layers of weights)"},
            "roofline": {"bound": "tensor", "kernel": "whole prefill step (attention + GEMMs)",
                         "achieved": tf / world, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / world / peak, "peak_kind": kind + " sustained",
                         "traffic": None, "per": "GPU (achieved = job FLOP/s / ranks)",
                         "flops_basis": "windowed attention pairs + dense block GEMMs"},
            "flops_per_step": fl,
            "halo_overlap": overlap,
            "cpu_baseline": cpu,
            "e2e": {"value": T / (e2e_per / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": ids_local_host.numel() * 8,
                    "d2h_bytes_per_step": cfg["vocab"] * 2},
            "clocks": clk.summary(),
            "gpu_launches": 6 * cfg["layers"] * args.steps,
        }), flush=True)
    if dist is not None:
        finish_distributed(dist)


def run_lm(args, rank, world, sub=False):
    """cfg2: one training step of MultiscreenLM(50257, d_model=256, 4 heads,
    4 layers, max_seq_len=512) on batch 16 x T=512 synthetic token ids per
    GPU: bf16 autocast forward + backward, fp32 master weights, fused AdamW;
    data parallel (DDP, NCCL all-reduce of the gradients) for N > 1."""
    import importlib
    ms = importlib.import_module(PKG)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    B, T, V = 16, 512, 50257
    torch.manual_seed(0)
    model = ms.MultiscreenLM(V, d_model=256, num_heads=4, num_layers=4, max_seq_len=T).to(dev)
    n_params = sum(p.numel() for p in model.parameters())
    net = model
    if dist is not None:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local])
    # one GPU: the whole step (forward, backward, AdamW) is captured once in a
    # CUDA graph and replayed -- the step is ~150 small kernels, so launch
    # overhead, not the GPU, bounds the eager loop
    use_graph = world == 1 and not args.no_graph
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True, capturable=use_graph)
    g = torch.Generator().manual_seed(100 + rank)
    ids_host = torch.randint(0, V, (B, T), generator=g).pin_memory()
    ids = ids_host.to(dev)

    def eager_step(inp):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = net(inp, labels=inp)
        out["loss"].backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return out["loss"]

    step = eager_step
    graph_note = "eager (multi-GPU DDP step)" if world > 1 else "eager (--no-graph)"
    if use_graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(args.warmup, 3)):
                eager_step(ids)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        static_ids = ids.clone()
        graph = torch.cuda.CUDAGraph()
        opt.zero_grad(set_to_none=True)
        with torch.cuda.graph(graph):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                static_out = net(static_ids, labels=static_ids)
            static_out["loss"].backward()
            opt.step()
        static_loss = static_out["loss"]

        def step(inp):
            if inp.data_ptr() != static_ids.data_ptr():
                static_ids.copy_(inp, non_blocking=True)
            graph.replay()
            return static_loss
        graph_note = "one CUDA graph per step (forward, backward, fused AdamW)"

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    clk = NullClock() if sub else ClockSampler(local)
    clk.__enter__()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        a.record()
        step(ids)
        b.record()
    torch.cuda.synchronize()
    total = sum(a.elapsed_time(b) for a, b in evs)
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()
    ids_dev = static_ids if use_graph else torch.empty_like(ids)
    e2e = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ids_dev.copy_(ids_host, non_blocking=True)
        loss = step(ids_dev)
        loss_host.copy_(loss.detach().float().view(1), non_blocking=True)
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e)
    if dist is not None:
        t = torch.tensor([total, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total, e2e_ms = (float(x) for x in t.tolist())
    ms_per = total / args.steps
    toks = B * T * world
    # training FLOPs per step: 6 x parameters x tokens for the dense layers
    # (lm_head tied to the embedding counts once) + windowed attention x 3
    w_def = torch.exp(torch.linspace(0, math.log(255), 4)) + 1.0
    attn = 3 * 4 * windowed_pairs(w_def, T) * B * 2 * (2 * 64)
    dense = 6.0 * (n_params - 512 * 256) * B * T
    pk, kind = peaks()
    peak = float(pk.get("bf16_tflops_sustained", pk["bf16_tflops"]))
    tf = (dense + attn) / (ms_per / 1e3) / 1e12
    cpu = None
    if sub:
        return {"workload": "cfg2: MultiscreenLM(50257, 256, 4, 4), batch 16 x 512, bf16 "
                            "autocast, fp32 master weights, fused AdamW, one CUDA graph per step",
                "ms_per_step": ms_per, "tokens_per_s": toks / (ms_per / 1e3),
                "e2e_tokens_per_s": toks / (e2e_ms / args.steps / 1e3),
                "tflops_per_gpu": tf / world, "frac_of_sustained_peak": tf / world / peak}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import screening_oracle as oracle
        nt = os.cpu_count() or 1
        torch.set_num_threads(nt)
        torch.manual_seed(0)
        om = oracle.OracleLM(V, d_model=256, num_heads=4, num_layers=4, max_seq_len=T,
                             windowed=True)
        oopt = torch.optim.AdamW(om.parameters(), lr=3e-4)
        oid = ids_host[:1].clone()
        t0 = time.perf_counter()
        out = om(oid, labels=oid)
        out["loss"].backward()
        oopt.step()
        dt = time.perf_counter() - t0
        cpu = {"value": T / dt, "unit": "tokens/s", "cores": nt, "kind": "port",
               "sample": f"oracle LM training step, 1 sequence x T={T} fp32, {dt:.2f} s"}
    if rank == 0:
        print(json.dumps({
            "metric": "MultiscreenLM training step tokens/s (cfg2: 50257 x 256 x 4 heads x 4 "
                      "layers, B=16, T=512, bf16)",
            "value": toks / (ms_per / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"cfg2: MultiscreenLM(50257, 256, 4, 4, max_seq_len=512), "
                                   f"{n_params} parameters, batch 16/GPU, T=512, bf16 autocast, "
                                   f"fp32 master weights, fused AdamW; {graph_note}",
                       "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world}",
                       "l2": "no flush: weights + optimizer state + activations > L2"},
            "roofline": {"bound": "tensor", "kernel": "whole training step", "achieved": tf / world,
                         "peak": peak, "unit": "TFLOP/s", "frac": tf / world / peak,
                         "peak_kind": kind + " sustained", "traffic": None,
                         "per": "GPU"},
            "cpu_baseline": cpu,
            "e2e": {"value": toks / (e2e_ms / args.steps / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": ids_host.numel() * 8, "d2h_bytes_per_step": 4},
            "clocks": clk.summary(),
        }), flush=True)
    if dist is not None:
        finish_distributed(dist)


def run_generate(args, rank, world, sub=False):
    """cfg5: MultiscreenLM(50257, 1024, 16, 12) at random init (w = 2..256 per
    head), 4 prompts of --prompt-len random tokens per GPU, 256 greedy new
    tokens through the paged KV cache.  Prefill and decode are timed apart
    (CUDA events); the decode loop is one CUDA-graph replay per token plus
    greedy sampling, exactly as generate() runs it.  No collective: every rank
    serves its own 4 sequences."""
    import importlib
    ms = importlib.import_module(PKG)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    B, T0, NEW, V = 4, args.prompt_len, 256, 50257
    torch.manual_seed(0)
    model = ms.MultiscreenLM(V, d_model=1024, num_heads=16, num_layers=12,
                             max_seq_len=T0 + NEW).to(dev).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(7 + rank)
    prompt = torch.randint(0, V, (B, T0), generator=g).to(dev)

    def one():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.no_grad():
            ev[0].record()
            cache = model.make_cache(B, T0 + NEW)
            state = model._decode_state()
            logits = model.prefill(prompt, cache)
            ev[1].record()
            graph, g_tok, g_pos, g_logits = model._capture_decode(B, T0, cache, state)
            ev[2].record()
            toks = []
            for step in range(NEW):
                nxt = logits.argmax(-1, keepdim=True)
                toks.append(nxt)
                if step + 1 < NEW:
                    g_tok.copy_(nxt)
                    g_pos.fill_(T0 + step)
                    graph.replay()
                    logits = g_logits
            ev[3].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3]), torch.cat(toks, 1)

    for _ in range(args.warmup):
        one()
    clk = NullClock() if sub else ClockSampler(local)
    clk.__enter__()
    if dist is not None:
        dist.barrier()
    runs = [one() for _ in range(args.steps)]
    clk.__exit__(None, None, None)
    pre = sum(r[0] for r in runs) / len(runs)
    dec = sum(r[1] for r in runs) / len(runs)
    if dist is not None:
        t = torch.tensor([pre, dec], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre, dec = (float(x) for x in t.tolist())
    if sub:
        return {"workload": f"cfg5: MultiscreenLM(50257, 1024, 16, 12), 4 sequences x {T0}-token "
                            f"prompts, {NEW} greedy tokens, paged bf16 cache, one CUDA-graph "
                            "replay per token",
                "decode_ms_per_token": dec / NEW, "decode_tokens_per_s": B * NEW / (dec / 1e3),
                "prefill_ms": pre, "prefill_tokens_per_s": B * T0 / (pre / 1e3)}
    if rank == 0:
        print(json.dumps({
            "metric": "generate() decode tokens/s (cfg5: MultiscreenLM 1024 x 16 x 12, 100K-token "
                      "prompts, 256 greedy tokens, bf16 paged KV cache)",
            "value": B * NEW * world / (dec / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dec,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"cfg5: 4 sequences/GPU x {T0}-token random prompts, "
                                   f"{NEW} new tokens (top_k=1), random init (w = 2..256)",
                       "global_batch": B * world, "seq_len": T0, "parallelism": f"batch x{world}",
                       "decode": "one CUDA-graph replay per token (12 layers + lm_head)"},
            "prefill_ms": pre, "prefill_tokens_per_s": B * T0 * world / (pre / 1e3),
            "decode_ms_per_token": dec / NEW,
            "clocks": clk.summary(),
        }), flush=True)
    if dist is not None:
        finish_distributed(dist)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=0,
                    help="per-GPU batch override (profiling); default global batch / GPUs")
    ap.add_argument("--global-batch", type=int, default=BATCH)
    ap.add_argument("--no-sub", action="store_true",
                    help="cfg3: skip the sub-records (weak scaling, other configurations)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-reps", type=int, default=5)
    ap.add_argument("--workload", default="cfg3", choices=["cfg3", "decode", "prefill", "lm", "generate"],
                    help="cfg3: the headline fwd+bwd step; decode: the paged-cache decode "
                         "kernel's HBM roofline (cfg5 shapes, long window)")
    ap.add_argument("--decode-window", type=int, default=100_000)
    ap.add_argument("--prefill-len", type=int, default=131072)
    ap.add_argument("--prompt-len", type=int, default=100_000)
    ap.add_argument("--decode-splits", type=int, default=0,
                    help="override the cache's split count (0: its own heuristic)")
    ap.add_argument("--no-graph", action="store_true",
                    help="cfg3 / lm workloads: run the training step eagerly instead of as a "
                         "CUDA graph")
    ap.add_argument("--profile-only", action="store_true",
                    help="warm-up steps + one step, nothing else (for ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "decode":
        run_decode(args, rank, world)
        return
    if args.workload == "prefill":
        run_prefill(args, rank, world)
        return
    if args.workload == "lm":
        run_lm(args, rank, world)
        return
    if args.workload == "generate":
        run_generate(args, rank, world)
        return

    run_cfg3(args, rank, world, local)


def time_events(fn, reps, flush=None, warmup=1):
    """Median CUDA-event time (ms) of fn() on the current stream."""
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b))
    return statistics.median(out)


def measure_long_context(dev, T: int, reps: int = 3) -> dict:
    """Attention-only fwd+bwd (the screening core: screen_fwd, screen_bwd) at
    batch 1, 16 heads x 64, length T, with the cfg3 per-head r / w draws;
    q, k, v ~ N(0, 1) bf16.  TFLOP/s on the windowed algorithmic pairs
    (2 GEMMs forward, 5 backward, 2*D flops per pair per GEMM)."""
    import importlib
    L = importlib.import_module(PKG)._lib
    g = torch.Generator(device=dev).manual_seed(T)
    q, k, v, dy = (torch.randn(1, T, HEADS, HEAD_DIM, device=dev, generator=g)
                   .to(torch.bfloat16) for _ in range(4))
    r, w = (t.to(dev) for t in head_params())
    y, no, nq, nk, nv, q2, k2, v2 = L.screen_fwd(q, k, v, r, w, True)
    fwd = time_events(lambda: L.screen_fwd(q, k, v, r, w, True), reps)
    bwd = time_events(lambda: L.screen_bwd(q2, k2, v2, nq, nk, nv, y, no, dy, r, w), reps)
    pairs = windowed_pairs(w.cpu(), T)
    gemm = 2.0 * HEAD_DIM
    pk, kind = peaks()
    peak = float(pk["bf16_tflops"])
    tf_f = 2 * gemm * pairs / (fwd / 1e3) / 1e12
    tf_b = 5 * gemm * pairs / (bwd / 1e3) / 1e12
    tf = 7 * gemm * pairs / ((fwd + bwd) / 1e3) / 1e12
    return {"T": T, "batch": 1, "fwd_ms": fwd, "bwd_ms": bwd,
            "tokens_per_s": T / ((fwd + bwd) / 1e3),
            "tflops_windowed": {"fwd": tf_f, "bwd": tf_b, "fwd_bwd": tf},
            "frac_of_peak": {"fwd": tf_f / peak, "bwd": tf_b / peak, "fwd_bwd": tf / peak},
            "peak_tflops": peak, "peak_kind": kind,
            "windowed_pairs": pairs, "dense_pairs": HEADS * T * (T + 1) / 2}


def measure_prior_art_triton(dev, ours_fwd_ms: float, ours_bwd_ms: float, reps: int = 3) -> dict:
    """The reference's own GPU path, its Triton kernels screening_attention_fwd
    (multiscreen/kernels/screening_fwd.py:216-270) and screening_attention_bwd
    (multiscreen/kernels/screening_bwd.py:229-287), unmodified from the
    installed copy under baseline/_ref, at the cfg3 attention shapes (B=8,
    H=16, T=4096, D=64, bf16 unit rows, the cfg3 r / w draws).  Its backward
    returns dq, dk, dv only (no dr, dw)."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "multiscreen").exists():
        return {"unavailable": "reference not installed under baseline/_ref"}
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from multiscreen.kernels.screening_fwd import screening_attention_fwd
    from multiscreen.kernels.screening_bwd import screening_attention_bwd
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v, do = (torch.nn.functional.normalize(
        torch.randn(BATCH, HEADS, SEQ, HEAD_DIM, device=dev, generator=g), dim=-1)
        .to(torch.bfloat16) for _ in range(4))
    r, w = (t.to(dev) for t in head_params())
    fwd = time_events(lambda: screening_attention_fwd(q, k, v, r, w, causal=True), reps)
    bwd = time_events(lambda: screening_attention_bwd(q, k, v, do, r, w, causal=True), reps)
    return {"source": "multiscreen.kernels (Triton), unmodified, baseline/_ref",
            "shape": "B=8, H=16, T=4096, D=64, causal, bf16 in, fp32 out",
            "triton_fwd_ms": fwd, "triton_bwd_ms": bwd, "ours_fwd_ms": ours_fwd_ms,
            "ours_bwd_ms": ours_bwd_ms, "speedup_fwd": fwd / ours_fwd_ms,
            "speedup_bwd": bwd / ours_bwd_ms,
            "note": "the Triton backward computes dq, dk, dv only; ours adds dr, dw"}


def _sub(fn):
    try:
        return fn()
    except Exception as e:  # a sub-record must not sink the headline line
        return {"error": f"{type(e).__name__}: {e}"[:300]}


class TrainStep:
    """One cfg3 training step: module forward, backward and (N > 1) the
    data-parallel gradient all-reduce (mean over the ranks).  The out_proj
    weight gradient -- ready as soon as the backward starts -- is all-reduced
    on a side stream from its post-accumulate hook, overlapping the screening
    backward; the q/k/v/s_r/s_v gradients follow as one flat bucket.  With
    `graph` the whole step is captured once as a CUDA graph and replayed (at
    one sequence per GPU the eager step is bound by host-side launch work,
    ~0.9 ms against ~0.35 ms of GPU work)."""

    def __init__(self, attn, params, cot, dist, graph: bool, warmup: int, n_inputs: int = 1):
        self.attn, self.params, self.cot, self.dist = attn, params, cot, dist
        self.rest = [p for p in params if p is not attn.out_proj.weight]
        self.side = torch.cuda.Stream()
        self.graph = None
        if dist is not None:
            # one hook per module; it reduces on the side stream of the step
            # being run (or captured)
            attn._grad_side = self.side
            if not hasattr(attn, "_grad_hook"):
                def hook(p):
                    side = attn._grad_side
                    side.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(side):
                        dist.all_reduce(p.grad, op=dist.ReduceOp.AVG)
                attn._grad_hook = attn.out_proj.weight.register_post_accumulate_grad_hook(hook)
        if graph:
            # one graph per static input buffer, so that an input pipeline
            # can fill one buffer from the host while the other one's graph
            # runs, with no device-to-device copy in between
            self.xs, self.ys, self.graphs = [], [], []
            cur = torch.cuda.current_stream()
            for i in range(n_inputs):
                xi = torch.empty_like(cot)
                xi.copy_(cot)
                ws = torch.cuda.Stream()
                ws.wait_stream(cur)
                with torch.cuda.stream(ws):
                    for _ in range(max(warmup, 3) if i == 0 else 1):
                        self._body(xi)
                cur.wait_stream(ws)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    yi = self._body(xi)
                self.xs.append(xi)
                self.ys.append(yi)
                self.graphs.append(g)
            self.x, self.y, self.graph = self.xs[0], self.ys[0], self.graphs[0]

    def _body(self, inp):
        if self.dist is not None:
            self.attn._grad_side = self.side
        for p in self.params:
            p.grad = None
        y = self.attn(inp, inp, inp)
        y.backward(self.cot)
        if self.dist is not None:
            flat = torch.cat([p.grad.reshape(-1) for p in self.rest])
            self.dist.all_reduce(flat, op=self.dist.ReduceOp.AVG)
            off = 0
            for p in self.rest:
                n = p.grad.numel()
                p.grad.copy_(flat[off:off + n].view_as(p.grad))
                off += n
            torch.cuda.current_stream().wait_stream(self.side)
        return y

    def replay(self, i: int):
        """Run the step on static input buffer i (filled by the caller)."""
        self.graphs[i].replay()
        return self.ys[i]

    def __call__(self, inp):
        if self.graph is None:
            return self._body(inp)
        if inp.data_ptr() != self.x.data_ptr():
            self.x.copy_(inp, non_blocking=True)
        self.graph.replay()
        return self.y


def output_metric(y: torch.Tensor) -> torch.Tensor:
    """The step's result read back to the host in the end-to-end loop: the
    mean square of the module output, as one fp32 reduction over the bf16
    tensor (no fp32 copy of the output)."""
    return (torch.linalg.vector_norm(y, dtype=torch.float32).square() / y.numel()).view(1)


def run_cfg3(args, rank, world, local):
    import argparse as _ap
    import importlib
    ms = importlib.import_module(PKG)
    L = ms._lib
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.profile_only):
        cpu_reference_sample()                   # warm-up (allocator, thread pool)
        dt, toks, nt = cpu_reference_sample()
        cpu = {"value": toks / dt, "unit": "tokens/s", "cores": nt, "kind": "port",
               "sample": f"windowed CPU restatement of multiscreen/attention.py (oracle) fwd+bwd, "
                         f"fp32, 1 sequence x T={SEQ} x {HEADS} heads = 1/{BATCH} of the cfg3 "
                         f"batch, {dt:.1f} s"}

    # strong scaling: the global batch of 8 is split over the ranks
    GB = args.global_batch
    if GB % world:
        raise SystemExit(f"global batch {GB} is not divisible by {world} ranks")
    B = args.batch if args.batch else GB // world
    torch.manual_seed(0)
    attn = ms.ScreeningAttention(D_MODEL, HEADS)
    r_h, w_h = head_params()
    with torch.no_grad():
        attn.s_r.copy_(torch.log(r_h - 1.0))
        attn.s_v.copy_(torch.log(w_h - 1.0))
    attn = attn.to(dev).to(torch.bfloat16)
    params = [p for p in attn.parameters()]

    def make_inputs(batch, seed_rank):
        gen = torch.Generator(device=dev).manual_seed(1000 + seed_rank)
        xx = torch.randn(batch, SEQ, D_MODEL, device=dev, generator=gen).to(torch.bfloat16)
        cc = torch.randn(batch, SEQ, D_MODEL, device=dev, generator=gen).to(torch.bfloat16)
        return xx, cc

    x, cot = make_inputs(B, rank)
    use_graph = not args.no_graph
    train = TrainStep(attn, params, cot, dist, use_graph, args.warmup,
                      n_inputs=2 if use_graph and not args.profile_only else 1)
    if use_graph:
        # the timed steps read the graph's own static input (no copy per step)
        train.x.copy_(x)
        x = train.x

    def step(inp, tr=None):
        return (tr or train)(inp)

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    # clocks are sampled from the warm-up through the e2e loop (all GPU-bound);
    # the median is taken over samples drawing > 200 W
    clk = ClockSampler(local)
    if not args.profile_only:
        clk.__enter__()
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    if args.profile_only:
        step(x)
        torch.cuda.synchronize()
        return

    def timed(inp, tr=None):
        """K steps, L2 flushed between steps (outside the events); the job
        time is the max over ranks of the summed step times."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        for s0, s1 in evs:
            flush.zero_()
            s0.record()
            step(inp, tr)
            s1.record()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        tot = sum(a.elapsed_time(b) for a, b in evs)
        if dist is not None:
            t = torch.tensor([tot], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            tot = float(t.item())
        return tot / args.steps

    ms_per_step = timed(x)
    tokens_per_step = B * SEQ * world
    value = tokens_per_step / (ms_per_step / 1e3)

    weak = None
    if world > 1 and not args.no_sub:
        # weak scaling beside it: a full batch of 8 on every rank
        xw, cw = make_inputs(BATCH, rank)
        tw = TrainStep(attn, params, cw, dist, use_graph, args.warmup)
        for _ in range(args.warmup):
            step(xw, tw)
        wms = timed(xw, tw)
        weak = {"per_gpu_batch": BATCH, "global_batch": BATCH * world, "ms_per_step": wms,
                "value": BATCH * SEQ * world / (wms / 1e3), "unit": "tokens/s"}
        del xw, cw, tw

    # ---- per-kernel timing of the screening core (CUDA events, same stream)
    H, Dh = HEADS, HEAD_DIM
    qkv = torch.nn.functional.linear(x, torch.cat([attn.q_proj.weight, attn.k_proj.weight,
                                                   attn.v_proj.weight], 0)).view(B, SEQ, 3, H, Dh)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    rr, ww = attn.sharpness().detach(), attn.window().detach()
    stats = torch.zeros(2, dtype=torch.int64, device=dev)
    y, no, nq, nk, nv, q2, k2, v2 = L.screen_fwd(q, k, v, rr, ww, True, tile_stats=stats)
    dy = cot.view(B, SEQ, H, Dh)
    reps = args.kernel_reps
    kt = {
        "fwd": time_events(lambda: L.screen_fwd(q, k, v, rr, ww, True, norms=(nq, nk, nv),
                                                stages=2), reps, flush),
        "bwd_prologue": time_events(lambda: L.screen_bwd(q, k, v, nq, nk, nv, y, no, dy, rr, ww,
                                                         stages=1), reps, flush),
        # stage 4: the fused key-major kernel (dk, dv and dq) + the dq finalize
        "bwd": time_events(lambda: L.screen_bwd(q, k, v, nq, nk, nv, y, no, dy, rr, ww,
                                                stages=5), reps, flush),
    }
    # stage 5 includes the prologue; isolate the attention kernel
    kt["bwd"] = max(kt["bwd"] - kt["bwd_prologue"], 1e-6)
    stats.zero_()
    L.screen_fwd(q, k, v, rr, ww, True, norms=(nq, nk, nv), stages=2, tile_stats=stats)
    torch.cuda.synchronize()
    visited, live = (int(t) for t in stats.tolist())

    pairs_w = windowed_pairs(ww.cpu(), SEQ) * B
    pairs_dense = H * SEQ * (SEQ + 1) / 2 * B
    gemm = 2.0 * Dh  # flops per (i, j) pair per GEMM
    # algorithmic GEMMs per in-window pair: fwd S, alpha V; bwd S, dP, dV, dK, dQ
    kernel_flops = {"fwd": 2 * gemm * pairs_w, "bwd": 5 * gemm * pairs_w}
    dom = max(kernel_flops, key=lambda n: kt[n])
    pk, pk_kind = peaks()
    peak = float(pk["bf16_tflops"])
    achieved = kernel_flops[dom] / (kt[dom] / 1e3) / 1e12
    blk = 16 * 64 * gemm  # flops of one 16x64 score block per GEMM
    fwd_exec = (visited + live) * blk
    step_s = ms_per_step / 1e3
    tflops = {
        "dense_equiv": 7 * gemm * pairs_dense / step_s / 1e12 * world,
        "windowed": 7 * gemm * pairs_w / step_s / 1e12 * world,
        "fwd_executed_fraction_of_windowed": fwd_exec / (2 * gemm * pairs_w),
    }
    # the fused backward as executed: its tiles x 6 MMA products of 128 x 64 x
    # D (S, dP from the G hi and lo planes, dV, dK, dQ) -- beside the
    # algorithmic 5 GEMMs per in-window pair of the roofline line
    bwd_exec = bwd_executed_tiles(ww.cpu(), SEQ) * B * 6 * 128 * 64 * gemm
    tflops["bwd_executed_tile"] = bwd_exec / (kt["bwd"] / 1e3) / 1e12
    tflops["bwd_executed_tile_frac_of_peak"] = tflops["bwd_executed_tile"] / peak
    traffic = None
    tfile = REPO / "profiles" / f"{dom}_traffic.txt"
    if tfile.exists() and B == BATCH:
        for ln in tfile.read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch_full_workload:"):
                traffic = float(ln.split(":")[1])

    # ---- end to end through the module with host buffers
    x_host = x.cpu().pin_memory()
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    # the step's input buffers: the graphs' static inputs (no device copy)
    bufs = train.xs if use_graph else [torch.empty_like(x), torch.empty_like(x)]

    def run_on(i):
        return train.replay(i) if use_graph else step(bufs[i])

    # (a) serial: copy in, step, loss out, one after the other
    e2e_ev = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        bufs[0].copy_(x_host, non_blocking=True)
        yy = run_on(0)
        loss_host.copy_(output_metric(yy), non_blocking=True)
        b.record()
        if i >= args.warmup:
            e2e_ev.append((a, b))
    torch.cuda.synchronize()
    e2e_serial_ms = sum(a.elapsed_time(b) for a, b in e2e_ev) / len(e2e_ev)
    # (b) pipelined, as an input loader runs it: step i+1's pinned host ->
    # device copy on a copy stream overlaps step i; two device buffers.  The
    # timed region holds K steps, K copies and K loss read-backs.
    cur = torch.cuda.current_stream()
    cp = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    used = [False, False]

    def issue_copy(i):
        k2_ = i % 2
        with torch.cuda.stream(cp):
            if used[k2_]:
                cp.wait_event(free[k2_])
            bufs[k2_].copy_(x_host, non_blocking=True)
            ready[k2_].record(cp)

    n_all = args.warmup + args.steps
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    issue_copy(0)
    for i in range(n_all):
        if i == args.warmup:
            t0.record()
        cur.wait_event(ready[i % 2])
        issue_copy(i + 1)   # the last one stands for the next step's input
        yy = run_on(i % 2)
        free[i % 2].record(cur)
        used[i % 2] = True
        loss_host.copy_(output_metric(yy), non_blocking=True)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1) / args.steps
    # the host link on its own: pinned host -> device copy of one step's input
    a, bb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(3):
        x_dev.copy_(x_host, non_blocking=True)
    bb.record()
    torch.cuda.synchronize()
    h2d_gbs = 3 * x.numel() * x.element_size() / (a.elapsed_time(bb) / 1e3) / 1e9
    clk.__exit__(None, None, None)
    if dist is not None:
        t = torch.tensor([e2e_ms, e2e_serial_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms, e2e_serial_ms = (float(v_) for v_ in t.tolist())

    # ---- sub-records (one GPU): the other configurations' key numbers
    sub = None
    if world == 1 and not args.no_sub:
        del qkv, q, k, v, y, q2, k2, v2, bufs
        torch.cuda.empty_cache()
        sub = {}
        sub["prior_art_triton"] = _sub(lambda: measure_prior_art_triton(dev, kt["fwd"],
                                                                        kt["bwd"] + kt["bwd_prologue"]))
        sub["decode_kernel_100k"] = _sub(lambda: measure_decode(dev, 100_000, 10, 3))
        for T_ in (32768, 131072):
            sub[f"attention_T{T_ // 1024}k"] = _sub(lambda: measure_long_context(dev, T_))
        torch.cuda.empty_cache()
        sa = _ap.Namespace(**vars(args))
        sa.steps, sa.warmup, sa.no_graph = 10, 3, False
        sub["cfg2_lm_step"] = _sub(lambda: run_lm(sa, 0, 1, sub=True))
        torch.cuda.empty_cache()
        sp = _ap.Namespace(**vars(args))
        sp.steps, sp.warmup, sp.prefill_len = 3, 3, 131072
        sub["cfg4_prefill"] = _sub(lambda: run_prefill(sp, 0, 1, sub=True))
        torch.cuda.empty_cache()
        sg = _ap.Namespace(**vars(args))
        sg.steps, sg.warmup, sg.prompt_len = 1, 1, 100_000
        sub["cfg5_generate"] = _sub(lambda: run_generate(sg, 0, 1, sub=True))

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "ScreeningAttention(1024, 16)",
                       "global_batch": B * world, "per_gpu_batch": B, "seq_len": SEQ,
                       "parallelism": (f"dp{world} (batch sharding; gradient all-reduce over "
                                       f"NCCL, out_proj bucket overlapped with the backward)"
                                       if world > 1 else "dp1"),
                       "step": ("one CUDA graph per step (forward, backward, all-reduce)"
                                if use_graph else "eager"),
                       "l2": "flushed (256 MiB write) between steps"},
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_kind": pk_kind,
                         "traffic": traffic,
                         "flops_basis": "windowed algorithmic pairs x 2*D per GEMM"},
            "kernel_ms": kt, "tflops": tflops,
            "tile_stats": {"fwd_blocks_in_window": visited, "fwd_blocks_live": live},
            "cpu_baseline": cpu,
            # the two input pipelines, each timed over K steps with the copy
            # and the read-back inside; the line reports the faster (at 8
            # ranks the copy engine's H2D copy and NCCL's traffic contend,
            # and the serial order wins)
            "e2e": {"value": tokens_per_step / (min(e2e_ms, e2e_serial_ms) / 1e3),
                    "unit": "tokens/s",
                    "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                    "h2d_gbs_measured": h2d_gbs, "pinned": bool(x_host.is_pinned()),
                    "input_pipeline": ("next step's H2D copy on a copy stream during this step"
                                       if e2e_ms <= e2e_serial_ms else
                                       "serial: H2D copy, step, loss read-back"),
                    "pipelined_value": tokens_per_step / (e2e_ms / 1e3),
                    "serial_value": tokens_per_step / (e2e_serial_ms / 1e3)},
            "weak_scaling": weak,
            "clocks": clk.summary(),
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "sub": sub,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        finish_distributed(dist)


if __name__ == "__main__":
    main()
