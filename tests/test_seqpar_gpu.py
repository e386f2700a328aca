"""Sequence-sharded attention and LM on the CUDA kernels.

world = 1 (any box): the interior / boundary split of the block with the
kernels' q_offset must give the rows of one unsharded call.
world = 2 (boxes with two GPUs, NCCL): the halo exchange between ranks, the
reverse gradient exchange and the sharded LM loss against the unsharded
model on the same GPU.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import load_pkg, rel_err

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attn_inputs(B, T, H, D, dtype, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, T, H, D, device=dev, generator=g)
    k = (q + 0.6 * torch.randn(B, T, H, D, device=dev, generator=g)).to(dtype)
    v = torch.randn(B, T, H, D, device=dev, generator=g).to(dtype)
    cot = torch.randn(B, T, H, D, device=dev, generator=g).to(dtype)
    return q.to(dtype), k, v, cot


def _run(ms, q, k, v, r, w, cot, sharded, s0=0, s1=None, shard=None):
    s1 = q.shape[1] if s1 is None else s1
    ql, kl, vl = (t[:, s0:s1].clone().requires_grad_(True) for t in (q, k, v))
    rr, ww = r.clone().requires_grad_(True), w.clone().requires_grad_(True)
    if sharded:
        y = ms.screening_attention_sharded(ql, kl, vl, rr, ww, shard=shard)
    else:
        y = ms.screening_attention(ql, kl, vl, rr, ww, True)
    (y.float() * cot[:, s0:s1].float()).sum().backward()
    return [y, ql.grad, kl.grad, vl.grad, rr.grad, ww.grad]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_world1_split_rows_match_one_call(ms, dtype):
    dev = torch.device("cuda:0")
    if not dist.is_initialized():
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
        own = True
    else:
        own = False
    try:
        B, T, H, D = 2, 700, 3, 64
        q, k, v, cot = _attn_inputs(B, T, H, D, dtype, dev)
        r = torch.tensor([1.1, 1.3, 1.02], device=dev)
        w = torch.tensor([250.0, 40.5, 130.0], device=dev)
        ref = _run(ms, q, k, v, r, w, cot, False)
        with ms.sequence_parallel(T) as shard:
            got = _run(ms, q, k, v, r, w, cot, True, shard=shard)
        tol = 1e-4 if dtype == torch.float32 else 2e-2
        for name, a, b in zip(("y", "dq", "dk", "dv", "dr", "dw"), got, ref):
            assert rel_err(a, b) <= tol, name
    finally:
        if own:
            dist.destroy_process_group()


def _worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        ms = load_pkg()
        dist.barrier()
        # attention: halo 1499 rows, block 1024 -> rank 1 needs most of rank 0
        B, L, H, D = 1, 1024, 2, 64
        T = L * world
        for dtype in (torch.float32, torch.bfloat16):
            q, k, v, cot = _attn_inputs(B, T, H, D, dtype, dev, seed=4)
            r = torch.tensor([1.05, 1.2], device=dev)
            w = torch.tensor([1500.0, 300.0], device=dev)
            ref = _run(ms, q, k, v, r, w, cot, False)
            s0, s1 = rank * L, (rank + 1) * L
            with ms.sequence_parallel(L) as shard:
                got = _run(ms, q, k, v, r, w, cot, True, s0, s1, shard)
            gs = torch.stack([got[4], got[5]])
            dist.all_reduce(gs)
            tol = 1e-4 if dtype == torch.float32 else 2e-2
            for name, a, b in zip(("y", "dq", "dk", "dv"), got[:4], ref[:4]):
                assert rel_err(a, b[:, s0:s1]) <= tol, (name, dtype, rank)
            assert rel_err(gs[0], ref[4]) <= tol, ("dr", dtype, rank)
            assert rel_err(gs[1], ref[5]) <= tol, ("dw", dtype, rank)

        # LM: logits, global loss and summed parameter gradients
        torch.manual_seed(0)
        m = ms.MultiscreenLM(101, d_model=128, num_heads=2, num_layers=2, max_seq_len=2 * L,
                             ffn_dim=256).to(dev)
        with torch.no_grad():
            for blk in m.blocks:
                blk.attn.s_r.fill_(math.log(0.05))
                blk.attn.s_v.copy_(torch.tensor([math.log(1200.0), math.log(60.0)]))
        g = torch.Generator(device=dev).manual_seed(9)
        ids = torch.randint(0, 101, (2, T), device=dev, generator=g)
        labels = ids.clone()
        labels[:, :7] = -100
        out = m(ids, labels=labels)
        out["loss"].backward()
        ref_grads = {n: p.grad.clone() for n, p in m.named_parameters()}
        m.zero_grad(set_to_none=True)
        s0, s1 = rank * L, (rank + 1) * L
        with ms.sequence_parallel(L):
            out_s = m(ids[:, s0:s1], labels=labels[:, s0:s1])
        out_s["loss"].backward()
        assert rel_err(out_s["logits"], out["logits"][:, s0:s1]) <= 1e-4
        assert abs(out_s["loss"].item() - out["loss"].item()) <= 1e-5 * abs(out["loss"].item())
        for n, p in m.named_parameters():
            gsum = p.grad.clone()
            dist.all_reduce(gsum)
            assert rel_err(gsum, ref_grads[n]) <= 1e-4, n
        # prefill: the last rank's last-position logits are the prompt's
        with torch.no_grad():
            full_last = m.prefill(ids, None)
            with ms.sequence_parallel(L):
                sh_last = m.prefill(ids[:, s0:s1], None)
        if rank == world - 1:
            assert rel_err(sh_last, full_last) <= 1e-4
    finally:
        dist.destroy_process_group()


def test_two_gpu_halo_exchange_and_sharded_lm():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
