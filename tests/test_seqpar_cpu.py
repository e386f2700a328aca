"""Sequence-sharded causal attention: host logic on CPU ranks (gloo).

Each rank runs screening_attention_sharded on its block with the oracle's
windowed CPU restatement as the single-device attention, so what is checked
here is everything around the kernels: the halo plan (one and several hops),
the point-to-point exchange of K/V (and key-padding rows), the q_offset of
the interior and boundary calls, the reverse exchange of halo gradients, and
the global loss of a sharded LM batch.  Every rank compares its rows and
gradients with one unsharded oracle call over the whole sequence.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import load_pkg, rel_err


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_halo_plan_one_and_several_hops():
    ms = load_pkg()
    plan = ms.sequence_parallel.__module__
    from importlib import import_module
    sp = import_module(plan)
    # halo inside one block
    assert sp.halo_plan(1, 4, 100, 30) == ([(2, 70, 100)], [(0, 70, 100)])
    assert sp.halo_plan(0, 4, 100, 30) == ([(1, 70, 100)], [])
    assert sp.halo_plan(3, 4, 100, 30) == ([], [(2, 70, 100)])
    # halo of 2.5 blocks: three hops, the oldest block partially
    sends, recvs = sp.halo_plan(3, 4, 8, 20)
    assert recvs == [(0, 4, 8), (1, 0, 8), (2, 0, 8)]
    assert sum(hi - lo for _, lo, hi in recvs) == 20
    assert sends == []
    sends, recvs = sp.halo_plan(0, 4, 8, 20)
    assert sends == [(1, 0, 8), (2, 0, 8), (3, 4, 8)] and recvs == []
    # rank 1 with a halo longer than everything before it
    sends, recvs = sp.halo_plan(1, 4, 8, 20)
    assert recvs == [(0, 0, 8)]
    assert sp.halo_plan(2, 4, 8, 0) == ([], [])


def _inputs(B, T, H, D, ws, rs, seed, with_mask):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    k = q + 0.6 * torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    v = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    s_v = torch.log(torch.tensor(ws, dtype=torch.float64) - 1.0)
    s_r = torch.log(torch.tensor(rs, dtype=torch.float64) - 1.0)
    mask = (torch.rand(B, T, generator=g) < 0.15) if with_mask else None
    cot = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    return q, k, v, s_v, s_r, mask, cot


def _worker(rank, world, port, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = load_pkg()
        from oracle import screening_oracle as orc
        B, L, H, D, ws, rs, with_mask = case
        T = L * world
        q, k, v, s_v, s_r, mask, cot = _inputs(B, T, H, D, ws, rs, 5, with_mask)

        def attn(qq, kk, vv, r, w, causal, kpm, eps, q_offset):
            return orc.screening_core_windowed(qq, kk, vv, r, w, causal, kpm, eps, q_offset,
                                               chunk=16)

        # reference: one call over the whole sequence
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v, s_v, s_r)]
        qf, kf, vf, svf, srf = leaves
        y_full = attn(qf, kf, vf, torch.exp(srf) + 1, torch.exp(svf) + 1, True, mask, 1e-8, 0)
        (y_full * cot).sum().backward()

        s0, s1 = rank * L, (rank + 1) * L
        ql, kl, vl = (t[:, s0:s1].clone().requires_grad_(True) for t in (q, k, v))
        sv = s_v.clone().requires_grad_(True)
        sr = s_r.clone().requires_grad_(True)
        with ms.sequence_parallel(L) as shard:
            y = ms.screening_attention_sharded(ql, kl, vl, torch.exp(sr) + 1, torch.exp(sv) + 1,
                                               None if mask is None else mask[:, s0:s1],
                                               1e-8, shard=shard, attn_fn=attn)
        (y * cot[:, s0:s1]).sum().backward()
        gs = torch.stack([sr.grad, sv.grad])
        dist.all_reduce(gs)
        tol = 1e-10
        assert rel_err(y, y_full[:, s0:s1]) <= tol, ("y", rank)
        assert rel_err(ql.grad, qf.grad[:, s0:s1]) <= tol, ("dq", rank)
        assert rel_err(kl.grad, kf.grad[:, s0:s1]) <= tol, ("dk", rank)
        assert rel_err(vl.grad, vf.grad[:, s0:s1]) <= tol, ("dv", rank)
        assert rel_err(gs[0], srf.grad) <= tol, ("ds_r", rank)
        assert rel_err(gs[1], svf.grad) <= tol, ("ds_v", rank)
    finally:
        dist.destroy_process_group()


CASES = {
    # B, L, H, D, windows, sharpness, key padding
    "one_hop_w2": (2, 40, 2, 16, [10.0, 25.0], [1.3, 1.1], False),
    "one_hop_mask_w2": (1, 40, 2, 16, [10.0, 33.5], [1.3, 1.1], True),
    "multi_hop_w3": (1, 16, 2, 8, [40.0, 7.0], [1.2, 1.05], True),
    "multi_hop_w4": (1, 8, 1, 8, [20.5], [1.1], False),
}
WORLD = {"one_hop_w2": 2, "one_hop_mask_w2": 2, "multi_hop_w3": 3, "multi_hop_w4": 4}


@pytest.mark.parametrize("name", list(CASES))
def test_sharded_attention_matches_unsharded(name):
    world = WORLD[name]
    mp.spawn(_worker, args=(world, _free_port(), CASES[name]), nprocs=world, join=True)


def _ce_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = load_pkg()
        from importlib import import_module
        model_mod = import_module(ms.MultiscreenLM.__module__)
        g = torch.Generator().manual_seed(3)
        B, T, V = 2, 12, 7
        logits = torch.randn(B, T, V, generator=g, dtype=torch.float64)
        labels = torch.randint(0, V, (B, T), generator=g)
        labels[0, :5] = -100                      # uneven ignored counts across the shards
        full = logits.clone().requires_grad_(True)
        ref = torch.nn.functional.cross_entropy(full.view(-1, V), labels.view(-1),
                                                ignore_index=-100)
        ref.backward()
        L = T // world
        loc = logits[:, rank * L:(rank + 1) * L].clone().requires_grad_(True)
        with ms.sequence_parallel(L) as shard:
            loss = model_mod._sharded_mean_ce(loc, labels[:, rank * L:(rank + 1) * L], shard)
        loss.backward()
        assert abs(loss.item() - ref.item()) <= 1e-12
        assert rel_err(loc.grad, full.grad[:, rank * L:(rank + 1) * L]) <= 1e-12
    finally:
        dist.destroy_process_group()


def test_sharded_loss_is_the_global_mean():
    mp.spawn(_ce_worker, args=(3, _free_port()), nprocs=3, join=True)
