"""Expert-parallel prefill exchange (ep.moe_prefill_ep) with world_size 2 on
CPU over gloo: dispatch by expert owner, per-rank expert compute, combine.

The per-rank expert compute is the CPU oracle (the checker), injected through
moe_prefill_ep's `compute` argument; the result on every rank must equal the
single-process oracle over all tokens with the whole expert table.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import synthetic
from conftest import rel_err

E, TOPK, T_PER_RANK, WORLD = 8, 3, 6, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    blocks = synthetic.make_blocks(E, seed=61)
    s2 = synthetic.make_s2(E, seed=62, spread=True)
    T = T_PER_RANK * WORLD
    x = synthetic.make_x(T * 2560, seed=63, dtype=torch.float32).view(T, 2560).numpy()
    ti, tv = oracle.route(synthetic.zipf_logits(T, seed=64, n_experts=E), TOPK)
    return blocks, s2, x, ti, tv


def _cpu_compute(x_pairs, e_local, w, table, s2, L):
    out = oracle.moe_prefill(x_pairs.float().numpy(), e_local.numpy().astype(np.int32), w.numpy(),
                             table.numpy(), L * s2.shape[0], s2.numpy())
    return torch.from_numpy(out)


def _cpu_compute_ag(x_all, ti_loc, tv_all, table, s2, L):
    # pairs of other ranks' experts are marked -1: give them weight 0 on expert 0
    ti = ti_loc.numpy().astype(np.int32)
    w = np.where(ti >= 0, tv_all.numpy(), 0.0).astype(np.float32)
    out = oracle.moe_prefill(x_all.float().numpy(), np.maximum(ti, 0), w, table.numpy(), L * s2.shape[0], s2.numpy())
    return torch.from_numpy(out)


def _load(ti):
    """Calibration histogram for the load-aware placement: pairs per expert."""
    return np.bincount(ti.ravel(), minlength=E)


def _worker(rank, port, results, mode="a2a", placement="contiguous"):
    import ep
    os.environ["GLOO_SOCKET_IFNAME"] = "lo"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        blocks, s2, x, ti, tv = _inputs()
        shard = ep.ExpertShard(E, WORLD, rank, load=_load(ti) if placement == "lpt" else None)
        own = shard.experts
        toks = slice(rank * T_PER_RANK, (rank + 1) * T_PER_RANK)
        fn, compute = (ep.moe_prefill_ep, _cpu_compute) if mode == "a2a" else (ep.moe_prefill_ep_ag, _cpu_compute_ag)
        if mode == "ag2":    # the all-gather exchange pipelined over two slices of the tokens
            fn = lambda *a, **k: ep.moe_prefill_ep_ag(*a, chunks=2, **k)
        out = fn(torch.from_numpy(x[toks]), torch.from_numpy(ti[toks]).long(), torch.from_numpy(tv[toks]),
                 torch.from_numpy(blocks[own]), torch.from_numpy(s2[own]), 0, shard, compute=compute)
        results[rank] = out.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("placement", ["contiguous", "lpt"])
@pytest.mark.parametrize("mode", ["a2a", "ag", "ag2"])
def test_expert_parallel_prefill_matches_single_process(mode, placement):
    """mode a2a: all-to-all dispatch/combine; ag: all-gather + reduce-scatter;
    ag2: the same pipelined over two slices of the tokens.
    placement: contiguous ranges or the load-aware (LPT) placement."""
    blocks, s2, x, ti, tv = _inputs()
    # both ranks really exchange: some pairs of each rank's tokens live on the other rank
    owners = ti // (E // WORLD)
    assert (owners[:T_PER_RANK] == 1).any() and (owners[T_PER_RANK:] == 0).any()
    ref = oracle.moe_prefill(x, ti, tv, blocks, 0, s2)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, results, mode, placement)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        out = np.concatenate([results[r] for r in range(WORLD)])
    assert rel_err(out, ref) <= 1e-5


def test_expert_shard_placement():
    import ep
    sh = ep.ExpertShard(512, 8, 3)
    assert sh.per_rank == 64 and sh.first == 192
    assert sh.owner(191) == 2 and sh.owner(192) == 3 and sh.local(200) == 8
    with pytest.raises(ValueError):
        ep.ExpertShard(512, 3, 0)


def test_load_aware_placement_balances_zipf_routing():
    """LPT placement under BASELINE config 3 routing (2048 tokens, top-10 of
    512, Zipf(1.1)): every rank holds 512 / N experts, each expert exactly
    once, and the busiest rank's pairs come within 5 % of the mean at N = 8,
    where contiguous ranges leave it far above."""
    import ep
    both, _ = oracle.route(synthetic.zipf_logits(4096, seed=5), 10)     # one popularity permutation
    ti, calib = both[:2048], both[2048:]      # placement from other tokens than the ones measured
    load = np.bincount(ti.ravel(), minlength=512)
    for world in (2, 4, 8):
        lpt = ep.ExpertShard(512, world, 0, load=np.bincount(calib.ravel(), minlength=512))
        cont = ep.ExpertShard(512, world, 0)
        assert sorted(sum(lpt.lists, [])) == list(range(512))
        assert all(len(l) == 512 // world for l in lpt.lists)
        for r in range(world):
            sh = ep.ExpertShard(512, world, r, load=np.bincount(calib.ravel(), minlength=512))
            assert sh.lists == lpt.lists and sh.experts == lpt.lists[r]
            assert all(sh.owner(e) == r and sh.experts[sh.local(e)] == e for e in sh.experts)
        imb_lpt = lpt.rank_loads(load).max() / load.mean() / (512 / world)
        imb_cont = cont.rank_loads(load).max() / load.mean() / (512 / world)
        if world == 8:
            assert imb_lpt <= 1.05 < 1.2 <= imb_cont, (imb_lpt, imb_cont)
        assert imb_lpt <= imb_cont
