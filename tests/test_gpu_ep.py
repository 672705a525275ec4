"""Expert-parallel prefill on 2 GPUs over NCCL: each rank holds half of the
layer's experts and its own tokens; the exchanged result must equal the CPU
oracle of the whole layer.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
import synthetic
from conftest import rel_err

pytestmark = pytest.mark.gpu

E, TOPK, T_PER_RANK, WORLD = 64, 10, 40, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    blocks = synthetic.make_blocks(E, seed=71)
    s2 = synthetic.make_s2(E, seed=72, spread=True)
    T = T_PER_RANK * WORLD
    x = synthetic.make_x(T * 2560, seed=73).view(T, 2560)
    ti, tv = oracle.route(synthetic.zipf_logits(T, seed=74, n_experts=E), TOPK)
    return blocks, s2, x, ti, tv


def _worker(rank, port, results, mode="a2a"):
    import datetime
    import torch.distributed as dist
    import ep
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        blocks, s2, x, ti, tv = _inputs()
        shard = ep.ExpertShard(E, WORLD, rank)
        own = shard.experts
        toks = slice(rank * T_PER_RANK, (rank + 1) * T_PER_RANK)
        fn = ep.moe_prefill_ep if mode == "a2a" else ep.moe_prefill_ep_ag
        comm = None
        if mode == "nccl_c":   # the C-ABI layer over libqfn's own NCCL communicator
            uid = [ep.NcclComm.unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            comm = ep.NcclComm(WORLD, rank, uid[0])
            fn = lambda *a: ep.moe_prefill_ep_nccl(*a, comm)
        if mode == "ag2":    # pipelined over two slices of the tokens, GEMMs on 132 SMs
            import _lib
            _lib.set_prefill_sm_budget(132)
            fn = lambda *a, **k: ep.moe_prefill_ep_ag(*a, chunks=2, **k)
        out = fn(x[toks].to(dev), torch.from_numpy(ti[toks]).long().to(dev),
                 torch.from_numpy(tv[toks]).to(dev).to(torch.bfloat16),
                 torch.from_numpy(blocks[own]).to(dev), torch.from_numpy(s2[own]).to(dev), 0, shard)
        torch.cuda.synchronize()
        results[rank] = out.cpu().numpy()
        if comm is not None:
            comm.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["a2a", "ag", "ag2", "nccl_c"])
def test_expert_parallel_prefill_two_gpus_matches_oracle(mode):
    """a2a: all-to-all dispatch/combine; ag: all-gather + reduce-scatter (pairs of
    the other rank's experts passed to the grouped GEMM as -1)."""
    import torch.multiprocessing as mp
    blocks, s2, x, ti, tv = _inputs()
    ref = oracle.moe_prefill(x.float().numpy(), ti, tv, blocks, 0, s2)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, results, mode)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        out = np.concatenate([results[r] for r in range(WORLD)])
    assert rel_err(out, ref) <= 1e-4


def test_c_abi_expert_parallel_layer_one_rank_matches_oracle():
    """qfn_moe_prefill_ep over a one-rank NCCL communicator (the exchange
    degenerates to copies; runs on a one-GPU box): all experts local."""
    import ep
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    blocks, s2, x, ti, tv = _inputs()
    comm = ep.NcclComm(1, 0, ep.NcclComm.unique_id())
    try:
        shard = ep.ExpertShard(E, 1, 0)
        own = shard.experts
        out = ep.moe_prefill_ep_nccl(x.to(dev), torch.from_numpy(ti).long().to(dev),
                                     torch.from_numpy(tv).to(dev).to(torch.bfloat16),
                                     torch.from_numpy(blocks[own]).to(dev), torch.from_numpy(s2[own]).to(dev), 0,
                                     shard, comm)
        torch.cuda.synchronize()
    finally:
        comm.close()
    ref = oracle.moe_prefill(x.float().numpy(), ti, tv, blocks, 0, s2)
    assert rel_err(out.cpu().numpy(), ref) <= 1e-4
