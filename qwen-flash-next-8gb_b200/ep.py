"""Expert-parallel batched prefill over N ranks (one process per GPU).

The layer's n_experts experts are split over N ranks, n_experts / N each
(ExpertShard: contiguous ranges, or a load-aware placement that spreads the
popular experts of a Zipf-like routing evenly); rank r holds the blocks of
its experts of every layer in its own table (block L * E_r + local index),
and the tokens are split across ranks (each rank routes its own tokens).
One MoE layer is then

  1. dispatch: every (token, slot) pair goes to the rank that owns its expert
     -- counts with one all-to-all, then the pairs' bf16 x rows and their
     (local expert, routing weight) with two uneven all-to-alls;
  2. expert compute: the received pairs run through the grouped GEMM
     (qmoe.moe_prefill) as tokens routed to one local expert each, weight
     applied;
  3. combine: the fp32 rows go back with one uneven all-to-all and are added
     onto their tokens (index_add_, fp32 atomics as in the reference loop,
     qwen_engine.py:849).

The result on each rank equals the single-GPU qmoe.moe_prefill of its tokens
(the reference's expert loop, qwen_engine.py:835-852) to fp32 accumulation
order.  Collectives run on the given process group (NCCL between GPUs; gloo
works for CPU tensors).  Batched decode uses the same exchange.

moe_prefill_ep_ag is the second exchange: every rank all-gathers all ranks'
tokens (x, expert ids, weights: fixed sizes), runs the grouped GEMM over all
of them with the pairs of other ranks' experts marked -1 (skipped), and a
reduce-scatter returns each rank the fp32 sums of its own tokens.  No split
sizes and no host synchronisation: a layer of it can be captured in a CUDA
graph.  It moves every token to every rank, so it suits small batches
(batched decode); the all-to-all exchange moves only routed rows.
"""
import ctypes

import numpy as np
import torch
import torch.distributed as dist

import qmoe
from _lib import DTYPE_BF16, DTYPE_F32, check, lib, on_device, require_cuda, stream_of


class ExpertShard:
    """Placement of one layer's experts over the ranks of a group.

    Every rank holds the same number of experts, n_experts / world, so all
    ranks' tables have one shape.  Without `load` the placement is contiguous
    ranges (rank r: experts [r E_r, (r + 1) E_r)).  With `load` (the expected
    pairs per expert, e.g. a histogram of routed calibration tokens) it is the
    longest-processing-time greedy under that capacity: experts in decreasing
    load, each to the rank with the least load so far among ranks with room.
    Under Zipf(1.1) popularity contiguous ranges leave the busiest rank
    1.4-1.9x the mean; the greedy brings it to within a few percent.

    experts: this rank's global expert ids in local (table) order.
    owner_of[e], local_of[e]: the rank holding expert e and its index there.
    """

    def __init__(self, n_experts, world, rank, load=None):
        if n_experts % world:
            raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside [0, {world})")
        self.n_experts, self.world, self.rank = n_experts, world, rank
        self.per_rank = n_experts // world
        if load is None:
            lists = [list(range(r * self.per_rank, (r + 1) * self.per_rank)) for r in range(world)]
        else:
            load = np.asarray(load, np.float64).reshape(-1)
            if load.shape[0] != n_experts:
                raise ValueError(f"load must have {n_experts} entries")
            lists = [[] for _ in range(world)]
            tot = np.zeros(world)
            # stable order: equal loads keep ascending expert ids (same placement on every rank)
            for e in np.argsort(-load, kind="stable"):
                room = [r for r in range(world) if len(lists[r]) < self.per_rank]
                r = min(room, key=lambda q: (tot[q], q))
                lists[r].append(int(e))
                tot[r] += load[e]
            lists = [sorted(l) for l in lists]
        self.lists = lists
        self.experts = lists[rank]
        self.owner_of = np.empty(n_experts, np.int64)
        self.local_of = np.empty(n_experts, np.int64)
        for r, l in enumerate(lists):
            for i, e in enumerate(l):
                self.owner_of[e], self.local_of[e] = r, i
        self.contiguous = load is None
        self._dev_maps = {}

    @property
    def first(self):
        """First expert of a contiguous placement (its table holds [first, first + per_rank))."""
        if not self.contiguous:
            raise AttributeError("a load-aware placement has no contiguous range; use .experts")
        return self.rank * self.per_rank

    def owner(self, e):
        return int(self.owner_of[e])

    def local(self, e):
        return int(self.local_of[e])

    def rank_loads(self, load):
        """Sum of `load` over each rank's experts (e.g. routed pairs per rank)."""
        load = np.asarray(load, np.float64).reshape(-1)
        return np.array([load[l].sum() for l in self.lists])

    def maps(self, dev):
        """Device tensors (owner int64 [E], local int64 [E], mine int32 [E]): the
        owner rank and local index of every expert, and this rank's local index
        of every expert it holds (-1 for the others)."""
        key = str(dev)
        if key not in self._dev_maps:
            mine = np.where(self.owner_of == self.rank, self.local_of, -1).astype(np.int32)
            self._dev_maps[key] = (torch.from_numpy(self.owner_of).to(dev), torch.from_numpy(self.local_of).to(dev),
                                   torch.from_numpy(mine).to(dev))
        return self._dev_maps[key]


def _a2a(out, inp, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


def moe_prefill_ep(x, ti, tv, table, s2, L, shard, group=None, compute=None):
    """One expert-parallel MoE layer for this rank's tokens.

    x bf16 [T, 2560] . ti int64/int32 [T, topk] global expert ids of layer L .
    tv bf16/fp32 [T, topk] . table u8 [n_layers * E_r, BLOCK] this rank's
    expert blocks . s2 f32 [E_r, 3] ws2 of this rank's experts of layer L .
    shard: ExpertShard of the group -> fp32 [T, 2560].

    `compute(x_pairs, e_local [R,1], w [R,1], table, s2, L)` defaults to
    qmoe.moe_prefill (the CUDA kernels); tests substitute a CPU checker to
    exercise the exchange with gloo.
    """
    compute = compute or qmoe.moe_prefill
    dev = x.device
    T, K = ti.shape
    N = shard.world
    ti_flat = ti.reshape(-1).long()
    owner, local, _ = shard.maps(dev)
    dest = owner[ti_flat]
    order = torch.argsort(dest, stable=True)                       # pairs grouped by owner rank
    send_counts = torch.bincount(dest, minlength=N)
    recv_counts = torch.empty_like(send_counts)
    _a2a(recv_counts, send_counts, None, None, group)
    send_splits, recv_splits = send_counts.tolist(), recv_counts.tolist()
    R = sum(recv_splits)

    tok = torch.div(order, K, rounding_mode="floor")
    x_send = x.index_select(0, tok)
    meta_send = torch.stack([local[ti_flat[order]].to(torch.int32),
                             tv.reshape(-1)[order].float().contiguous().view(torch.int32)], 1).contiguous()
    x_recv = torch.empty(R, x.shape[1], dtype=x.dtype, device=dev)
    meta_recv = torch.empty(R, 2, dtype=torch.int32, device=dev)
    _a2a(x_recv, x_send, recv_splits, send_splits, group)
    _a2a(meta_recv, meta_send, recv_splits, send_splits, group)

    e_local = meta_recv[:, 0:1].contiguous()
    w = meta_recv[:, 1:2].contiguous().view(torch.float32)
    y = compute(x_recv, e_local, w, table, s2, L) if R else torch.empty(0, x.shape[1], dtype=torch.float32,
                                                                        device=dev)
    y_back = torch.empty(T * K, x.shape[1], dtype=torch.float32, device=dev)
    _a2a(y_back, y.contiguous(), send_splits, recv_splits, group)
    out = torch.zeros(T, x.shape[1], dtype=torch.float32, device=dev)
    out.index_add_(0, tok, y_back)
    return out


def moe_prefill_ep_ag(x, ti, tv, table, s2, L, shard, group=None, compute=None, chunks=1):
    """Expert-parallel MoE layer through all-gather + reduce-scatter (no host sync).

    Arguments as moe_prefill_ep; every rank passes the same number of tokens T.
    `compute(x_all, ti_local [N*T, topk] (-1 = another rank's expert), tv_all,
    table, s2, L)` defaults to qmoe.moe_prefill.

    chunks > 1 pipelines the layer over that many slices of the tokens: every
    all-gather is queued first, then each slice's grouped GEMM runs as soon as
    its gather has landed and its reduce-scatter is queued behind it, so the
    NCCL stream carries one slice's exchange while the compute stream runs
    another slice's GEMMs (the GEMMs leave SMs for NCCL's kernels when the
    caller has set a prefill SM budget, _lib.set_prefill_sm_budget)."""
    compute = compute or qmoe.moe_prefill
    N = shard.world
    T, K = ti.shape
    dev = x.device
    gloo = dist.get_backend(group) == "gloo"      # gloo has no reduce_scatter_tensor
    mine = shard.maps(dev)[2]
    bounds = [T * c // max(chunks, 1) for c in range(max(chunks, 1) + 1)]
    pending = []
    for c in range(len(bounds) - 1):              # queue every all-gather first
        a, b = bounds[c], bounds[c + 1]
        x_all = torch.empty(N * (b - a), x.shape[1], dtype=x.dtype, device=dev)
        meta = torch.cat([ti[a:b].to(torch.int32), tv[a:b].float().contiguous().view(torch.int32)], 1).contiguous()
        meta_all = torch.empty(N * (b - a), 2 * K, dtype=torch.int32, device=dev)
        w1 = dist.all_gather_into_tensor(x_all, x[a:b].contiguous(), group=group, async_op=True)
        w2 = dist.all_gather_into_tensor(meta_all, meta, group=group, async_op=True)
        pending.append((a, b, x_all, meta_all, meta, w1, w2))
    out = torch.empty(T, x.shape[1], dtype=torch.float32, device=dev)
    scatters = []
    for a, b, x_all, meta_all, meta, w1, w2 in pending:
        w1.wait()                                 # the compute stream waits for the gather (no host wait)
        w2.wait()
        ti_loc = mine[meta_all[:, :K].long()]     # this rank's local index, -1 elsewhere
        tv_all = meta_all[:, K:].contiguous().view(torch.float32)
        y_all = compute(x_all, ti_loc, tv_all, table, s2, L)
        if gloo:
            dist.all_reduce(y_all, group=group)
            out[a:b].copy_(y_all[shard.rank * (b - a):(shard.rank + 1) * (b - a)])
        else:
            scatters.append((dist.reduce_scatter_tensor(out[a:b], y_all, group=group, async_op=True), y_all))
    for w, _ in scatters:
        w.wait()
    return out


class NcclComm:
    """An NCCL communicator made through libqfn's bootstrap (qfn_nccl_comm_init)
    on the current device, for the C-ABI expert-parallel layer
    (moe_prefill_ep_nccl).  Rank 0 makes the 128-byte id with unique_id() and
    every rank receives it by its own means."""

    @staticmethod
    def unique_id():
        buf = ctypes.create_string_buffer(128)
        check(lib().qfn_nccl_unique_id(buf), "qfn_nccl_unique_id")
        return buf.raw

    def __init__(self, world, rank, uid):
        if len(uid) != 128:
            raise ValueError("the NCCL unique id is 128 bytes")
        self.world, self.rank = world, rank
        self.ptr = ctypes.c_void_p()
        check(lib().qfn_nccl_comm_init(ctypes.byref(self.ptr), world, rank, ctypes.create_string_buffer(uid, 128)),
              "qfn_nccl_comm_init")

    def close(self):
        if self.ptr:
            check(lib().qfn_nccl_comm_destroy(self.ptr), "qfn_nccl_comm_destroy")
            self.ptr = ctypes.c_void_p()


def moe_prefill_ep_nccl(x, ti, tv, table, s2, L, shard, comm):
    """moe_prefill_ep_ag through the C ABI (qfn_moe_prefill_ep): the exchange
    and the grouped GEMM in one library call over an NCCL communicator
    (`comm`: an NcclComm or a raw ncclComm_t pointer), for engines that drive
    NCCL without torch.distributed.  Arguments as moe_prefill_ep."""
    for name, t in (("x", x), ("ti", ti), ("tv", tv), ("table", table), ("s2", s2)):
        require_cuda(name, t)
    T, K = ti.shape
    dev = x.device
    mine = shard.maps(dev)[2]
    E_r = s2.shape[0]
    out = torch.empty(T, x.shape[1], dtype=torch.float32, device=dev)
    L_ = lib()
    nbytes = L_.qfn_moe_prefill_ep_workspace(T, K, E_r, shard.world)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    ptr = comm.ptr if isinstance(comm, NcclComm) else comm
    with on_device(dev):
        rc = L_.qfn_moe_prefill_ep(x.data_ptr(), T, ti.data_ptr(), int(ti.dtype == torch.int64), tv.data_ptr(),
                                   DTYPE_BF16 if tv.dtype == torch.bfloat16 else DTYPE_F32, K, table.data_ptr(),
                                   table.shape[0], int(L) * E_r, s2.data_ptr(), E_r, mine.data_ptr(), len(mine), ptr,
                                   out.data_ptr(), ws.data_ptr(), nbytes, stream_of(out))
    check(rc, "qfn_moe_prefill_ep")
    return out
