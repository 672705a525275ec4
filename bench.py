"""Benchmark of the quantized matrix-product path of qwen-flash-next-8gb on B200.

BASELINE metric: "bs1 MoE-layer us & HBM GB/s vs 8 TB/s; prefill tokens/s at
1/2/4/8 B200".  The headline line, at every N, is the batched prefill of one
NVFP4 MoE layer (config 3): 2,048 tokens per GPU of x ~ N(0,1) bf16, routed
top-10 of 512 experts with Zipf(1.1) popularity (fp32 logits = log p[perm] +
Gumbel noise, one popularity permutation shared by all ranks), through the
grouped SwiGLU expert GEMM and the weighted combine (qmoe.moe_prefill).

  N = 1  : one GPU holds the layer's 512 experts.
  N > 1  : expert-parallel, weak scaling: 512 / N experts per rank, placed by
           load (a histogram of routed calibration tokens, ep.ExpertShard),
           each rank routes its own 2,048 tokens; NCCL all-gather of the
           tokens, the grouped GEMM over the rank's experts, reduce-scatter of
           the fp32 sums (ep.moe_prefill_ep_ag; --ep-mode a2a: all-to-all).

  value  : tokens/s of the whole job (all ranks' tokens / max-over-ranks device
           time per step), inputs resident in HBM; every step reads >= 1.4 GB
           of distinct expert blocks at N = 1 (> 126 MB L2: no flush needed).
  e2e    : the same metric through the public call (qmoe.moe_prefill, or the
           ep.* exchange at N > 1) with x, ti, tv copied in from pinned host
           memory and the fp32 result copied back inside the timed region.
  parity : a seeded sample of every rank's tokens checked against the CPU
           oracle (tests' checker) after the timed region; the run exits
           non-zero when it fails.

Sub-records in the same line (same process, same expert table): at N = 1 the
bs=1 decode layer over the 48-layer stack (config 2, the first half of the
BASELINE metric), the FP8 GEMV (config 1), the decode MoE block, the delta
rule, the FP8 linear layer for T > 1 (config-1 weight shapes, 2,048 tokens)
and batched decode (config 4); at N > 1 batched decode expert-parallel
(config 4).  Each carries its own roofline, e2e and parity.

`--workload decode|gemv|batch-decode|fp8-linear|decode-block|deltanet` prints
one of those alone.
`--impl reference` times the reference's CPU path (the C restatement in
oracle/) on this host's cores on a bounded sample of the same workload.
"""
import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen-flash-next-8gb_b200")
sys.path.insert(0, PKG)

HID, INTER, BLOCK = 2560, 640, 2764800
TOPK, N_EXPERTS, N_LAYERS = 10, 512, 48
WS2 = 1.0 / 448.0
# algorithmic bytes of one decode layer: 10 expert blocks + s2 + coef + x (bf16) + out (fp32)
LAYER_BYTES = TOPK * BLOCK + TOPK * 12 + TOPK * 4 + HID * 2 + HID * 4
PF_FLOP_PER_PAIR = 2 * 3 * INTER * HID          # gate, up and down: 9,830,400 FLOP per (token, expert)
# our kernel launches per call
PF_LAUNCHES = 7        # routing count / plan / scatter, x gather, gate/up GEMM, h packing, down GEMM
PF_METRIC = "prefill tokens/s (one NVFP4 MoE layer: 2048 tokens per GPU, top-10 of 512 experts, Zipf(1.1))"
DECODE_METRIC = "bs1 decode MoE-layer HBM GB/s (48-layer stack, experts resident in HBM)"
GEMV_METRIC = "FP8 E4M3 row-scaled GEMV HBM GB/s (12288x2560, bs=1, per call)"
BD_METRIC = "batched-decode tokens/s (batch 64 per GPU, 48-layer NVFP4 MoE stack, top-10 of 512 uniform)"
GEMV_SHAPES = ((12288, 2560), (2560, 4096))   # the DeltaNet projections of config 1 (N x K)
GEMV_COPIES = 8                                # weight copies rotated per shape (8 x 31.5 MB > 2 x L2)
GEMV_CALLS = 64                                # calls per graph replay (one step)
LIN_COPIES = 4

# DRAM bytes (read + written) per launch of the dominant kernel of each
# record, from ncu captures of the same shapes (None: not captured).
TRAFFIC = {
    "decode": 27.72e6,              # moe_decode_slice, one layer (K = 10)
    "prefill": 1.7469e9,            # pf_gemm<0> + pf_gemm<1>, one config-3 layer
    "gemv_ratio": 31.555328e6 / 31.536128e6,   # gemv_stream_kernel (12288 x 2560) DRAM bytes / algorithmic bytes
    # route logits + select + moe_decode_slice + shared gate/up + down, one layer
    "decode_block": 2.635e6 + 0.023e6 + 27.72e6 + 6.581e6 + 3.299e6,
    # deltanet_step_kernel: the state's reads (its writes reach DRAM from L2 after the launch)
    "deltanet": 2.140e6,
}
PARITY_TOL = 1e-3       # north_star: max |err| <= 1e-3 x RMS of the oracle's output


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="qfn", choices=["qfn", "reference"])
    p.add_argument("--workload", default="prefill",
                   choices=["prefill", "decode", "gemv", "batch-decode", "fp8-linear", "decode-block", "deltanet"],
                   help="prefill: config 3, the headline (with sub-records); the others print one record alone")
    p.add_argument("--no-sub", action="store_true", help="headline only, no sub-records")
    p.add_argument("--sub-steps", type=int, default=64, help="timed steps of each sub-record")
    p.add_argument("--tokens", type=int, default=2048, help="prefill: tokens per GPU per step (config 3: 2048)")
    p.add_argument("--batch", type=int, default=64, help="batch-decode: tokens per GPU per step (config 4: 64)")
    p.add_argument("--n-layers", type=int, default=N_LAYERS, help="decode / batch-decode layers (48 = full)")
    p.add_argument("--routes", type=int, default=32, help="decode: distinct routed steps (cycled)")
    p.add_argument("--e2e-steps", type=int, default=32)
    p.add_argument("--ep-mode", default="ag", choices=["ag", "a2a"],
                   help="expert-parallel exchange: ag = all-gather + reduce-scatter (no host sync), "
                        "a2a = all-to-all of routed rows (host sync for split sizes)")
    p.add_argument("--ep-chunks", type=int, default=1,
                   help="ag exchange: token slices pipelined so one slice's exchange overlaps another's GEMMs")
    p.add_argument("--ep-sm-budget", type=int, default=-16,
                   help="SMs for the persistent prefill GEMMs under expert parallelism with --ep-chunks > 1 "
                        "(<= 0: all SMs minus that many, left to NCCL's kernels)")
    p.add_argument("--placement", default="lpt", choices=["lpt", "contiguous"],
                   help="expert placement over ranks for prefill: load-aware (LPT) or contiguous ranges")
    p.add_argument("--parity-tokens", type=int, default=16, help="tokens per rank checked against the oracle")
    p.add_argument("--cpu-tokens", type=int, default=128, help="prefill tokens timed for the CPU baseline")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--variant", type=int, default=0, help="decode kernel path: 0 auto, 4 slice, 2 CUDA-core")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, kind) from MEASURED_PEAKS.json, else the pool's fallback."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, cuda_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            try:
                p = torch.cuda.get_device_properties(cuda_index)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                r = self._reasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nvml:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.nvml:
            self._stop.set()
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- run context
class Ctx:
    """Device, process group and the shared 48-layer expert table of one rank."""

    def __init__(self, args):
        import torch
        self.args = args
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist
        self._table48 = None
        self.failed = []

    def table48(self):
        """All n_layers x 512 experts of the stack (63.3 GiB at 48 layers), config-0 blocks."""
        if self._table48 is None:
            from expert_table import ExpertTable
            t = ExpertTable(K=TOPK, dev=self.dev, n_layers=self.args.n_layers, n_experts=N_EXPERTS)
            t.fill_synthetic(seed=self.args.seed)
            self._table48 = t
        return self._table48

    def barrier(self):
        import torch
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(self, v):
        import torch
        if self.dist is None:
            return v
        t = torch.tensor([float(v)], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def min_over_ranks(self, v):
        return -self.max_over_ranks(-v)

    def timed(self, fn, steps, warmup, clocks=False):
        """Device time per step (ms) of fn(i): warm-up, barrier + sync, CUDA events on
        the current stream around `steps` calls, sync, max over ranks."""
        import torch
        for i in range(max(warmup, 3)):
            fn(i)
        self.barrier()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(self.local) if clocks else None
        if clk:
            clk.__enter__()
        torch.cuda.nvtx.range_push("timed")
        e0.record(st)
        for i in range(steps):
            fn(i)
        e1.record(st)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        if clk:
            clk.__exit__()
        ms = self.max_over_ranks(e0.elapsed_time(e1) / steps)
        return (ms, clk.summary()) if clocks else ms

    def parity(self, errs, argmax_ok, n):
        """Max-over-ranks parity summary; records a failure."""
        err = self.max_over_ranks(max(errs) if errs else 0.0)
        ok = self.min_over_ranks(1.0 if argmax_ok else 0.0) > 0.5
        total = int(round(self.max_over_ranks(n))) * self.world
        res = {"max_err_rms": err, "argmax_equal": ok, "tol": PARITY_TOL, "checked_rows": total,
               "checker": "oracle/ C restatement of the reference path on sampled rows", "pass": err <= PARITY_TOL and ok}
        return res


def rel_err(a, ref):
    import numpy as np
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(a - ref)) / np.sqrt(np.mean(ref * ref)))


def oracle_mod(threads):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    oracle.threads(threads)
    return oracle


def host_threads(ctx):
    return max(1, (os.cpu_count() or 1) // max(1, ctx.world))


class OracleSlices:
    """The reference's expert loop (qwen_engine.py:838-852) on the CPU, one balanced slice
    of a layer at a time: the layer's experts are split into `n` slices of equal expert
    count and near-equal pairs (the load-aware placement of ep.ExpertShard), and a slice
    runs every pair routed to its experts (block dequant + fp32 GEMMs + index_add into
    the tokens' rows).  A slice is ~1/n of the full batch's work at the full batch's
    expert reuse, so tokens/s = T / (n x time per slice)."""

    def __init__(self, oracle, x, ti, tv, block_fn, n=64):
        import numpy as np
        import ep
        self.oracle, self.x, self.ti, self.tv, self.block_fn, self.n = oracle, x, ti, tv, block_fn, n
        load = np.bincount(ti.ravel(), minlength=N_EXPERTS)
        self.lists = ep.ExpertShard(N_EXPERTS, n, 0, load=load).lists
        self.out = np.zeros((x.shape[0], HID), np.float32)

    def blocks(self, i):
        return [self.block_fn(e) for e in self.lists[i % self.n]]

    def run(self, i):
        import numpy as np
        experts = np.asarray(self.lists[i % self.n])
        t, k = np.nonzero(np.isin(self.ti, experts))
        if len(t) == 0:
            return
        used = np.unique(self.ti[t, k])
        y = self.oracle.moe_prefill(self.x[t], np.searchsorted(used, self.ti[t, k]).astype(np.int32)[:, None],
                                    self.tv[t, k][:, None], np.stack([self.block_fn(int(e)) for e in used]), 0,
                                    np.full((len(used), 3), WS2, np.float32))
        np.add.at(self.out, t, y)


# ---------------------------------------------------------------- routing inputs
def zipf_routes(dev, seed, rank_seed, T, R):
    """R steps of T tokens: fp32 logits = log p[perm] + Gumbel, p_r ~ r^-1.1 with one
    popularity permutation (from `seed`, shared by every rank), the noise and x from
    `rank_seed`; routed top-10 + renormalised bf16 weights (the engine's router)."""
    import torch
    import routing
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    logp = -1.1 * torch.log(torch.arange(1, N_EXPERTS + 1, device=dev, dtype=torch.float64))
    logp = (logp - torch.logsumexp(logp, 0)).float()
    perm = torch.randperm(N_EXPERTS, device=dev, generator=g)
    lp = logp[perm][None]
    g.manual_seed(rank_seed)
    xs, tis, tvs = [], [], []
    for _ in range(R):
        u = torch.rand(T, N_EXPERTS, device=dev, generator=g).clamp_(1e-12, 1 - 1e-7)
        ti, tv = routing.route(lp - torch.log(-torch.log(u)), TOPK)
        xs.append(torch.randn(T, HID, device=dev, generator=g).to(torch.bfloat16))
        tis.append(ti)
        tvs.append(tv)
    return xs, tis, tvs


def prefill_parity(ctx, out, x, ti, tv, layer, n, seed):
    """out rows of n seeded tokens against the oracle's expert loop (qwen_engine.py:835-852);
    the blocks the tokens route to are regenerated from their (layer, expert) seeds."""
    import numpy as np
    import torch
    import synthetic
    oracle = oracle_mod(host_threads(ctx))
    T = x.shape[0]
    rng = np.random.Generator(np.random.PCG64(seed))
    tok = np.sort(rng.choice(T, size=min(n, T), replace=False))
    ti_s = ti[torch.from_numpy(tok).to(ti.device)].cpu().numpy()
    used = np.unique(ti_s)
    blocks = torch.stack([synthetic.expert_block(layer, int(e), ctx.args.seed, ctx.dev) for e in used]).cpu().numpy()
    ref = oracle.moe_prefill(x[tok].float().cpu().numpy(), np.searchsorted(used, ti_s).astype(np.int32),
                             tv[tok].float().cpu().numpy(), blocks, 0, np.full((len(used), 3), WS2, np.float32))
    got = out[tok].cpu().numpy()
    return rel_err(got, ref), bool((got.argmax(1) == ref.argmax(1)).all()), len(tok)


# ---------------------------------------------------------------- prefill (config 3): the headline
def prefill_record(ctx):
    import numpy as np
    import torch
    import qmoe
    from expert_table import ExpertTable
    args, dev, world, rank = ctx.args, ctx.dev, ctx.world, ctx.rank
    T, R = args.tokens, 4
    shard = ep_fn = None
    if world == 1:
        table = ctx.table48()
        s2 = table.s2[0]
    else:
        import ep
        load = None
        if args.placement == "lpt":
            # calibration: a histogram of 4,096 routed tokens of the same popularity (same on every rank)
            _, cti, _ = zipf_routes(dev, args.seed + 7, args.seed + 99, 4096, 1)
            load = torch.bincount(cti[0].view(-1), minlength=N_EXPERTS).cpu().numpy()
        shard = ep.ExpertShard(N_EXPERTS, world, rank, load=load)
        table = ExpertTable(K=TOPK, dev=dev, n_layers=1, n_experts=shard.per_rank)
        table.fill_synthetic(seed=args.seed, experts=shard.experts)
        s2 = table.s2[0]
        if args.ep_mode == "ag":
            ep_fn = lambda *a: ep.moe_prefill_ep_ag(*a, chunks=args.ep_chunks)
            ep_fn.__name__ = "moe_prefill_ep_ag"
            if args.ep_chunks > 1:
                import _lib
                sms = torch.cuda.get_device_properties(dev).multi_processor_count
                _lib.set_prefill_sm_budget(args.ep_sm_budget if args.ep_sm_budget > 0 else sms + args.ep_sm_budget)
        else:
            ep_fn = ep.moe_prefill_ep
    xs, tis, tvs = zipf_routes(dev, args.seed + 7, args.seed + 8 + 1000 * rank, T, R)

    def call(x, ti, tv):
        if shard is None:
            return qmoe.moe_prefill(x, ti, tv, table.slots, s2, 0)
        return ep_fn(x, ti, tv, table.slots, s2, 0, shard)

    ms, clk = ctx.timed(lambda i: call(xs[i % R], tis[i % R], tvs[i % R]), args.steps, args.warmup, clocks=True)

    # work per step on this rank: its experts' distinct blocks + activations in + fp32 out
    if shard is None:
        distinct = [int(torch.unique(t).numel()) for t in tis]
        pairs_rank = [T * TOPK] * R
        rows = T
    else:
        # all ranks' tokens pass through every rank's grouped GEMM (ag) -- count this rank's experts' pairs
        mine = shard.maps(dev)[2]
        all_ti = [torch.cat(ctx_all_gather(ctx, t)) for t in tis]
        distinct = [int(torch.unique(t[mine[t] >= 0]).numel()) for t in all_ti]
        pairs_rank = [int((mine[t] >= 0).sum()) for t in all_ti]
        rows = world * T if args.ep_mode == "ag" else T
    step_bytes = sum(d * BLOCK for d in distinct) / R + rows * HID * (2 + 4)
    pairs = sum(pairs_rank) / R
    tok_s = world * T / (ms * 1e-3)
    tflops_rank = pairs * PF_FLOP_PER_PAIR / (ms * 1e-3) / 1e12
    gbs_rank = step_bytes / (ms * 1e-3) / 1e9
    hbm, tc, kind = peaks()

    # parity: step 0's output for a sample of this rank's tokens
    out0 = call(xs[0], tis[0], tvs[0])
    torch.cuda.synchronize()
    e, ok, n = prefill_parity(ctx, out0, xs[0], tis[0], tvs[0], 0, args.parity_tokens, 1000 + rank)
    parity = ctx.parity([e], ok, n)
    del out0

    # e2e: host buffers in (x, ti, tv) and the fp32 result out, every step,
    # pipelined as a serving loop runs it: step i + 1's inputs copy in on one
    # copy stream and step i - 1's result copies out on another while step i
    # computes (two device buffer sets); the timed region holds E whole steps,
    # the first step's copy in and the last step's copy out included.
    h_x = [x.cpu().pin_memory() for x in xs]
    h_ti = [t.cpu().pin_memory() for t in tis]
    h_tv = [t.cpu().pin_memory() for t in tvs]
    h_out = [torch.empty(T, HID, dtype=torch.float32).pin_memory() for _ in range(2)]
    d_in = [(torch.empty_like(xs[0]), torch.empty_like(tis[0]), torch.empty_like(tvs[0])) for _ in range(2)]
    h2d = d_in[0][0].numel() * 2 + d_in[0][1].numel() * 8 + d_in[0][2].numel() * 2
    d2h = T * HID * 4
    E = min(args.e2e_steps, args.steps)
    e2e_pipelined = make_e2e_pipeline(
        lambda i, k: (d_in[k][0].copy_(h_x[i % R], non_blocking=True), d_in[k][1].copy_(h_ti[i % R], non_blocking=True),
                      d_in[k][2].copy_(h_tv[i % R], non_blocking=True)),
        lambda i, k: call(*d_in[k]),
        lambda i, k, out: h_out[k].copy_(out, non_blocking=True))
    ms_e2e = ctx.timed(lambda i: e2e_pipelined(E), 1, 2) / E

    breakdown = ep_breakdown(ctx, shard, table, s2, xs[0], tis[0], tvs[0]) if shard is not None and \
        args.ep_mode == "ag" else None
    rec = {
        "metric": PF_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 tensor-core products of nvfp4 weights (exact) and bf16 activations, "
                                      "fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"prefill-moe-1L (config 3): {T} tokens per GPU, top-{TOPK} of {N_EXPERTS}, Zipf(1.1)",
                   "pairs_per_gpu": T * TOPK, "distinct_experts_per_step_rank": sum(distinct) / R,
                   "tflops_per_gpu": tflops_rank, "hbm_gbs_per_gpu": gbs_rank, "bytes_per_step_rank": step_bytes,
                   "l2": f"no flush: each step reads {step_bytes / 1e9:.2f} GB per rank (the distinct expert "
                         "blocks of its routing and the activations; > 126 MB L2)",
                   "parallelism": "single GPU" if world == 1 else
                   f"expert-parallel x{world} ({'all-gather + reduce-scatter' if args.ep_mode == 'ag' else 'all-to-all'}"
                   f" over NCCL, {args.placement} placement, {N_EXPERTS // world} experts per rank)"},
        "e2e": {"value": world * T / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E, "ms_per_step": ms_e2e,
                "path": ("qmoe.moe_prefill" if world == 1 else f"ep.{ep_fn.__name__}") +
                        " (public API) with pinned host x, ti, tv in and the fp32 result out, pipelined over two "
                        "buffer sets (copies in and out on two copy streams overlap the neighbouring steps' compute)"},
        "roofline": {"bound": "hbm", "achieved": gbs_rank, "peak": hbm, "unit": "GB/s", "frac": gbs_rank / hbm,
                     "peak_kind": kind, "tensor_tflops": tflops_rank, "tensor_peak": tc,
                     "tensor_frac": tflops_rank / tc,
                     "traffic": TRAFFIC["prefill"] if world == 1 and T == 2048 else None,
                     "kernel": "qfn_moe_prefill, one layer (7 launches; the time is the whole layer's)" +
                               ("" if world == 1 else " + the NCCL exchange")},
        "parity": parity,
        "gpu_launches": args.steps * PF_LAUNCHES,
        "clocks": clk,
    }
    if shard is not None:
        mean_pairs = T * TOPK
        rec["config"]["pairs_per_rank_max_over_mean"] = ctx.max_over_ranks(sum(pairs_rank) / R) / mean_pairs
        rec["config"]["ep_chunks"] = args.ep_chunks if args.ep_mode == "ag" else None
        rec["config"]["ep_breakdown_ms"] = breakdown
    if world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = prefill_cpu_baseline(ctx, xs[0], tis[0], tvs[0])
    if not parity["pass"]:
        ctx.failed.append("prefill")
    return rec


def ep_breakdown(ctx, shard, table, s2, x, ti, tv, reps=10):
    """The unpipelined all-gather exchange's parts timed one at a time (max over ranks,
    CUDA events): the two all-gathers, the grouped GEMM on the gathered tokens, the
    reduce-scatter of the fp32 sums -- what the expert-parallel step is made of."""
    import torch
    import qmoe
    import _lib
    dist, dev, N = ctx.dist, ctx.dev, ctx.world
    T, K = ti.shape
    x_all = torch.empty(N * T, x.shape[1], dtype=x.dtype, device=dev)
    meta = torch.cat([ti.to(torch.int32), tv.float().contiguous().view(torch.int32)], 1).contiguous()
    meta_all = torch.empty(N * T, 2 * K, dtype=torch.int32, device=dev)
    out = torch.empty(T, x.shape[1], dtype=torch.float32, device=dev)
    mine = shard.maps(dev)[2]

    def gather():
        dist.all_gather_into_tensor(x_all, x.contiguous())
        dist.all_gather_into_tensor(meta_all, meta)

    gather()
    ti_loc = mine[meta_all[:, :K].long()]
    tv_all = meta_all[:, K:].contiguous().view(torch.float32)
    _lib.set_prefill_sm_budget(0)
    y = qmoe.moe_prefill(x_all, ti_loc, tv_all, table.slots, s2, 0)
    parts = {"all_gather": gather,
             "grouped_gemm": lambda: qmoe.moe_prefill(x_all, ti_loc, tv_all, table.slots, s2, 0),
             "reduce_scatter": lambda: dist.reduce_scatter_tensor(out, y)}
    res = {k: round(ctx.timed(lambda i, f=f: f(), reps, 2), 4) for k, f in parts.items()}
    if ctx.args.ep_chunks > 1:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        b = ctx.args.ep_sm_budget
        _lib.set_prefill_sm_budget(b if b > 0 else sms + b)
    return res


def make_e2e_pipeline(copy_in, compute, copy_out):
    """A serving loop over n steps with two device buffer sets: copy_in(i, k)
    (host -> set k) on a copy stream, compute(i, k) -> device result on the
    current stream, copy_out(i, k, result) (-> host buffer k) on a second copy
    stream; step i + 1's copy in and step i - 1's copy out overlap step i's
    compute.  The returned run(n) leaves the current stream waiting for the
    last copy out."""
    import torch
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    outs = [None, None]

    def run(n):
        cur = torch.cuda.current_stream()   # (inside a graph capture: the capturing stream)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            copy_in(0, 0)
            ready[0].record(s_in)
        for i in range(n):
            k = i & 1
            if i + 1 < n:                       # the next step's inputs, once step i - 1 has read set 1 - k
                with torch.cuda.stream(s_in):
                    if i >= 1:
                        s_in.wait_event(done[1 - k])
                    copy_in(i + 1, 1 - k)
                    ready[1 - k].record(s_in)
            cur.wait_event(ready[k])
            if i >= 2:                          # result buffer k is free once step i - 2's copy out is done
                cur.wait_event(copied[k])
            outs[k] = compute(i, k)
            done[k].record(cur)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[k])
                copy_out(i, k, outs[k])
                copied[k].record(s_out)
        cur.wait_stream(s_out)
    return run


def ctx_all_gather(ctx, t):
    import torch
    out = [torch.empty_like(t) for _ in range(ctx.world)]
    ctx.dist.all_gather(out, t.contiguous())
    return out


def prefill_cpu_baseline(ctx, x, ti, tv):
    """The C oracle's restatement of the expert loop (qwen_engine.py:838-852) on this host's
    cores: 8 of the 64 balanced expert slices of step 0 (each slice: all pairs of its
    experts at the full batch's reuse), scaled to the whole layer."""
    import numpy as np
    cores = host_threads(ctx)
    oracle = oracle_mod(cores)
    table = ctx.table48()
    cache = {}

    def block(e):
        if e not in cache:
            cache[e] = table.slots[e].cpu().numpy()
        return cache[e]

    sl = OracleSlices(oracle, x.float().cpu().numpy(), ti.cpu().numpy(), tv.float().cpu().numpy(), block)
    m = 8
    for i in range(m):
        sl.blocks(i)             # device -> host copies stay out of the timed region
    t0 = time.perf_counter()
    for i in range(m):
        sl.run(i)
    dt = (time.perf_counter() - t0) / m
    T = x.shape[0]
    return {"value": T / (sl.n * dt), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{m} of {sl.n} balanced expert slices of step 0 ({T} tokens, top-{TOPK}; each slice: "
                      f"block dequant + fp32 GEMMs + index_add for every pair of its experts), "
                      f"{dt:.2f} s per slice, scaled x{sl.n}"}


# ---------------------------------------------------------------- bs=1 decode (config 2)
def decode_record(ctx, steps):
    import numpy as np
    import torch
    import qmoe
    import routing
    args, dev = ctx.args, ctx.dev
    table = ctx.table48()
    L, R = args.n_layers, args.routes
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 1)
    # Zipf(1.1) popularity, one permutation per layer; Gumbel-top-10 per step
    logp = -1.1 * torch.log(torch.arange(1, N_EXPERTS + 1, device=dev, dtype=torch.float64))
    logp = (logp - torch.logsumexp(logp, 0)).float()
    perm = torch.stack([torch.randperm(N_EXPERTS, device=dev, generator=g) for _ in range(L)])
    u = torch.rand(R, L, N_EXPERTS, device=dev, generator=g).clamp_(1e-12, 1 - 1e-7)
    ti, tv = routing.route((logp[perm][None] - torch.log(-torch.log(u))).view(R * L, N_EXPERTS), TOPK)
    ti = ti.view(R, L, TOPK)
    layer = torch.arange(L, device=dev).view(1, L, 1)
    sidx = (ti + layer * N_EXPERTS).to(torch.int32).contiguous()
    s2 = table.s2[layer.expand_as(ti), ti].contiguous()              # [R, L, K, 3]
    coef = tv.view(R, L, TOPK).float().contiguous()
    x = torch.randn(R, L, HID, device=dev, generator=g).to(torch.bfloat16)
    hb = torch.empty(TOPK, INTER, device=dev)
    ob = torch.empty(TOPK, HID, device=dev)

    def layer_call(r, l, xl=None):
        xl = x[r, l] if xl is None else xl
        if args.variant:
            return qmoe._moe_decode(table.slots, sidx[r, l], s2[r, l], coef[r, l], xl, hb, args.variant)
        return qmoe.moe_decode(table.slots, sidx[r, l], s2[r, l], coef[r, l], xl, hb, ob)

    def step_eager(r):
        for l in range(L):
            layer_call(r, l)

    step_eager(0)
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs = []
    for r in range(R):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, pool=pool):
            step_eager(r)
        graphs.append(gr)
    ms, clk = ctx.timed(lambda i: graphs[i % R].replay(), steps, args.warmup, clocks=True)
    us_layer = ms * 1e3 / L
    step_bytes = L * LAYER_BYTES

    # parity: two layers of route 0 against the oracle
    oracle = oracle_mod(host_threads(ctx))
    errs, ok = [], True
    for l in (0, L - 1):
        y = layer_call(0, l).cpu().numpy()
        blocks = table.slots[sidx[0, l].long()].cpu().numpy()
        ref = oracle.moe_decode(blocks, np.arange(TOPK, dtype=np.int32), s2[0, l].cpu().numpy(),
                                coef[0, l].cpu().numpy(), x[0, l].float().cpu().numpy())
        errs.append(rel_err(y, ref))
        ok = ok and int(y.argmax()) == int(ref.argmax())
    parity = ctx.parity(errs, ok, 2)

    # e2e: public API, host inputs copied in and outputs copied out every step
    E = min(args.e2e_steps, R)
    h_x = x[:E].cpu().pin_memory()
    h_sidx, h_s2, h_coef = sidx[:E].cpu().pin_memory(), s2[:E].cpu().pin_memory(), coef[:E].cpu().pin_memory()
    d_in = [(torch.empty_like(x[0]), torch.empty_like(sidx[0]), torch.empty_like(s2[0]), torch.empty_like(coef[0]))
            for _ in range(2)]
    h_out = torch.empty(E, L, HID).pin_memory()
    h2d = d_in[0][0].numel() * 2 + d_in[0][1].numel() * 4 + d_in[0][2].numel() * 4 + d_in[0][3].numel() * 4

    def e2e_in(i, k):
        for d, h in zip(d_in[k], (h_x, h_sidx, h_s2, h_coef)):
            d.copy_(h[i % E], non_blocking=True)

    def e2e_compute(i, k):
        dx, ds, d2, dc = d_in[k]
        return torch.stack([qmoe.moe_decode(table.slots, ds[l], d2[l], dc[l], dx[l], hb, ob) for l in range(L)])

    # the steps as a serving loop runs them: each step's copies in, its 48 calls
    # and its copy out, pipelined over two buffer sets (the next step's inputs and
    # the previous step's outputs copy during this step's layers), E steps in one
    # CUDA graph (host launch cost off the critical path)
    e2e_pipelined = make_e2e_pipeline(e2e_in, e2e_compute,
                                      lambda i, k, out: h_out[i % E].copy_(out, non_blocking=True))
    e2e_pipelined(2)
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_pipelined(E)
    ms_e2e = ctx.timed(lambda i: e2e_graph.replay(), 4, 2) / E
    del e2e_graph
    hbm, _, kind = peaks()
    achieved = LAYER_BYTES / (us_layer * 1e-6) / 1e9
    rec = {
        "metric": DECODE_METRIC, "value": ctx.world * step_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "us_per_layer": us_layer, "ms_per_step": ms, "steps": steps, "higher_is_better": True,
        "dtype": "nvfp4 weights (e2m1 + e4m3 scales), fp32 accumulate",
        "config": {"workload": f"decode-moe-{L}L (config 2): bs=1, top-{TOPK} of {N_EXPERTS}, Zipf(1.1), "
                               f"{L}x{N_EXPERTS} experts resident ({L * N_EXPERTS * BLOCK / 2**30:.1f} GiB); "
                               f"a step = {L} layers in one CUDA graph",
                   "routes": R, "layer_bytes": LAYER_BYTES,
                   "l2": "no flush: each step streams 1.33 GB of distinct expert bytes (> 126 MB L2)"},
        "e2e": {"value": E * step_bytes / (ms_e2e * E * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": L * HID * 4, "ms_per_step": ms_e2e,
                "path": "qmoe.moe_decode per layer (public API) with pinned host x, sidx, s2, coef in and the 48 "
                        "fp32 outputs out every step, steps pipelined over two buffer sets (copies on two copy "
                        f"streams), {E} steps per CUDA graph"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "frac_of_8tbs": achieved / 8000.0,
                     "traffic": TRAFFIC["decode"] if args.variant in (0, 4) else None, "per_launch_bytes": LAYER_BYTES,
                     "kernel": "moe_decode_slice (one launch per decode layer)" if args.variant in (0, 4)
                     else "moe_gate_up_generic + moe_down_generic"},
        "parity": parity,
        "gpu_launches": steps * L * (2 if args.variant == 2 else 1),
        "clocks": clk,
    }
    if ctx.world == 1 and not args.no_cpu_baseline:
        n = 2
        layers = [(table.slots[sidx[0, l].long()].cpu().numpy(), np.arange(TOPK, dtype=np.int32),
                   s2[0, l].cpu().numpy(), coef[0, l].cpu().numpy(), x[0, l].float().cpu().numpy()) for l in range(n)]
        t0 = time.perf_counter()
        for a in layers:
            oracle.moe_decode(*a)
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": n * LAYER_BYTES / dt / 1e9, "unit": "GB/s", "cores": host_threads(ctx),
                               "kind": "port", "sample": f"{n} layers of routed step 0 (C oracle: dequantize + fp32 "
                                                         f"SwiGLU + combine), {dt / n * 1e3:.1f} ms/layer"}
    if not parity["pass"]:
        ctx.failed.append("decode")
    del graphs
    return rec


# ---------------------------------------------------------------- FP8 GEMV (config 1)
def gemv_bytes(N, K):
    return N * K + 4 * N + 2 * K + 2 * N       # weights + row scales + x (bf16) + y (bf16)


def gemv_record(ctx, steps):
    import numpy as np
    import torch
    import fp8gemv
    import synthetic
    args, dev = ctx.args, ctx.dev
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 11)
    per_shape = {}
    for (N, K) in GEMV_SHAPES:
        qs, ss = [], []
        for _ in range(GEMV_COPIES):
            w = torch.randn(N, K, device=dev, generator=g) * 0.02        # W ~ N(0, 0.02) (config 1)
            q, sc = synthetic.to_fp8_rows(w)                              # the engine's quantizer
            qs.append(q.contiguous())
            ss.append(sc.view(-1).contiguous())
            del w
        xs = [torch.randn(K, device=dev, generator=g).to(torch.bfloat16) for _ in range(4)]
        per_shape[(N, K)] = (qs, ss, xs)

    def calls(N, K):
        qs, ss, xs = per_shape[(N, K)]
        for i in range(GEMV_CALLS):
            fp8gemv.gemv(qs[i % GEMV_COPIES], ss[i % GEMV_COPIES], xs[i % 4])

    graphs = {}
    for shape in GEMV_SHAPES:
        calls(*shape)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            calls(*shape)
        graphs[shape] = gr
    us_call, clk = {}, None
    for shape in GEMV_SHAPES:
        ms, c = ctx.timed(lambda i, s=shape: graphs[s].replay(), steps, args.warmup, clocks=True)
        us_call[shape] = ms * 1e3 / GEMV_CALLS
        clk = clk or c
    N0, K0 = GEMV_SHAPES[0]
    b0 = gemv_bytes(N0, K0)

    # parity: one call of each shape (fp32 result before the bf16 rounding) against the oracle
    oracle = oracle_mod(host_threads(ctx))
    errs = []
    for (N, K), (qs, ss, xs) in per_shape.items():
        y = fp8gemv.gemv_f32(qs[0], ss[0], xs[0]).cpu().numpy()
        ref = oracle.gemv(qs[0].view(torch.uint8).cpu().numpy(), ss[0].cpu().numpy(), xs[0].float().cpu().numpy())
        errs.append(rel_err(y, ref))
    parity = ctx.parity(errs, True, len(errs))

    # e2e: the public API per call, x copied in from pinned host memory, y copied back
    qs, ss, xs = per_shape[GEMV_SHAPES[0]]
    h_x = [x.cpu().pin_memory() for x in xs]
    h_y = [torch.empty(N0, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    d_x = [torch.empty_like(xs[0]) for _ in range(2)]
    e2e_pipelined = make_e2e_pipeline(
        lambda i, k: d_x[k].copy_(h_x[i % 4], non_blocking=True),
        lambda i, k: fp8gemv.gemv(qs[i % GEMV_COPIES], ss[i % GEMV_COPIES], d_x[k]),
        lambda i, k, y: h_y[k].copy_(y, non_blocking=True))

    # GEMV_CALLS calls, each with its copy in and copy out (pipelined: call i + 1's x
    # copies in and call i - 1's y copies out during call i), in one CUDA graph, as an
    # engine's decode step captures its projections
    e2e_pipelined(2)
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_pipelined(GEMV_CALLS)
    ms_e2e = ctx.timed(lambda i: e2e_graph.replay(), 16, 3) / GEMV_CALLS
    del e2e_graph
    hbm, _, kind = peaks()
    achieved = b0 / (us_call[GEMV_SHAPES[0]] * 1e-6) / 1e9
    rec = {
        "metric": GEMV_METRIC, "value": ctx.world * achieved, "unit": "GB/s", "steps": steps,
        "us_per_call": {f"{N}x{K}": us_call[(N, K)] for (N, K) in GEMV_SHAPES}, "higher_is_better": True,
        "dtype": "e4m3 weights, bf16 x, fp32 accumulate",
        "config": {"workload": f"fp8-gemv (config 1): {N0}x{K0} per call, bs=1; a step = {GEMV_CALLS} calls in one "
                               f"CUDA graph over {GEMV_COPIES} rotated weight copies",
                   "gbs_per_shape": {f"{N}x{K}": gemv_bytes(N, K) / (us_call[(N, K)] * 1e-6) / 1e9
                                     for (N, K) in GEMV_SHAPES},
                   "bytes_per_call": {f"{N}x{K}": gemv_bytes(N, K) for (N, K) in GEMV_SHAPES},
                   "l2": f"no flush: {GEMV_COPIES} rotated weight copies per shape "
                         f"({GEMV_COPIES * N0 * K0 / 1e6:.0f} MB > 2 x 126 MB L2)"},
        "e2e": {"value": ctx.world * b0 / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": K0 * 2,
                "d2h_bytes_per_step": N0 * 2, "us_per_call": ms_e2e * 1e3,
                "path": "fp8gemv.gemv (public API) with x from pinned host memory and y copied back every call, "
                        f"{GEMV_CALLS} calls per CUDA graph, copies on two copy streams overlapping the neighbouring "
                        "calls"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "kernel": "gemv_stream_kernel",
                     # the capture is of the 2560x4096 shape; scaled to this shape by its algorithmic bytes
                     "traffic": TRAFFIC["gemv_ratio"] * b0, "per_launch_bytes": b0},
        "parity": parity,
        "gpu_launches": steps * GEMV_CALLS,
        "clocks": clk,
    }
    if ctx.world == 1 and not args.no_cpu_baseline:
        q, sc, xf = qs[0].view(torch.uint8).cpu().numpy(), ss[0].cpu().numpy(), xs[0].float().cpu().numpy()
        n = 3
        t0 = time.perf_counter()
        for _ in range(n):
            oracle.gemv(q, sc, xf)
        dt = (time.perf_counter() - t0) / n
        rec["cpu_baseline"] = {"value": b0 / dt / 1e9, "unit": "GB/s", "cores": host_threads(ctx), "kind": "port",
                               "sample": f"{n} calls of the {N0}x{K0} GEMV (C oracle: e4m3 decode, fp64 dot "
                                         f"products), {dt * 1e3:.1f} ms/call"}
    if not parity["pass"]:
        ctx.failed.append("gemv")
    del graphs
    return rec


# ---------------------------------------------------------------- batched decode (config 4)
def batch_decode_record(ctx, steps):
    """A step = one decode step of --batch tokens per GPU through all --n-layers MoE
    layers; router logits ~ N(0,1) (uniform popularity), top-10 of 512 per layer.  1 GPU:
    qmoe.moe_prefill per layer on the 48-layer table, one CUDA graph per step.  N GPUs:
    expert-parallel (512 / N experts of every layer per rank, contiguous: the popularity
    is uniform), NCCL all-gather + reduce-scatter per layer, eager."""
    import numpy as np
    import torch
    import qmoe
    import routing
    from expert_table import ExpertTable
    args, dev, world, rank = ctx.args, ctx.dev, ctx.world, ctx.rank
    L, B = args.n_layers, args.batch
    shard = None
    if world == 1:
        table = ctx.table48()
    else:
        import ep
        shard = ep.ExpertShard(N_EXPERTS, world, rank)
        table = ExpertTable(K=TOPK, dev=dev, n_layers=L, n_experts=shard.per_rank)
        table.fill_synthetic(seed=args.seed, experts=shard.experts)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 23 + 1000 * rank)
    R = 2
    xs = torch.randn(R, L, B, HID, device=dev, generator=g).to(torch.bfloat16)
    ti, tv = routing.route(torch.randn(R * L * B, N_EXPERTS, device=dev, generator=g), TOPK)
    ti, tv = ti.view(R, L, B, TOPK).contiguous(), tv.view(R, L, B, TOPK).contiguous()

    def layer(x, t, v, l):
        if shard is None:
            return qmoe.moe_prefill(x, t, v, table.slots, table.s2[l], l)
        if args.ep_mode == "ag":
            return ep.moe_prefill_ep_ag(x, t, v, table.slots, table.s2[l], l, shard)
        return ep.moe_prefill_ep(x, t, v, table.slots, table.s2[l], l, shard)

    def step(r):
        for l in range(L):
            layer(xs[r, l], ti[r, l], tv[r, l], l)

    graphs = None
    if shard is None:   # expert-parallel steps run eagerly (their NCCL collectives are not captured)
        step(0)
        torch.cuda.synchronize()
        graphs = []
        for r in range(R):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step(r)
            graphs.append(gr)

    def run(i):
        if graphs is not None:
            graphs[i % R].replay()
        else:
            step(i % R)

    ms, clk = ctx.timed(run, steps, args.warmup, clocks=True)
    if shard is None:
        distinct = sum(int(torch.unique(ti[r, l]).numel()) for r in range(R) for l in range(L)) / R
    else:
        mine = shard.maps(dev)[2]
        distinct = 0
        for r in range(R):
            for l in range(L):
                a = torch.cat(ctx_all_gather(ctx, ti[r, l]))
                distinct += int(torch.unique(a[mine[a] >= 0]).numel())
        distinct /= R
    rows = B * (world if (shard is not None and args.ep_mode == "ag") else 1)
    step_bytes = distinct * BLOCK + L * rows * HID * (2 + 4)
    gbs = step_bytes / (ms * 1e-3) / 1e9

    # parity: layer 0 and the last layer of step 0, a sample of this rank's tokens
    errs, ok, n = [], True, 0
    for l in (0, L - 1):
        out = layer(xs[0, l], ti[0, l], tv[0, l], l)
        torch.cuda.synchronize()
        e, o, k = prefill_parity(ctx, out, xs[0, l], ti[0, l], tv[0, l], l, 8, 2000 + 10 * rank + l)
        errs.append(e)
        ok, n = ok and o, n + k
    parity = ctx.parity(errs, ok, n)

    # e2e: per step every layer's x, ti, tv from pinned host memory and its fp32
    # output back, pipelined over two buffer sets (the next step's copy in and
    # the previous step's copy out overlap this step's layers)
    h_x, h_ti, h_tv = xs[0].cpu().pin_memory(), ti[0].cpu().pin_memory(), tv[0].cpu().pin_memory()
    h_out = [torch.empty(L, B, HID, dtype=torch.float32).pin_memory() for _ in range(2)]
    d_in = [(torch.empty_like(xs[0]), torch.empty_like(ti[0]), torch.empty_like(tv[0])) for _ in range(2)]
    d_x = d_in[0][0]

    def e2e_out(i, k, outs):
        for l in range(L):
            h_out[k][l].copy_(outs[l], non_blocking=True)

    e2e_pipelined = make_e2e_pipeline(
        lambda i, k: (d_in[k][0].copy_(h_x, non_blocking=True), d_in[k][1].copy_(h_ti, non_blocking=True),
                      d_in[k][2].copy_(h_tv, non_blocking=True)),
        lambda i, k: [layer(d_in[k][0][l], d_in[k][1][l], d_in[k][2][l], l) for l in range(L)],
        e2e_out)
    E = min(args.e2e_steps, 8)
    ms_e2e = ctx.timed(lambda i: e2e_pipelined(E), 1, 1) / E
    hbm, _, kind = peaks()
    rec = {
        "metric": BD_METRIC, "value": world * B / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
        "steps": steps, "higher_is_better": True,
        "dtype": "f16 tensor-core products of nvfp4 weights (exact) and bf16 activations, fp32 accumulate",
        "config": {"workload": f"batch-decode (config 4): {B} tokens per GPU, {L} layers, top-{TOPK} of "
                               f"{N_EXPERTS} uniform; {distinct / L:.0f} distinct experts per layer per rank",
                   "hbm_gbs_per_gpu": gbs, "bytes_per_step_rank": step_bytes,
                   "l2": "no flush: each step reads ~48 GB of distinct expert blocks (>> 126 MB L2)",
                   "parallelism": "single GPU" if world == 1 else
                   f"expert-parallel x{world} (NCCL {'all-gather + reduce-scatter' if args.ep_mode == 'ag' else 'all-to-all'}, eager)"},
        "e2e": {"value": world * B / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": d_in[0][0].numel() * 2 + d_in[0][1].numel() * 8 + d_in[0][2].numel() * 2,
                "d2h_bytes_per_step": L * B * HID * 4, "ms_per_step": ms_e2e,
                "path": ("qmoe.moe_prefill" if shard is None else "ep.moe_prefill_ep" + ("_ag" if args.ep_mode == "ag" else "")) +
                        " per layer (public API, eager) with pinned host inputs and outputs, pipelined over two "
                        "buffer sets (copies on two copy streams overlap the neighbouring steps' layers)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "peak_kind": kind, "traffic": None,
                     "kernel": "qfn_moe_prefill per layer (7 launches; the time is the whole step's)"},
        "parity": parity,
        "gpu_launches": steps * L * PF_LAUNCHES,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        import synthetic
        oracle = oracle_mod(host_threads(ctx))
        n = min(8, B)
        t_l = ti[0, 0, :n].cpu().numpy()
        used = np.unique(t_l)
        blocks = table.slots[used.tolist()].cpu().numpy()
        t0 = time.perf_counter()
        oracle.moe_prefill(xs[0, 0, :n].float().cpu().numpy(), np.searchsorted(used, t_l).astype(np.int32),
                           tv[0, 0, :n].float().cpu().numpy(), blocks, 0, np.full((len(used), 3), WS2, np.float32))
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": n / (dt * L), "unit": "tokens/s", "cores": host_threads(ctx), "kind": "port",
                               "sample": f"{n} tokens of layer 0 ({len(used)} experts: block dequant + fp32 GEMMs "
                                         f"+ index_add) in {dt:.1f} s, extrapolated x{L} layers"}
    if not parity["pass"]:
        ctx.failed.append("batch-decode")
    del graphs
    return rec


# ---------------------------------------------------------------- the decode MoE block (router + routed + shared expert)
SH_INTER = 640      # shared-expert width: the checkpoint's config.json is absent here; the routed experts' 640 assumed
BLOCK_METRIC = "decode MoE block us/layer (router + 10 routed NVFP4 experts + bf16 shared expert, 48 layers)"


def decode_block_record(ctx, steps):
    """The whole T == 1 MoE block of QwenEngine.moe (qwen_engine.py:801-829) on the
    device: fused router (bf16 [512, 2560], N(0, 0.02)) -> routed experts on the
    48-layer table -> bf16 shared expert + combine; 48 layers in one CUDA graph,
    nothing read back to the host between layers."""
    import numpy as np
    import torch
    import moe_block
    import routing
    args, dev = ctx.args, ctx.dev
    table = ctx.table48()
    L = args.n_layers
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 41)
    routers = [(torch.randn(N_EXPERTS, HID, device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(L)]
    shared = [tuple((torch.randn(*shp, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                    for shp in ((SH_INTER, HID), (SH_INTER, HID), (HID, SH_INTER), (1, HID))) for _ in range(L)]
    x_all = torch.randn(L, 1, HID, device=dev, generator=g).to(torch.bfloat16)
    xs = list(x_all)                        # the layers' inputs: views of one buffer
    blk = moe_block.DecodeMoE(table, topk=TOPK)
    out_all = torch.empty(L, 1, HID, dtype=torch.bfloat16, device=dev)
    outs = list(out_all)

    def step():
        for l in range(L):
            blk(xs[l], l, routers[l], *shared[l], out=outs[l])

    step()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step()
    ms, clk = ctx.timed(lambda i: gr.replay(), steps, args.warmup, clocks=True)
    layer_bytes = LAYER_BYTES + N_EXPERTS * HID * 2 + 3 * SH_INTER * HID * 2 + HID * 2
    # parity: the last layer's block against the oracle on the kernel's routing
    oracle = oracle_mod(host_threads(ctx))
    l = L - 1
    blk(xs[l], l, routers[l], *shared[l], out=outs[l])
    torch.cuda.synchronize()
    r = blk.route_buf
    ti = r["ti"][0].cpu().numpy()
    logits = r["logits"].float().cpu().numpy()
    ti_ref, coef_ref = oracle.route(logits, TOPK)
    route_ok = bool(np.array_equal(ti, ti_ref[0]))
    blocks = table.slots[torch.from_numpy(ti + l * N_EXPERTS).long().to(dev)].cpu().numpy()
    y = oracle.moe_decode(blocks, np.arange(TOPK, dtype=np.int32), table.s2[l][torch.from_numpy(ti).long()].cpu().numpy(),
                          r["tv"][0].float().cpu().numpy(), xs[l].float().cpu().numpy()[0])
    ref = oracle.shared_expert(*(t.float().cpu().numpy() for t in (xs[l],) + shared[l]), y[None])
    got = outs[l].float().cpu().numpy()
    parity = ctx.parity([rel_err(got, ref)], route_ok and int(got.argmax()) == int(ref.argmax()), 1)
    parity["tol"] = 1e-2
    parity["pass"] = parity["max_err_rms"] <= 1e-2 and parity["argmax_equal"]
    parity["checker"] = "oracle router + moe_decode + shared expert (bf16 output: a few bf16 steps)"

    # e2e: x of every layer from pinned host memory and every layer's bf16 output
    # back each step, steps pipelined over two buffer sets (the next step's x
    # and the previous step's outputs copy on two copy streams during the graph)
    h_x = x_all.cpu().pin_memory()
    h_out = [torch.empty(L, 1, HID, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    d_x = [torch.empty_like(x_all) for _ in range(2)]
    d_o = [torch.empty_like(out_all) for _ in range(2)]

    def e2e_compute(i, k):
        x_all.copy_(d_x[k])
        gr.replay()
        return d_o[k].copy_(out_all)

    e2e_pipelined = make_e2e_pipeline(lambda i, k: d_x[k].copy_(h_x, non_blocking=True), e2e_compute,
                                      lambda i, k, o: h_out[k].copy_(o, non_blocking=True))
    E = min(args.e2e_steps, steps)
    ms_e2e = ctx.timed(lambda i: e2e_pipelined(E), 1, 2) / E
    hbm, _, kind = peaks()
    achieved = layer_bytes * L / (ms * 1e-3) / 1e9
    if not parity["pass"]:
        ctx.failed.append("decode-block")
    del gr
    return {
        "metric": BLOCK_METRIC, "value": ms * 1e3 / L, "unit": "us/layer", "higher_is_better": False,
        "ms_per_step": ms, "steps": steps,
        "config": {"workload": f"decode MoE block x {L} layers (bs=1): router bf16 [512, 2560], top-{TOPK} of 512 "
                               f"(routing from the router's logits), shared expert bf16 [{SH_INTER}, 2560] x 3 "
                               f"(width assumed: no config.json here)", "layer_bytes": layer_bytes,
                   "l2": "no flush: each step streams > 1.3 GB of distinct expert bytes (> 126 MB L2)"},
        "e2e": {"value": ms_e2e * 1e3 / L, "unit": "us/layer", "h2d_bytes_per_step": L * HID * 2,
                "d2h_bytes_per_step": L * HID * 2, "ms_per_step": ms_e2e,
                "path": "moe_block.DecodeMoE per layer (router, routed experts, shared expert) in one CUDA graph, "
                        "steps pipelined over two buffer sets (copies on two copy streams); "
                        "x in from and bf16 outputs out to pinned host memory"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": TRAFFIC["decode_block"],
                     "kernel": "moe_route_logits + moe_route_select + moe_decode_slice + shared_gate_up + shared_down"},
        "parity": parity,
        "gpu_launches": steps * L * 5,
        "clocks": clk,
    }


DN_HEADS, DN_KEY_HEADS, DN_DK, DN_DV, DN_LAYERS = 32, 32, 128, 128, 36   # from the config-1 GEMV shapes


def deltanet_record(ctx, steps):
    """One decoded token through the DeltaNet state updates of 36 linear-attention
    layers (qwen_engine.py:718-719): 32 value heads, dk = dv = 128 (the shapes the
    config-1 GEMVs imply: qkv 12288 = 2 x 32 x 128 + 32 x 128, out K = 4096),
    state 2 MB per layer read and written once; one CUDA graph per step."""
    import numpy as np
    import torch
    import deltanet
    import synthetic
    args, dev = ctx.args, ctx.dev
    H, Hk, dk, dv, L = DN_HEADS, DN_KEY_HEADS, DN_DK, DN_DV, DN_LAYERS
    q, k, v, g, beta, S0 = synthetic.deltanet_inputs(L, H, Hk, dk, dv, seed=args.seed + 51)
    q, k, v, g, beta = (t.to(dev) for t in (q, k, v, g, beta))
    S = [S0[None].clone().to(dev) for _ in range(L)]
    outs = []

    def step():
        outs.clear()
        for l in range(L):
            o, _ = deltanet.recurrent_gated_delta_rule(q[l][None, None], k[l][None, None], v[l][None, None],
                                                       g[l][None, None], beta[l][None, None], S[l])
            outs.append(o)

    step()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step()
    ms, clk = ctx.timed(lambda i: gr.replay(), steps, args.warmup, clocks=True)
    state_bytes = 2 * H * dk * dv * 4
    layer_bytes = state_bytes + (2 * Hk * dk + H * dv) * 2 + H * 6 + H * dv * 2
    # parity: one step of layer 0 from a known state against the fp64 oracle
    oracle = oracle_mod(host_threads(ctx))
    S_ref = S0.double().numpy().copy()
    S_k = S0[None].clone().to(dev)
    o, _ = deltanet.recurrent_gated_delta_rule(q[0][None, None], k[0][None, None], v[0][None, None],
                                               g[0][None, None], beta[0][None, None], S_k)
    ref = oracle.deltanet_step(q[0].float().cpu().numpy(), k[0].float().cpu().numpy(), v[0].float().cpu().numpy(),
                               g[0].cpu().numpy(), beta[0].float().cpu().numpy(), S_ref)
    s_err = float(np.abs(S_k[0].cpu().numpy() - S_ref).max() / np.sqrt(np.mean(S_ref ** 2)))
    got = np.ascontiguousarray(o[0, 0].float().cpu().numpy())
    steps_ = np.abs((got.view(np.int32) >> 16).astype(np.int64) - (ref.view(np.int32) >> 16).astype(np.int64))
    parity = ctx.parity([s_err], bool(steps_.max() <= 1), 1)
    parity["tol"] = 1e-5
    parity["pass"] = parity["max_err_rms"] <= 1e-5 and parity["argmax_equal"]
    parity["checker"] = ("oracle.deltanet_step (fp64): fp32 state within 1e-5 of RMS (max_err_rms); every bf16 "
                         "output within one bf16 step (argmax_equal)")
    hbm, _, kind = peaks()
    achieved = layer_bytes * L / (ms * 1e-3) / 1e9
    if not parity["pass"]:
        ctx.failed.append("deltanet")
    del gr

    # e2e: per step every layer's q, k, v, g, beta from pinned host memory and
    # its output back, steps pipelined over two buffer sets inside one CUDA graph
    h_in = [t.cpu().pin_memory() for t in (q, k, v, g, beta)]
    d_in = [[torch.empty_like(t) for t in (q, k, v, g, beta)] for _ in range(2)]

    def e2e_compute(i, kk):
        dq, dk_, dv_, dg, db = d_in[kk]
        return torch.stack([deltanet.recurrent_gated_delta_rule(dq[l][None, None], dk_[l][None, None],
                                                                dv_[l][None, None], dg[l][None, None],
                                                                db[l][None, None], S[l])[0] for l in range(L)])

    probe = e2e_compute(0, 0)
    h_out = [torch.empty(probe.shape, dtype=probe.dtype).pin_memory() for _ in range(2)]
    e2e_pipelined = make_e2e_pipeline(
        lambda i, kk: [d.copy_(h, non_blocking=True) for d, h in zip(d_in[kk], h_in)],
        e2e_compute,
        lambda i, kk, o: h_out[kk].copy_(o, non_blocking=True))
    E = 16
    e2e_pipelined(2)
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_pipelined(E)
    ms_e2e = ctx.timed(lambda i: e2e_graph.replay(), 4, 2) / E
    del e2e_graph
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = probe.numel() * probe.element_size()
    return {
        "metric": "DeltaNet one-token state update us/layer (32 heads, 128 x 128 fp32 state)", "value": ms * 1e3 / L,
        "unit": "us/layer", "higher_is_better": False, "ms_per_step": ms, "steps": steps,
        "config": {"workload": f"{L} linear-attention layers x one token; heads {H} (key heads {Hk}), dk {dk}, "
                               f"dv {dv}; one CUDA graph per step", "layer_bytes": layer_bytes,
                   "l2": f"no flush: {L} states of {state_bytes / 2 / 1e6:.1f} MB = {L * state_bytes / 2e6:.0f} MB "
                         "per step (> 126 MB L2 with reads and writes)"},
        "e2e": {"value": ms_e2e * 1e3 / L, "unit": "us/layer", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": ms_e2e,
                "path": "deltanet.recurrent_gated_delta_rule per layer (public API) with pinned host q, k, v, g, beta "
                        "in and the bf16 outputs out every step, steps pipelined over two buffer sets (copies on two "
                        f"copy streams), {E} steps per CUDA graph"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind, "traffic": TRAFFIC["deltanet"], "kernel": "deltanet_step_kernel"},
        "parity": parity,
        "gpu_launches": steps * L,
        "clocks": clk,
    }


# ---------------------------------------------------------------- FP8 linear layer for T > 1
def fp8_linear_record(ctx, steps):
    """The engine's FP8 linear layer for T > 1 tokens (Lin.__call__, qwen_engine.py:79-83):
    --tokens tokens through the config-1 shapes; a step = one call per shape through
    fp8gemv.linear (one qfn_linear_e4m3 GEMM each).  Also timed on the same GPU: the
    reference's own torch expression F.linear(x, (q.to(bf16) * s).to(bf16)), and the
    library path (the bit-identical bf16 weights of qfn_e4m3_rows_to_bf16, then cuBLAS)."""
    import torch
    import torch.nn.functional as F
    import fp8gemv
    import synthetic
    args, dev = ctx.args, ctx.dev
    T = args.tokens
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 31)
    data = {}
    for (N, K) in GEMV_SHAPES:
        qs, ss = [], []
        for _ in range(LIN_COPIES):
            w = torch.randn(N, K, device=dev, generator=g) * 0.02
            q, sc = synthetic.to_fp8_rows(w)
            qs.append(q.contiguous())
            ss.append(sc.view(-1, 1).contiguous())
            del w
        data[(N, K)] = (qs, ss, torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16))

    def ours(i):
        return [fp8gemv.linear(x, qs[i % LIN_COPIES], ss[i % LIN_COPIES]) for qs, ss, x in data.values()]

    def library(i):
        for qs, ss, x in data.values():
            F.linear(x, fp8gemv.dequant_bf16(qs[i % LIN_COPIES], ss[i % LIN_COPIES]))

    def reference(i):
        for qs, ss, x in data.values():
            q, sc = qs[i % LIN_COPIES], ss[i % LIN_COPIES]
            F.linear(x, (q.to(torch.bfloat16) * sc).to(torch.bfloat16))

    ms, clk = ctx.timed(ours, steps, args.warmup, clocks=True)
    ms_lib = ctx.timed(library, steps, args.warmup)
    ms_ref = ctx.timed(reference, steps, args.warmup)
    # parity: against the exact products of the reference's bf16 weights (q.to(bf16) * s).to(bf16)
    # (fp64 sums on the GPU, 64 sampled tokens per shape): every output within one bf16 step of the
    # exact value (less 1e-5 x RMS for the fp32 accumulation), and nearly all equal to its bf16
    # rounding (the fp32 summation order aside)
    steps_off, differ, rows = 0.0, 0.0, 0
    for qs, ss, x in data.values():
        sel = torch.randperm(T, generator=torch.Generator().manual_seed(args.seed + 5))[:64].to(dev)
        a = fp8gemv.linear(x, qs[0], ss[0])[sel].double()
        w = (qs[0].to(torch.bfloat16) * ss[0]).to(torch.bfloat16).double()
        exact = x[sel].double() @ w.T
        step = torch.exp2(torch.floor(torch.log2(exact.abs().clamp_min(1e-30))) - 7)
        off = ((a - exact).abs() - 1e-5 * exact.pow(2).mean().sqrt()).clamp_min(0) / step
        steps_off = max(steps_off, float(off.max()))
        differ = max(differ, float((a != exact.float().to(torch.bfloat16).double()).double().mean()))
        rows += int(sel.numel())
    steps_off = ctx.max_over_ranks(steps_off)
    differ = ctx.max_over_ranks(differ)
    parity = {"max_bf16_steps": steps_off, "frac_not_rounded_exact": differ, "tol": "<= 1 bf16 step, < 1 % not RN(exact)",
              "checked_rows": rows,
              "checker": "fp64 sums of the reference's bf16 weights (q.to(bf16) * s).to(bf16) on sampled tokens",
              "pass": steps_off <= 1.0 and differ < 0.01}
    if not parity["pass"]:
        ctx.failed.append("fp8-linear")
    hx = {k: v[2].cpu().pin_memory() for k, v in data.items()}
    hy = {(N, K): torch.empty(T, N, dtype=torch.bfloat16).pin_memory() for (N, K) in GEMV_SHAPES}
    dx = {k: torch.empty_like(v[2]) for k, v in data.items()}

    def e2e(i):
        for k, (qs, ss, _) in data.items():
            dx[k].copy_(hx[k], non_blocking=True)
            hy[k].copy_(fp8gemv.linear(dx[k], qs[i % LIN_COPIES], ss[i % LIN_COPIES]), non_blocking=True)

    ms_e2e = ctx.timed(e2e, steps, args.warmup)
    flop = sum(2 * T * N * K for (N, K) in GEMV_SHAPES)
    _, tensor_peak, kind = peaks()
    tflops = flop / (ms * 1e-3) / 1e12
    return {
        "metric": f"fp8 linear layer, T={T} tokens, TFLOP/s (config-1 weight shapes)",
        "value": ctx.world * tflops, "unit": "TFLOP/s", "n_gpus": ctx.world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 weights -> bf16 on chip, bf16 tensor-core products, fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"fp8-linear: {T} tokens x (12288x2560 + 2560x4096), bf16 out",
                   "us_reference_expression_same_gpu": ms_ref * 1e3,
                   "us_library_path_same_gpu": ms_lib * 1e3,
                   "l2": f"no flush: {LIN_COPIES} rotated weight copies per shape (> 126 MB L2)",
                   "parallelism": "single GPU" if ctx.world == 1 else f"{ctx.world} replicas"},
        "e2e": {"value": ctx.world * flop / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": sum(T * K * 2 for (N, K) in GEMV_SHAPES),
                "d2h_bytes_per_step": sum(T * N * 2 for (N, K) in GEMV_SHAPES), "ms_per_step": ms_e2e,
                "path": "fp8gemv.linear (public API) with pinned host x in and y out"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": tensor_peak, "unit": "TFLOP/s",
                     "frac": tflops / tensor_peak, "peak_kind": kind, "traffic": None,
                     "kernel": "ln_gemm_kernel, both shapes (two launches; the time is the pair's)"},
        "parity": parity,
        "gpu_launches": steps * len(GEMV_SHAPES),
        "clocks": clk,
    }


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank):
    """The reference's CPU path (C restatement in oracle/, all host cores) on a bounded sample
    per step of the same workload; rank 0 alone runs it."""
    if rank != 0:
        return
    import numpy as np
    import torch
    import synthetic
    oracle = oracle_mod(os.cpu_count() or 1)
    cores = oracle.threads(0)
    line = {"impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic"}

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            fn(args.warmup + i)
        return time.perf_counter() - t0

    if args.workload in ("prefill", "batch-decode"):
        T = args.tokens if args.workload == "prefill" else args.batch
        if args.workload == "prefill":
            ti, tv = oracle.route(synthetic.zipf_logits(T, seed=args.seed + 7), TOPK)
        else:
            ti, tv = oracle.route(synthetic.normal_logits(T, seed=args.seed + 23), TOPK)
        x = synthetic.make_x(T * HID, seed=args.seed + 8, dtype=torch.float32).view(T, HID).numpy()
        cache = {}

        def block(e):
            if e not in cache:
                cache[e] = synthetic.make_blocks(1, seed=synthetic.block_seed(args.seed, 0, e))[0]
            return cache[e]

        n_slices = 64 if args.workload == "prefill" else 8
        sl = OracleSlices(oracle, x, ti, tv, block, n=n_slices)
        for i in range(min(n_slices, args.steps + args.warmup)):   # block generation stays out of the timing
            sl.blocks(i)
        dt = timed(sl.run)
        per_token_layers = 1 if args.workload == "prefill" else args.n_layers
        v = T * args.steps / (n_slices * dt) / per_token_layers
        line.update({"metric": PF_METRIC if args.workload == "prefill" else BD_METRIC, "value": v,
                     "unit": "tokens/s", "ms_per_step": dt / args.steps * 1e3,
                     "config": {"workload": f"{args.workload} (config {'3' if args.workload == 'prefill' else '4'}), "
                                            f"CPU sample: one of {n_slices} balanced expert slices of a {T}-token "
                                            "layer per step", "parallelism": "cpu"}})
        sample = (f"a step = 1/{n_slices} of one layer of {T} tokens (the pairs of {N_EXPERTS // n_slices} experts: "
                  f"block dequant + fp32 GEMMs + index_add), C oracle, {cores} OpenMP threads; tokens/s = "
                  f"{T} / ({n_slices} x time per step)" +
                  ("" if args.workload == "prefill" else f" / {args.n_layers} layers"))
    elif args.workload == "gemv":
        N, K = GEMV_SHAPES[0]
        q, sc = oracle.to_fp8_rows(synthetic.gemv_weights(N, K, seed=args.seed).float().numpy())
        x = synthetic.make_x(K, seed=args.seed).float().numpy()
        dt = timed(lambda i: oracle.gemv(q, sc, x))
        v = args.steps * gemv_bytes(N, K) / dt / 1e9
        line.update({"metric": GEMV_METRIC, "value": v, "unit": "GB/s", "ms_per_step": dt / args.steps * 1e3,
                     "config": {"workload": f"fp8-gemv (config 1): {N}x{K} per call, bs=1", "parallelism": "cpu"}})
        sample = f"one {N}x{K} GEMV per step, C oracle, {cores} OpenMP threads"
    else:  # decode
        blocks = synthetic.make_blocks(TOPK, seed=args.seed)
        sidx = np.arange(TOPK, dtype=np.int32)
        s2 = synthetic.make_s2(TOPK)
        _, coef = oracle.route(synthetic.zipf_logits(1, seed=args.seed))
        x = synthetic.make_x(HID, seed=args.seed).float().numpy()
        dt = timed(lambda i: oracle.moe_decode(blocks, sidx, s2, coef[0], x))
        v = args.steps * LAYER_BYTES / dt / 1e9
        line.update({"metric": DECODE_METRIC, "value": v, "unit": "GB/s", "ms_per_step": dt / args.steps * 1e3,
                     "config": {"workload": "decode-moe-48L (config 2), CPU sample: 1 layer per step",
                                "parallelism": "cpu"}})
        sample = f"one decode layer (10 synthetic expert blocks) per step, C oracle, {cores} OpenMP threads"
    line["cpu_baseline"] = {"value": line["value"], "unit": line["unit"], "cores": cores, "kind": "port",
                            "sample": sample}
    line["e2e"] = {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    print(json.dumps(line))


# ---------------------------------------------------------------- main
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    ctx = Ctx(args)
    sub_steps = min(args.sub_steps, args.steps) if args.steps > 0 else args.sub_steps
    if args.workload == "prefill":
        line = prefill_record(ctx)
        if not args.no_sub:
            subs = {}
            if ctx.world == 1:
                subs["decode_config2"] = decode_record(ctx, max(sub_steps, 4))
                subs["gemv_config1"] = gemv_record(ctx, max(sub_steps, 4))
                subs["decode_moe_block"] = decode_block_record(ctx, max(sub_steps // 2, 4))
                subs["deltanet_step"] = deltanet_record(ctx, max(sub_steps, 4))
            if ctx.world == 1:
                subs["fp8_linear"] = fp8_linear_record(ctx, max(sub_steps // 2, 4))
            subs["batch_decode_config4"] = batch_decode_record(ctx, max(sub_steps // 4, 4))
            line["sub"] = subs
    else:
        fn = {"decode": decode_record, "gemv": gemv_record, "batch-decode": batch_decode_record,
              "fp8-linear": fp8_linear_record, "decode-block": decode_block_record,
              "deltanet": deltanet_record}[args.workload]
        line = fn(ctx, args.steps)
        line.setdefault("n_gpus", ctx.world)
        line.setdefault("warmup", max(args.warmup, 3))
        line.setdefault("scaling", "weak")
        line.setdefault("vs_baseline", None)
        line.setdefault("data", "synthetic")
    if ctx.dist is not None:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))
    if ctx.failed:
        if rank == 0:
            print(f"parity FAILED: {ctx.failed}", file=sys.stderr)
        sys.exit(3)


if __name__ == "__main__":
    main()
