"""Benchmark of the bs=1 NVFP4 decode MoE stack.

Workload: all 48 x 512 NVFP4 expert blocks (63.3 GiB, config-0 shapes and
scale distributions) resident in HBM; per decode step (one token) 48 layers,
each routed top-10 of 512 by fp32 logits with Zipf(1.1) popularity (one
popularity permutation per layer, fresh Gumbel noise per step); x ~ N(0,1)
bf16 per layer.  A step = 48 calls of the fused decode expert layer.
Every step streams 48 x 27.66 MB of distinct expert bytes (1.33 GB >> the
126 MB L2), so no L2 flush is needed between steps.

  value  : aggregate algorithmic HBM GB/s (bytes of the 48 layers / device
           time), graph-replayed steps with inputs resident in HBM, max over ranks.
  e2e    : same metric through the public API (qmoe.moe_decode per layer,
           eager), each step copying its inputs host->device from pinned memory
           and its 48 outputs device->host.
  N > 1  : replicas (bs=1 decode does not shard): every rank holds its own
           table and runs the same workload; scaling "weak".

`--impl reference` times the reference's CPU path (the C restatement in
oracle/) on this host's cores on a bounded sample of the same workload.
"""
import argparse
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
TOPK, N_EXPERTS = 10, 512
# algorithmic bytes of one decode layer: 10 expert blocks + s2 + coef + x (bf16) + out (fp32)
LAYER_BYTES = TOPK * BLOCK + TOPK * 12 + TOPK * 4 + HID * 2 + HID * 4
METRIC = "bs1 decode MoE-layer HBM GB/s (48-layer stack, experts resident in HBM)"
# DRAM bytes (read + written) per launch measured with ncu (profiles/*.md)
TRAFFIC_DECODE_SLICE = 27.74e6          # moe_decode_slice, one layer (K = 10)
TRAFFIC_PREFILL_GEMMS = 1.767e9         # pf_gemm<0> + pf_gemm<1>, one config-3 layer
TRAFFIC_GEMV_RATIO = 10.55e6 / 10.509312e6   # gemv_stream_kernel DRAM bytes / algorithmic bytes
UNIT = "GB/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", default="qfn", choices=["qfn", "reference"])
    p.add_argument("--n-layers", type=int, default=48, help="table layers (48 = full config 2)")
    p.add_argument("--routes", type=int, default=256, help="distinct routed steps (cycled)")
    p.add_argument("--e2e-steps", type=int, default=32)
    p.add_argument("--cpu-layers", type=int, default=4, help="layers timed for the CPU baseline")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--workload", default="decode", choices=["decode", "prefill", "gemv", "batch-decode", "fp8-linear"],
                   help="decode: config 2 (default, the headline line); prefill: config 3; gemv: config 1; "
                        "batch-decode: config 4; fp8-linear: the FP8 linear layer for T > 1 tokens")
    p.add_argument("--batch", type=int, default=64, help="batch-decode: tokens per GPU per step (config 4: 64)")
    p.add_argument("--ep-mode", default="auto", choices=["auto", "a2a", "ag"],
                   help="expert-parallel exchange under torchrun: a2a = all-to-all of routed rows (host sync "
                        "for split sizes), ag = all-gather + reduce-scatter (no host sync); auto = ag")
    p.add_argument("--tokens", type=int, default=2048, help="prefill: tokens per step (config 3: 2048)")
    p.add_argument("--cpu-tokens", type=int, default=24, help="prefill: tokens timed for the CPU baseline")
    p.add_argument("--variant", type=int, default=0,
                   help="decode kernel path: 0 auto (slice path for K <= 10), 3 stream, 4 slice, 2 CUDA-core")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


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


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle
    import synthetic
    cores = oracle.threads(os.cpu_count())
    if args.workload == "gemv":
        N, K = GEMV_SHAPES[0]
        q, sc = oracle.to_fp8_rows(synthetic.gemv_weights(N, K, seed=args.seed).float().numpy())
        x = synthetic.make_x(K, seed=args.seed).float().numpy()
        for _ in range(args.warmup):
            oracle.gemv(q, sc, x)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            oracle.gemv(q, sc, x)
        dt = time.perf_counter() - t0
        v = args.steps * gemv_bytes(N, K) / dt / 1e9
        sample = f"one {N}x{K} GEMV per step, C oracle, {cores} OpenMP threads"
        print(json.dumps({
            "impl": "reference", "metric": GEMV_METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"fp8-gemv (config 1): {N}x{K} per call, bs=1", "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    blocks = synthetic.make_blocks(TOPK, seed=args.seed)
    sidx = np.arange(TOPK, dtype=np.int32)
    s2 = synthetic.make_s2(TOPK)
    ti, coef = oracle.route(synthetic.zipf_logits(1, seed=args.seed))
    x = synthetic.make_x(HID, seed=args.seed).float().numpy()
    for _ in range(args.warmup):
        oracle.moe_decode(blocks, sidx, s2, coef[0], x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.moe_decode(blocks, sidx, s2, coef[0], x)
    dt = time.perf_counter() - t0
    v = args.steps * LAYER_BYTES / dt / 1e9
    sample = f"one decode layer (10 synthetic expert blocks) per step, C oracle, {cores} OpenMP threads"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "decode-moe-48L (config 2), CPU sample: 1 layer per step",
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ---------------------------------------------------------------- qfn arm
def build_workload(args, dev):
    import torch
    import routing
    from expert_table import ExpertTable
    L = args.n_layers
    table = ExpertTable(K=TOPK, dev=dev, n_layers=L, n_experts=N_EXPERTS)
    table.fill_synthetic(seed=args.seed)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 1)
    R = args.routes
    # Zipf(1.1) popularity, one permutation per layer; Gumbel-top-10 per step
    logp = -1.1 * torch.log(torch.arange(1, N_EXPERTS + 1, device=dev, dtype=torch.float64))
    logp = (logp - torch.logsumexp(logp, 0)).float()
    perm = torch.stack([torch.randperm(N_EXPERTS, device=dev, generator=g) for _ in range(L)])
    u = torch.rand(R, L, N_EXPERTS, device=dev, generator=g).clamp_(1e-12, 1 - 1e-7)
    logits = logp[perm][None] - torch.log(-torch.log(u))
    ti, tv = routing.route(logits.view(R * L, N_EXPERTS), TOPK)
    ti = ti.view(R, L, TOPK)
    layer = torch.arange(L, device=dev).view(1, L, 1)
    sidx = (ti + layer * N_EXPERTS).to(torch.int32).contiguous()
    s2 = table.s2[layer.expand_as(ti), ti].contiguous()              # [R, L, K, 3]
    coef = tv.view(R, L, TOPK).float().contiguous()
    x = torch.randn(R, L, HID, device=dev, generator=g).to(torch.bfloat16)
    return table, sidx, s2, coef, x


# ---------------------------------------------------------------- prefill (config 3)
PF_TOPK = 10
PF_FLOP_PER_PAIR = 2 * 3 * INTER * HID          # gate, up and down: 9,830,400 FLOP per (token, expert)
PF_METRIC = "prefill tokens/s (one NVFP4 MoE layer: top-10 of 512 experts, Zipf(1.1) popularity)"


def prefill_inputs(args, dev, R):
    """R routed steps of config 3: x bf16 [T, 2560] ~ N(0,1); fp32 logits = log p[perm] + Gumbel with
    p_r ~ r^-1.1 (one popularity permutation), top-10 + renormalised bf16 weights (the engine's router)."""
    import torch
    import routing
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 7)
    T = args.tokens
    logp = -1.1 * torch.log(torch.arange(1, N_EXPERTS + 1, device=dev, dtype=torch.float64))
    logp = (logp - torch.logsumexp(logp, 0)).float()
    perm = torch.randperm(N_EXPERTS, device=dev, generator=g)
    xs, tis, tvs = [], [], []
    for _ in range(R):
        u = torch.rand(T, N_EXPERTS, device=dev, generator=g).clamp_(1e-12, 1 - 1e-7)
        ti, tv = routing.route(logp[perm][None] - torch.log(-torch.log(u)), PF_TOPK)
        xs.append(torch.randn(T, HID, device=dev, generator=g).to(torch.bfloat16))
        tis.append(ti)
        tvs.append(tv)
    return xs, tis, tvs


def run_prefill(args, rank, world):
    import torch
    import qmoe
    from expert_table import ExpertTable
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = shard = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        import ep
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        shard = ep.ExpertShard(N_EXPERTS, world, rank)
    # expert-parallel: this rank holds 512 / world experts of the layer (its shard)
    e_local = N_EXPERTS // world
    table = ExpertTable(K=TOPK, dev=dev, n_layers=1, n_experts=e_local)
    table.fill_synthetic(seed=args.seed + rank)
    s2 = table.s2[0].contiguous()
    R = 4
    args.seed += 1000 * rank              # every rank routes its own tokens (same popularity permutation)
    xs, tis, tvs = prefill_inputs(args, dev, R)
    T = args.tokens
    pairs = T * PF_TOPK
    distinct = [int(torch.unique(t).numel()) for t in tis]
    layer_bytes = [d * BLOCK + T * HID * 2 + T * HID * 4 for d in distinct]

    ep_fn = None
    if shard is not None:
        ep_fn = ep.moe_prefill_ep if args.ep_mode == "a2a" else ep.moe_prefill_ep_ag

    def step(i):
        if shard is None:
            return qmoe.moe_prefill(xs[i % R], tis[i % R], tvs[i % R], table.slots, s2, 0)
        return ep_fn(xs[i % R], tis[i % R], tvs[i % R], table.slots, s2, 0, shard)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(max(args.warmup, 3)):
        step(i)
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        e0.record(st)
        for i in range(args.steps):
            step(i)
        e1.record(st)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t_ = torch.tensor([ms], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms = float(t_.item())
    tok_s = world * T / (ms * 1e-3)
    tflops = world * pairs * PF_FLOP_PER_PAIR / (ms * 1e-3) / 1e12
    avg_bytes = sum(layer_bytes[i % R] for i in range(args.steps)) / args.steps
    gbs = avg_bytes / (ms * 1e-3) / 1e9       # one rank's expert bytes (for world > 1: its shard's share)

    # e2e: host buffers in (x, ti, tv) and the fp32 result out, every step
    h_x = [x.cpu().pin_memory() for x in xs]
    h_ti = [t.cpu().pin_memory() for t in tis]
    h_tv = [t.cpu().pin_memory() for t in tvs]
    h_out = torch.empty(T, HID, dtype=torch.float32).pin_memory()
    d_x, d_ti, d_tv = torch.empty_like(xs[0]), torch.empty_like(tis[0]), torch.empty_like(tvs[0])
    h2d = d_x.numel() * 2 + d_ti.numel() * 8 + d_tv.numel() * 2
    d2h = T * HID * 4

    def e2e_step(i):
        d_x.copy_(h_x[i % R], non_blocking=True)
        d_ti.copy_(h_ti[i % R], non_blocking=True)
        d_tv.copy_(h_tv[i % R], non_blocking=True)
        if shard is None:
            y = qmoe.moe_prefill(d_x, d_ti, d_tv, table.slots, s2, 0)
        else:
            y = ep_fn(d_x, d_ti, d_tv, table.slots, s2, 0, shard)
        h_out.copy_(y, non_blocking=True)

    E = min(args.e2e_steps, args.steps)
    for i in range(2):
        e2e_step(i)
    barrier()
    e0.record(st)
    for i in range(E):
        e2e_step(i)
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / E
    if dist is not None:
        t_ = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms_e2e = float(t_.item())

    tc_peak, tc_kind = tensor_peak()
    line = {
        "metric": PF_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 tensor-core products of nvfp4 weights (exact) and bf16 activations, "
                                      "fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"prefill-moe-1L (config 3): {T} tokens per GPU, top-{PF_TOPK} of {N_EXPERTS}, "
                               f"Zipf(1.1), {pairs} pairs per GPU, {sum(distinct) / R:.0f} distinct experts per step"
                               f" routed from rank 0's tokens",
                   "tflops": tflops, "hbm_gbs": gbs, "bytes_per_step": avg_bytes,
                   "flop_per_step": pairs * PF_FLOP_PER_PAIR,
                   "l2": "no flush: each step reads >= 1.4 GB of distinct expert blocks (> 126 MB L2)",
                   "parallelism": (f"expert-parallel x{world} (NCCL "
                                   + ("all-to-all dispatch/combine" if args.ep_mode == "a2a"
                                      else "all-gather + reduce-scatter") + ")") if world > 1
                   else "single GPU"},
        "e2e": {"value": world * T / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E, "ms_per_step": ms_e2e,
                "path": "qmoe.moe_prefill (public API) with pinned host inputs and output"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": tflops / tc_peak, "peak_kind": tc_kind,
                     "hbm_frac": gbs / peaks()[0],
                     # the two GEMMs' DRAM bytes per layer, profiles/pf_gemm_prefill-layer.md
                     "traffic": TRAFFIC_PREFILL_GEMMS if world == 1 and args.tokens == 2048 else None,
                     "kernel": "pf_gemm<gate/up> + pf_gemm<down> (+ routing, gather, h packing)"},
        "gpu_launches": args.steps * 6,
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = prefill_cpu_baseline(args, table, s2, xs[0], tis[0], tvs[0])
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def tensor_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def prefill_cpu_baseline(args, table, s2, x, ti, tv):
    """The C oracle's restatement of the expert loop (qwen_engine.py:838-852) on this host's cores for
    the first `cpu_tokens` tokens of step 0 (every expert those tokens route to)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle
    cores = oracle.threads(os.cpu_count())
    n = min(args.cpu_tokens, x.shape[0])
    ti_n = ti[:n].cpu().numpy().astype(np.int32)
    used = sorted(set(ti_n.ravel().tolist()))
    remap = {e: i for i, e in enumerate(used)}
    blocks = table.slots[used].cpu().numpy()
    ti_local = np.vectorize(remap.get)(ti_n).astype(np.int32)
    s2_local = s2[used].cpu().numpy()
    xf = x[:n].float().cpu().numpy()
    tvf = tv[:n].float().cpu().numpy()
    t0 = time.perf_counter()
    oracle.moe_prefill(xf, ti_local, tvf, blocks, 0, s2_local)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n} tokens of step 0 ({len(used)} experts: block dequant + fp32 GEMMs + index_add), "
                      f"{dt:.1f} s"}


# ---------------------------------------------------------------- FP8 GEMV (config 1)
GEMV_SHAPES = ((12288, 2560), (2560, 4096))   # the DeltaNet projections of config 1 (N x K)
GEMV_COPIES = 8                                # weight copies rotated per shape (8 x 31.5 MB > 2 x L2)
GEMV_CALLS = 64                                # calls per graph replay (one step)
GEMV_METRIC = "FP8 E4M3 row-scaled GEMV HBM GB/s (12288x2560, bs=1, per call)"


def gemv_bytes(N, K):
    return N * K + 4 * N + 2 * K + 2 * N       # weights + row scales + x (bf16) + y (bf16)


def run_gemv(args, rank, world):
    import torch
    import fp8gemv
    import synthetic
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    us_call = {}
    clk_summary = None
    for shape in GEMV_SHAPES:
        for _ in range(max(args.warmup, 3)):
            graphs[shape].replay()
        barrier()
        with ClockSampler(local) as clk:
            e0.record(st)
            for _ in range(args.steps):
                graphs[shape].replay()
            e1.record(st)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist is not None:
            t_ = torch.tensor([ms], device=dev)
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            ms = float(t_.item())
        us_call[shape] = ms * 1e3 / (args.steps * GEMV_CALLS)
        if shape == GEMV_SHAPES[0]:
            clk_summary = clk.summary()
            ms_main = ms
    N0, K0 = GEMV_SHAPES[0]
    b0 = gemv_bytes(N0, K0)
    value = world * b0 / (us_call[GEMV_SHAPES[0]] * 1e-6) / 1e9

    # e2e: the public API per call, x copied in from pinned host memory, y copied back
    qs, ss, xs = per_shape[GEMV_SHAPES[0]]
    h_x = [x.cpu().pin_memory() for x in xs]
    h_y = torch.empty(N0, dtype=torch.bfloat16).pin_memory()
    d_x = torch.empty_like(xs[0])
    E = 256

    def e2e_call(i):
        d_x.copy_(h_x[i % 4], non_blocking=True)
        y = fp8gemv.gemv(qs[i % GEMV_COPIES], ss[i % GEMV_COPIES], d_x)
        h_y.copy_(y, non_blocking=True)

    for i in range(8):
        e2e_call(i)
    barrier()
    e0.record(st)
    for i in range(E):
        e2e_call(i)
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    if dist is not None:
        t_ = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms_e2e = float(t_.item())
    e2e_value = world * E * b0 / (ms_e2e * 1e-3) / 1e9

    peak, peak_kind = peaks()
    achieved = b0 / (us_call[GEMV_SHAPES[0]] * 1e-6) / 1e9
    line = {
        "metric": GEMV_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_main / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 weights, bf16 x, fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"fp8-gemv (config 1): {N0}x{K0} per call, bs=1; a step = {GEMV_CALLS} calls in one "
                               f"CUDA graph over {GEMV_COPIES} rotated weight copies",
                   "us_per_call": {f"{N}x{K}": us_call[(N, K)] for (N, K) in GEMV_SHAPES},
                   "gbs_per_shape": {f"{N}x{K}": gemv_bytes(N, K) / (us_call[(N, K)] * 1e-6) / 1e9
                                     for (N, K) in GEMV_SHAPES},
                   "bytes_per_call": {f"{N}x{K}": gemv_bytes(N, K) for (N, K) in GEMV_SHAPES},
                   "l2": f"no flush: {GEMV_COPIES} rotated weight copies per shape "
                         f"({GEMV_COPIES * N0 * K0 / 1e6:.0f} MB > 2 x 126 MB L2)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": K0 * 2, "d2h_bytes_per_step": N0 * 2,
                "steps": E, "us_per_call": ms_e2e * 1e3 / E,
                "path": "fp8gemv.gemv (public API, eager) with x from pinned host memory and y copied back"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "kernel": "gemv_stream_kernel",
                     # profiles/gemv_stream_fp8-gemv.md captured the 2560x4096 shape (10.55 MB per
                     # launch for 10.51 MB algorithmic); scaled to this shape by its bytes
                     "traffic": TRAFFIC_GEMV_RATIO * b0,
                     "per_launch_bytes": b0},
        "gpu_launches": args.steps * GEMV_CALLS,
        "clocks": clk_summary,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle
        cores = oracle.threads(os.cpu_count())
        q = qs[0].view(torch.uint8).cpu().numpy()
        sc = ss[0].cpu().numpy()
        xf = xs[0].float().cpu().numpy()
        oracle.gemv(q, sc, xf)
        n = 3
        t0 = time.perf_counter()
        for _ in range(n):
            oracle.gemv(q, sc, xf)
        dt = (time.perf_counter() - t0) / n
        line["cpu_baseline"] = {"value": b0 / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                "sample": f"{n} calls of the {N0}x{K0} GEMV (C oracle: e4m3 decode, fp64 dot "
                                          f"products), {dt * 1e3:.1f} ms/call"}
    if dist is not None:
        del graphs
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


# ---------------------------------------------------------------- batched decode (config 4)
BD_METRIC = "batched-decode tokens/s (batch 64 per GPU, 48-layer NVFP4 MoE stack, top-10 of 512 uniform)"


def run_batch_decode(args, rank, world):
    """Config 4: a step = one decode step of `--batch` tokens per GPU through all
    `--n-layers` MoE layers; router logits ~ N(0,1) (uniform popularity), top-10
    of 512 per layer, x ~ N(0,1) bf16 per layer.  1 GPU: the grouped expert GEMM
    (qmoe.moe_prefill) per layer on the full table, one CUDA graph per step.
    N GPUs: expert-parallel (each rank holds 512/N experts of every layer, its
    own --batch tokens; NCCL all-to-all dispatch and combine per layer)."""
    import torch
    import qmoe
    import routing
    from expert_table import ExpertTable
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = shard = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        import ep
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        shard = ep.ExpertShard(N_EXPERTS, world, rank)
    L, B = args.n_layers, args.batch
    e_local = N_EXPERTS // world
    table = ExpertTable(K=TOPK, dev=dev, n_layers=L, n_experts=e_local)
    table.fill_synthetic(seed=args.seed + rank)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 23 + 1000 * rank)
    R = 2
    xs = torch.randn(R, L, B, HID, device=dev, generator=g).to(torch.bfloat16)
    ti, tv = routing.route(torch.randn(R * L * B, N_EXPERTS, device=dev, generator=g), TOPK)
    ti, tv = ti.view(R, L, B, TOPK).contiguous(), tv.view(R, L, B, TOPK).contiguous()
    distinct = [[int(torch.unique(ti[r, l]).numel()) for l in range(L)] for r in range(R)]

    mode = "ag" if args.ep_mode == "auto" else args.ep_mode

    def layer(x, t, v, l):
        if shard is None:
            return qmoe.moe_prefill(x, t, v, table.slots, table.s2[l], l)
        if mode == "ag":
            return ep.moe_prefill_ep_ag(x, t, v, table.slots, table.s2[l], l, shard)
        return ep.moe_prefill_ep(x, t, v, table.slots, table.s2[l], l, shard)

    def step(r):
        for l in range(L):
            layer(xs[r, l], ti[r, l], tv[r, l], l)

    graphs = None
    if shard is None:  # expert-parallel steps run eagerly (NCCL collectives are not captured)
        step(0)
        torch.cuda.synchronize()
        graphs = []
        for r in range(R):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step(r)
            graphs.append(gr)

    def run(r):
        if graphs is not None:
            graphs[r % R].replay()
        else:
            step(r % R)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(max(args.warmup, 3)):
        run(i)
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(st)
        for i in range(args.steps):
            run(i)
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t_ = torch.tensor([ms], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms = float(t_.item())
    tok_s = world * B / (ms * 1e-3)
    step_bytes = sum(sum(d) * BLOCK for d in distinct) / R + L * B * HID * (2 + 4)   # experts + x in + fp32 out
    gbs = step_bytes / (ms * 1e-3) / 1e9

    # e2e: per step every layer's x, ti, tv from pinned host memory and its fp32 output back
    h_x, h_ti, h_tv = xs[0].cpu().pin_memory(), ti[0].cpu().pin_memory(), tv[0].cpu().pin_memory()
    h_out = torch.empty(L, B, HID, dtype=torch.float32).pin_memory()
    d_x, d_ti, d_tv = torch.empty_like(xs[0]), torch.empty_like(ti[0]), torch.empty_like(tv[0])
    h2d = d_x.numel() * 2 + d_ti.numel() * 8 + d_tv.numel() * 2
    d2h = L * B * HID * 4

    def e2e_step():
        d_x.copy_(h_x, non_blocking=True)
        d_ti.copy_(h_ti, non_blocking=True)
        d_tv.copy_(h_tv, non_blocking=True)
        for l in range(L):
            h_out[l].copy_(layer(d_x[l], d_ti[l], d_tv[l], l), non_blocking=True)

    E = min(args.e2e_steps, 8)
    e2e_step()
    barrier()
    e0.record(st)
    for _ in range(E):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / E
    if dist is not None:
        t_ = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms_e2e = float(t_.item())

    peak, peak_kind = peaks()
    line = {
        "metric": BD_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 tensor-core products of nvfp4 weights (exact) and bf16 activations, "
                                      "fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"batch-decode (config 4): {B} tokens per GPU, {L} layers, top-{TOPK} of "
                               f"{N_EXPERTS} uniform; {sum(map(sum, distinct)) / R / L:.0f} distinct experts per "
                               f"layer per rank's tokens",
                   "hbm_gbs": gbs, "bytes_per_step": step_bytes,
                   "l2": "no flush: each step reads ~48 GB of distinct expert blocks (>> 126 MB L2)",
                   "parallelism": (f"expert-parallel x{world} (NCCL " +
                                   ("all-gather + reduce-scatter" if mode == "ag" else "all-to-all dispatch/combine")
                                   + ")") if world > 1
                   else "single GPU"},
        "e2e": {"value": world * B / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E, "ms_per_step": ms_e2e,
                "path": "qmoe.moe_prefill per layer (public API, eager) with pinned host inputs and outputs"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_kind": peak_kind, "traffic": None,
                     "kernel": "pf_gemm<gate/up> + pf_gemm<down> (+ routing, gather, h packing) per layer"},
        "gpu_launches": args.steps * L * 6,
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline and world == 1:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import numpy as np
        import oracle
        cores = oracle.threads(os.cpu_count())
        n = min(8, B)
        t_l = ti[0, 0, :n].cpu().numpy()
        used = np.unique(t_l)
        remap = {int(e): i for i, e in enumerate(used)}
        ti_local = np.vectorize(lambda e: remap[int(e)])(t_l).astype(np.int32)
        blocks = table.slots[torch.from_numpy(used).to(dev)].cpu().numpy()
        s2_local = table.s2[0][torch.from_numpy(used).to(dev)].cpu().numpy()
        t0 = time.perf_counter()
        oracle.moe_prefill(xs[0, 0, :n].float().cpu().numpy(), ti_local, tv[0, 0, :n].float().cpu().numpy(),
                           blocks, 0, s2_local)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": n / (dt * L), "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": f"{n} tokens of layer 0 ({len(used)} experts: block dequant + fp32 GEMMs "
                                          f"+ index_add) in {dt:.1f} s, extrapolated x{L} layers"}
    if dist is not None:
        del graphs  # graphs holding NCCL calls go before the process group
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


LIN_COPIES = 4                                 # weight copies per shape, rotated (4 x 42 MB > 126 MB L2)


def run_fp8_linear(args, rank, world):
    """The engine's FP8 linear layer for T > 1 tokens (Lin.__call__,
    qwen_engine.py:79-83): --tokens (2048) tokens through the config-1 shapes
    (12288x2560 and 2560x4096); a step = one call per shape through
    fp8gemv.linear (this library's e4m3 -> bf16 kernel + the bf16 GEMM).  Also
    timed on the same stream: the e4m3 -> bf16 kernel alone (its HBM roofline)
    and the reference's own torch expression F.linear(x, (q.to(bf16) * s).to(bf16)).
    N GPUs: replicas."""
    import torch
    import torch.nn.functional as F
    import fp8gemv
    import synthetic
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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

    def deq_only(i):
        for qs, ss, _ in data.values():
            fp8gemv.dequant_bf16(qs[i % LIN_COPIES], ss[i % LIN_COPIES])

    def reference(i):
        for qs, ss, x in data.values():
            q, sc = qs[i % LIN_COPIES], ss[i % LIN_COPIES]
            F.linear(x, (q.to(torch.bfloat16) * sc).to(torch.bfloat16))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    st = torch.cuda.current_stream()

    def timed(fn, clk=None):
        for i in range(max(args.warmup, 3)):
            fn(i)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(args.steps):
            fn(i)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if dist is not None:
            t_ = torch.tensor([ms], device=dev)
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            ms = float(t_.item())
        return ms

    with ClockSampler(local) as clk:
        ms = timed(ours)
    ms_deq = timed(deq_only)
    ms_ref = timed(reference)

    # e2e: the public call with x copied in from pinned host memory and y read back, every step
    hx = {k: v[2].cpu().pin_memory() for k, v in data.items()}
    hy = {(N, K): torch.empty(T, N, dtype=torch.bfloat16).pin_memory() for (N, K) in GEMV_SHAPES}
    dx = {k: torch.empty_like(v[2]) for k, v in data.items()}

    def e2e(i):
        for k, (qs, ss, _) in data.items():
            dx[k].copy_(hx[k], non_blocking=True)
            hy[k].copy_(fp8gemv.linear(dx[k], qs[i % LIN_COPIES], ss[i % LIN_COPIES]), non_blocking=True)

    ms_e2e = timed(e2e)
    flop = sum(2 * T * N * K for (N, K) in GEMV_SHAPES)
    deq_bytes = sum(3 * N * K + 4 * N for (N, K) in GEMV_SHAPES)
    value = world * flop / (ms * 1e-3) / 1e12
    hbm, hbm_kind = peaks()
    deq_gbs = deq_bytes / (ms_deq * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": f"fp8 linear layer, T={T} tokens, TFLOP/s (config-1 weight shapes)", "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 weights -> bf16, bf16 GEMM, fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"fp8-linear: {T} tokens x (12288x2560 + 2560x4096), bf16 out",
                       "us_reference_expression_same_gpu": ms_ref * 1e3, "us_dequant_kernel": ms_deq * 1e3,
                       "l2": f"no flush: {LIN_COPIES} rotated weight copies per shape (> 126 MB L2)",
                       "parallelism": "single GPU" if world == 1 else f"{world} replicas"},
            "e2e": {"value": world * flop / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": sum(T * K * 2 for (N, K) in GEMV_SHAPES),
                    "d2h_bytes_per_step": sum(T * N * 2 for (N, K) in GEMV_SHAPES), "ms_per_step": ms_e2e,
                    "path": "fp8gemv.linear (public API) with pinned host x in and y out"},
            "roofline": {"bound": "hbm", "achieved": deq_gbs, "peak": hbm, "unit": "GB/s", "frac": deq_gbs / hbm,
                         "peak_kind": hbm_kind, "traffic": None,
                         "kernel": "e4m3_rows_to_bf16_kernel (3 B per weight); the GEMM is cuBLAS"},
            "gpu_launches": args.steps * len(GEMV_SHAPES),
            "clocks": clk.summary(),
        }))
    if dist is not None:
        dist.destroy_process_group()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.workload == "prefill":
        return run_prefill(args, rank, world)
    if args.workload == "gemv":
        return run_gemv(args, rank, world)
    if args.workload == "batch-decode":
        return run_batch_decode(args, rank, world)
    if args.workload == "fp8-linear":
        return run_fp8_linear(args, rank, world)

    import torch
    import qmoe
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    table, sidx, s2, coef, x = build_workload(args, dev)
    L, R = args.n_layers, args.routes
    hb = torch.empty(TOPK, INTER, device=dev)
    ob = torch.empty(TOPK, HID, device=dev)

    def step_eager(r, outs=None):
        for l in range(L):
            if args.variant:
                y = qmoe._moe_decode(table.slots, sidx[r, l], s2[r, l], coef[r, l], x[r, l], hb, args.variant)
            else:
                y = qmoe.moe_decode(table.slots, sidx[r, l], s2[r, l], coef[r, l], x[r, l], hb, ob)
            if outs is not None:
                outs.append(y)

    # one CUDA graph per routed step (one kernel per layer)
    step_eager(0)
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs = []
    for r in range(R):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, pool=pool):
            step_eager(r)
        graphs.append(gr)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        graphs[i % R].replay()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        e0.record(st)
        for i in range(args.steps):
            graphs[(args.warmup + i) % R].replay()
        e1.record(st)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_bytes = L * LAYER_BYTES
    value = world * args.steps * step_bytes / (ms * 1e-3) / 1e9
    us_layer = ms * 1e3 / (args.steps * L)

    # e2e: public API, eager, host inputs copied in and outputs copied out every step
    E = min(args.e2e_steps, R)
    h_x = x[:E].cpu().pin_memory()
    h_sidx, h_s2, h_coef = sidx[:E].cpu().pin_memory(), s2[:E].cpu().pin_memory(), coef[:E].cpu().pin_memory()
    d_x, d_sidx = torch.empty_like(x[0]), torch.empty_like(sidx[0])
    d_s2, d_coef = torch.empty_like(s2[0]), torch.empty_like(coef[0])
    h_out = torch.empty(E, L, HID).pin_memory()
    h2d = d_x.numel() * 2 + d_sidx.numel() * 4 + d_s2.numel() * 4 + d_coef.numel() * 4
    d2h = L * HID * 4

    # per-layer views of the step's input buffers (the caller's per-layer tensors)
    per_layer = [(d_sidx[l], d_s2[l], d_coef[l], d_x[l]) for l in range(L)]

    def e2e_step(r):
        d_x.copy_(h_x[r], non_blocking=True)
        d_sidx.copy_(h_sidx[r], non_blocking=True)
        d_s2.copy_(h_s2[r], non_blocking=True)
        d_coef.copy_(h_coef[r], non_blocking=True)
        outs = [qmoe.moe_decode(table.slots, si, s2l, cl, xl, hb, ob) for si, s2l, cl, xl in per_layer]
        h_out[r].copy_(torch.stack(outs), non_blocking=True)

    for r in range(min(3, E)):
        e2e_step(r)
    barrier()
    e0.record(st)
    for r in range(E):
        e2e_step(r)
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e_value = world * E * step_bytes / (ms_e2e * 1e-3) / 1e9

    peak, peak_kind = peaks()
    achieved = LAYER_BYTES / (us_layer * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 weights (e2m1 + e4m3 scales), fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"decode-moe-{L}L (config 2): bs=1, top-{TOPK} of {N_EXPERTS}, Zipf(1.1), "
                               f"{L}x{N_EXPERTS} experts resident ({L * N_EXPERTS * BLOCK / 2**30:.1f} GiB)",
                   "routes": R, "layer_bytes": LAYER_BYTES, "us_per_layer": us_layer,
                   "l2": "no flush: each step streams >1.3 GB of distinct expert bytes (> 126 MB L2)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": E, "ms_per_step": ms_e2e / E, "path": "qmoe.moe_decode (eager, public API)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "kernel": {0: "moe_decode_slice", 4: "moe_decode_slice", 3: "moe_decode_stream",
                                2: "moe_gate_up_generic + moe_down_generic", 1: "moe_decode_persistent"}
                     .get(args.variant, "?") + " (one launch per decode layer)",
                     # DRAM bytes read + written per launch in the ncu capture of
                     # profiles/moe_decode_slice_decode-layer.md (same layer shape)
                     "traffic": TRAFFIC_DECODE_SLICE if args.variant in (0, 4) else None,
                     "per_launch_bytes": LAYER_BYTES},
        "gpu_launches": args.steps * L,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, table, sidx, s2, coef, x)
    if dist is not None:
        del graphs
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def cpu_baseline(args, table, sidx, s2, coef, x):
    """The C oracle on this host's cores, on the first layers of routed step 0
    (the same expert bytes the GPU read)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle
    cores = oracle.threads(os.cpu_count())
    n = min(args.cpu_layers, args.n_layers)
    layers = []
    for l in range(n):
        rows = sidx[0, l].long()
        blocks = table.slots[rows].cpu().numpy()
        layers.append((blocks, np.arange(TOPK, dtype=np.int32), s2[0, l].cpu().numpy(), coef[0, l].cpu().numpy(),
                       x[0, l].float().cpu().numpy()))
    oracle.moe_decode(*layers[0])
    t0 = time.perf_counter()
    for a in layers:
        oracle.moe_decode(*a)
    dt = time.perf_counter() - t0
    return {"value": n * LAYER_BYTES / dt / 1e9, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} layers of routed step 0 (C oracle: dequantize + fp32 SwiGLU + combine), "
                      f"{dt / n * 1e3:.1f} ms/layer"}


if __name__ == "__main__":
    main()
