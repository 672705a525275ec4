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
    p.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                   help="decode: config 2 (default, the headline line); prefill: config 3")
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

    def step(i):
        if shard is None:
            return qmoe.moe_prefill(xs[i % R], tis[i % R], tvs[i % R], table.slots, s2, 0)
        return ep.moe_prefill_ep(xs[i % R], tis[i % R], tvs[i % R], table.slots, s2, 0, shard)

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
            y = ep.moe_prefill_ep(d_x, d_ti, d_tv, table.slots, s2, 0, shard)
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
                   "parallelism": f"expert-parallel x{world} (NCCL all-to-all dispatch/combine)" if world > 1
                   else "single GPU"},
        "e2e": {"value": world * T / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E, "ms_per_step": ms_e2e,
                "path": "qmoe.moe_prefill (public API) with pinned host inputs and output"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": tflops / tc_peak, "peak_kind": tc_kind,
                     "hbm_frac": gbs / peaks()[0], "traffic": None,
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


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.workload == "prefill":
        return run_prefill(args, rank, world)

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

    # one CUDA graph per routed step (48 layers x 2 kernels each)
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

    def e2e_step(r):
        d_x.copy_(h_x[r], non_blocking=True)
        d_sidx.copy_(h_sidx[r], non_blocking=True)
        d_s2.copy_(h_s2[r], non_blocking=True)
        d_coef.copy_(h_coef[r], non_blocking=True)
        outs = [qmoe.moe_decode(table.slots, d_sidx[l], d_s2[l], d_coef[l], d_x[l], hb, ob) for l in range(L)]
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
                     "traffic": None, "per_launch_bytes": LAYER_BYTES},
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
