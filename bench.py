"""Benchmark of the B200 FP8 MoE layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload mixtral|dsv3|qwen3|tiny] [--impl reference]

A step is one forward of the MoE FFN layer of the workload through the scheme
API (``SchemeInstance.run()``): quant -> all-gather -> align -> GEMM1 -> GEMM2 ->
combine -> reduce-scatter.  Default workload: the Mixtral-8x7B shape of the
BASELINE configs (T=4096 tokens, H=4096, I=14336, E=8, top-2) with TP=N over the
N GPUs (strong scaling: the layer's T tokens are fixed, sharded T/N per rank).
Inputs are seeded synthetic tensors with the config's shapes and value
distributions (no dataset); the weights (>= 176 MB per rank) are larger than L2,
and L2 is also flushed (256 MB write) between timed steps, outside the events.

``value``: tokens/s of the whole layer (T / step time, step time = per-step max
over ranks, mean over steps), device-timed with CUDA events on inputs resident
in HBM.  ``e2e``: the same metric through ``SchemeInstance.run()`` with the
inputs copied from pinned host memory and the output copied back inside the
timed region.  ``roofline``: GEMM1 (gate/up, the dominant kernel) FP8 FLOPs of
the routed (unpadded) pairs over its event-timed duration, against the measured
FP8 dense peak in ``profiles/peaks.json``.  ``cpu_baseline``: the reference
algorithm (``oracle.golden.golden_moe``, the numpy restatement of
``moe_bench/verify.py:14-47``) timed on this host on a bounded token sample.
``--impl reference`` times only that CPU path (rank 0; other ranks exit 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: (preset, human label)
    "mixtral": ("mixtral", "mixtral-8x7b-moe-layer TP"),
    "dsv3": ("dsv3", "deepseek-v3-moe-layer EP (+shared)"),
    "qwen3": ("qwen3", "qwen3-30b-a3b-moe-layer TP decode"),
    "tiny": ("tiny", "tiny-moe-layer"),
}
# scheme code by (parallelism, exchange): d3/d4 fuse the all-gather / reduce-scatter
# through peer memory; d1/d2 are the unfused NCCL comparison (identical at N=1).
SCHEME = {("TP", "p2p"): "d3", ("EP", "p2p"): "d4", ("TP", "nccl"): "d1", ("EP", "nccl"): "d2"}


def _peaks() -> dict:
    out = {}
    mp = ROOT / "MEASURED_PEAKS.json"
    if mp.exists():
        out.update(json.loads(mp.read_text()))
    pp = ROOT / "profiles" / "peaks.json"
    if pp.exists():
        out.update(json.loads(pp.read_text()))
    return out


class ClockSampler:
    """SM clock and clock-event-reason sampling during the timed region.

    A thread reads this GPU's NVML counters (read-only queries; nothing is set) every
    `period` seconds; NVML is initialised and the device handle resolved (by UUID, so
    CUDA and NVML orderings cannot be confused) before the region starts, and one
    sample is taken synchronously at entry and at exit so that even a region of a few
    milliseconds has samples.  Records the SM clock, its maximum and the reasons
    hw_slowdown / hw_thermal_slowdown / sw_thermal_slowdown / sw_power_cap.
    """
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))

    def __init__(self, device, period: float = 0.002):
        import threading
        self.period = period
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        self.nv = None
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self._reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.masks = [(n, int(getattr(nv, attr, bit))) for n, attr, bit in self.REASONS]
            self.nv = nv
        except Exception as e:  # no NVML: the line says so
            self.error = f"{type(e).__name__}: {e}"

    def _sample(self) -> None:
        self.samples.append((float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)),
                             int(self._reasons(self.h))))

    def _loop(self) -> None:
        while not self._stop.wait(self.period):
            try:
                self._sample()
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
                return

    def __enter__(self):
        import threading
        if self.nv is not None:
            self._sample()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._sample()
            self._stop.set()
            self._thread.join()

    def summary(self) -> dict:
        sm = [c for c, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, m in self.masks if r & m}) if self.nv else []
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "NVML"}
        if self.error:
            out["error"] = self.error
        return out

    @staticmethod
    def merge(parts: list[dict]) -> dict:
        """All ranks' summaries: median of the per-rank medians, lowest rank median, union of reasons."""
        med = [p["sm_mhz"] for p in parts if p.get("sm_mhz") is not None]
        out = {"sm_mhz": statistics.median(med) if med else None,
               "sm_mhz_min_rank": min(med) if med else None,
               "sm_max_mhz": max((p["sm_max_mhz"] for p in parts if p.get("sm_max_mhz")), default=None),
               "reasons": sorted({r for p in parts for r in p.get("reasons", [])}),
               "samples": sum(p.get("samples", 0) for p in parts), "ranks": len(parts), "source": "NVML"}
        errs = [p["error"] for p in parts if p.get("error")]
        if errs:
            out["error"] = errs[0]
        return out


def gemm1_flops(topk_ids, expert_map, inter_local: int, hidden: int) -> float:
    """Algorithmic FP8 FLOPs of GEMM1 on this rank: 2 * (routed local pairs) * 2I_r * H (pads not counted)."""
    ids = topk_ids.reshape(-1)
    pairs = int(ids.numel()) if expert_map is None else int((expert_map[ids.long()] >= 0).sum().item())
    return 2.0 * pairs * 2 * inter_local * hidden


def layer_flops(cfg, topk_ids, expert_map, world: int, parallel: str) -> float:
    """Per-rank algorithmic FLOPs of the layer (routed + shared), unpadded."""
    s = cfg.shape
    ids = topk_ids.reshape(-1)
    if parallel == "TP":
        f = 6.0 * s.K * s.intermediate * ids.numel() / world
    else:
        pairs = ids.numel() if expert_map is None else int((expert_map[ids.long()] >= 0).sum().item())
        f = 6.0 * s.K * s.intermediate * pairs
    if s.shared_experts:
        tok = s.M_aligned(world) if parallel == "TP" else s.M_aligned(world) // world
        f += 6.0 * s.K * s.shared_intermediate * tok / (world if parallel == "TP" else 1)
    return f


class CpuGolden:
    """The numpy restatement of the reference golden (``moe_bench/verify.py:14-47``) on this host.

    Weights are held as bf16 bit patterns and widened per expert inside the loop,
    as the reference golden does (``w1_bf16[expert].float()``); the sample is the
    first ``n`` tokens of the same layer (every expert they route to is computed).
    """

    def __init__(self, bundle):
        import numpy as np
        import torch

        from td_benchmark_b200.weights import dequantize_block128

        ck = bundle.ckpt

        def bits(qt):
            return None if qt is None else dequantize_block128(qt.fp8, qt.scale).view(torch.int16).cpu().numpy().view(
                np.uint16)

        self.w1, self.w2, self.sw1, self.sw2 = bits(ck.w1), bits(ck.w2), bits(ck.shared_w1), bits(ck.shared_w2)
        self.hid = bundle.hidden_full.float().cpu().numpy()
        self.ids = bundle.routing.topk_ids_full.cpu().numpy()
        self.wts = bundle.routing.topk_weights_full.cpu().numpy()
        self.cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()

    def run(self, n: int) -> float:
        from oracle import golden as ogolden

        t0 = time.perf_counter()
        ogolden.golden_moe(self.hid[:n], self.ids[:n], self.wts[:n], self.w1, self.w2, self.sw1, self.sw2)
        return time.perf_counter() - t0

    def calibrate(self, budget_s: float) -> int:
        """Largest power-of-two token sample (>= 16) whose run fits the budget."""
        n = min(16, self.hid.shape[0])
        t = self.run(n)
        while 2 * t < budget_s and n < self.hid.shape[0]:
            n = min(self.hid.shape[0], n * 2)
            t = self.run(n)
        return n

    def describe(self, n: int, runs: int, mean_t: float) -> dict:
        return {"value": n / mean_t, "unit": "tokens/s", "cores": self.cores, "kind": "port",
                "sample": f"first {n} of {self.hid.shape[0]} tokens through the full layer (numpy fp32 golden of "
                          f"moe_bench/verify.py:14-47, BLAS threads = host cores); mean of {runs} run(s), "
                          f"{mean_t:.2f} s each"}


def run_reference(args) -> int:
    import torch

    from td_benchmark_b200 import configs, data

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    preset, label = WORKLOADS[args.workload]
    over = {"M": args.tokens} if args.tokens else {}
    cfg = configs.preset(preset, **over)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    gold = CpuGolden(data.build_bundle(cfg, device=dev))
    n = gold.calibrate(budget_s=min(15.0, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        gold.run(n)
    times = [gold.run(n) for _ in range(args.steps)]
    mean_t = sum(times) / len(times)
    cb = gold.describe(n, len(times), mean_t)
    s = cfg.shape
    line = {"impl": "reference", "metric": "moe_layer_tokens_per_s", "value": cb["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean_t * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded, BASELINE value distributions)",
            "config": {"workload": label, "tokens": s.M, "hidden": s.K, "intermediate": s.intermediate,
                       "experts": s.E, "top_k": s.top_k},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def _stages(starts, ends, evs) -> dict:
    """Median duration (us) of each stage of a step, keyed by the event that closes it.

    Every step records the same sequence of named events, so the list splits evenly."""
    n = len(evs) // max(1, len(starts))
    acc: dict[str, list[float]] = {}
    for i, (a, b) in enumerate(zip(starts, ends)):
        seq = evs[i * n:(i + 1) * n] + [("step_end", b)]
        prev = a
        for name, ev in seq:
            acc.setdefault(name, []).append(prev.elapsed_time(ev) * 1e3)
            prev = ev
    return {k: statistics.median(v) for k, v in acc.items()}


def _max_over_ranks(d: dict, world: int, dev) -> dict:
    import torch
    import torch.distributed as dist
    if world == 1 or not d:
        return d
    v = torch.tensor(list(d.values()), dtype=torch.float64, device=dev)
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return dict(zip(d.keys(), v.tolist()))


def _before_gemm1(starts, evs) -> float:
    """Mean time (ms) from each step's start to its gate/up GEMM launch point."""
    g = [ev for name, ev in evs if name == "gemm1_start"]
    t = [a.elapsed_time(b) for a, b in zip(starts, g)]
    return sum(t) / max(1, len(t))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="mixtral", choices=sorted(WORKLOADS))
    ap.add_argument("--tokens", type=int, default=None, help="override the workload's token count")
    ap.add_argument("--impl", default="b2m", choices=["b2m", "reference"])
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"],
                    help="exchange of the multi-GPU layer: fused peer memory (default) or NCCL")
    ap.add_argument("--rs-mode", default="sm", choices=["sm", "gemm", "ce"],
                    help="fused reduce-scatter: SM stores from the combine (default), from the down GEMM's epilogue, "
                         "or copy-engine push")
    ap.add_argument("--ag-mode", default="auto", choices=["auto", "sm", "ce", "push"],
                    help="fused all-gather: SM stores from the quant kernel, copy-engine copies, or by block size")
    ap.add_argument("--chunks", type=int, default=4, help="down-GEMM column chunks of the copy-engine push")
    ap.add_argument("--ce-streams", type=int, default=2, help="side streams carrying the copy-engine push")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from td_benchmark_b200 import configs, data
    from td_benchmark_b200.context import init_context
    from td_benchmark_b200.schemes import REGISTRY
    from td_benchmark_b200.schemes.b200 import build_layer

    ctx = init_context(backend="nccl", timeout_s=300.0)
    world, rank = ctx.world_size, ctx.rank
    dev = ctx.device
    preset, label = WORKLOADS[args.workload]
    over = {"M": args.tokens} if args.tokens else {}
    cfg = configs.preset(preset, **over)
    code = SCHEME[(cfg.parallel, args.comm)]
    spec = REGISTRY[code][0]
    bundle = data.build_bundle(cfg, rank=rank, world_size=world, device=dev)
    exchange = None
    if world > 1 and args.comm == "p2p":
        from td_benchmark_b200.layer import P2PExchange
        exchange = P2PExchange(ctx.group, chunks=args.chunks, rs_mode=args.rs_mode, ce_streams=args.ce_streams,
                               ag_mode=args.ag_mode)
    layer, level = build_layer(spec, cfg, ctx, bundle, exchange=exchange)
    T = layer.T
    x = bundle.hidden_local.contiguous()
    ids = bundle.routing.topk_ids_full.contiguous()
    wts = bundle.routing.topk_weights_full.contiguous()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-timed steps (inputs resident).  Warm-up steps run exactly what a timed
    # step runs (flush included) so that no first launch or lazy module load lands in
    # the timed region; the clock sampler is up before the barrier that opens it.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    layer.events = []
    for _ in range(args.warmup):
        flush.zero_()
        layer.forward(x, ids, wts)
    torch.cuda.synchronize()
    layer.check()
    layer.events = []
    clk = ClockSampler(dev)
    host_s = 0.0
    with clk:
        barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            h0 = time.perf_counter()
            layer.forward(x, ids, wts)
            host_s += time.perf_counter() - h0
            ends[i].record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    layer.check()
    local = torch.tensor([s.elapsed_time(e) for s, e in zip(starts, ends)], dtype=torch.float64, device=dev)
    evs = layer.events
    pre_g1 = _before_gemm1(starts, evs)
    stages = _max_over_ranks(_stages(starts, ends, evs), world, dev)
    g1 = []
    layer.events = None
    start = None
    for name, ev in evs:
        if name == "gemm1_start":
            start = ev
        elif name == "gemm1_end" and start is not None:
            g1.append(start.elapsed_time(ev))
            start = None
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
    per_step = local.cpu().tolist()
    ms = sum(per_step) / len(per_step)
    clocks = clk.summary()
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, clocks)
        clocks = ClockSampler.merge(parts)

    # ---- exposed communication (fused exchange, N > 1): the same kernels on local data
    # with every peer flag already satisfied and nothing sent; exposed = fused - that.
    comm = None
    if world > 1 and getattr(layer.exchange, "name", "") == "p2p":
        layer.exchange.compute_only = True
        for _ in range(args.warmup):
            flush.zero_()
            layer.forward(x, ids, wts)
        torch.cuda.synchronize()
        barrier()
        c_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        c_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        layer.events = []
        for i in range(args.steps):
            flush.zero_()
            c_s[i].record()
            layer.forward(x, ids, wts)
            c_e[i].record()
        torch.cuda.synchronize()
        c_pre_g1 = _before_gemm1(c_s, layer.events)
        c_stages = _max_over_ranks(_stages(c_s, c_e, layer.events), world, dev)
        layer.events = None
        layer.exchange.compute_only = False
        pre = torch.tensor([pre_g1, c_pre_g1], dtype=torch.float64, device=dev)
        dist.all_reduce(pre, op=dist.ReduceOp.MAX)
        pre_f, pre_c = (float(v) * 1e3 for v in pre.tolist())
        c_local = torch.tensor([a.elapsed_time(b) for a, b in zip(c_s, c_e)], dtype=torch.float64, device=dev)
        dist.all_reduce(c_local, op=dist.ReduceOp.MAX)
        c_ms = float(c_local.mean().item())
        H_ = cfg.shape.K
        ag_bytes = (world - 1) * layer.T_local * (H_ + 4 * H_ // 128)
        rs_bytes = (world - 1) * layer.T_local * H_ * 2
        comm = {"compute_only_us": c_ms * 1e3, "fused_us": ms * 1e3, "exposed_comm_us": (ms - c_ms) * 1e3,
                "exposed_all_gather_us": pre_f - pre_c, "exposed_reduce_scatter_us": (ms - c_ms) * 1e3 - (pre_f - pre_c),
                "stages_us_max_over_ranks": {"fused": {k: round(v, 1) for k, v in stages.items()},
                                             "compute_only": {k: round(v, 1) for k, v in c_stages.items()}},
                "nvlink_bytes_per_rank": {"all_gather_in": ag_bytes, "reduce_scatter_out": rs_bytes},
                "how": "same kernels with peer flags pre-satisfied and local data (no traffic); per-step max over ranks"}
        barrier()
        layer.forward(x, ids, wts)   # one regular step so every rank's epoch and buffers are in step again
        torch.cuda.synchronize()
        barrier()

    # ---- end-to-end with host buffers: every step copies its inputs from pinned host
    # memory and its result back.  Primary: the double-buffered HostPipeline (transfers of
    # steps i+1 / i-1 overlap the compute of step i), timed over the whole run on the
    # device; the weights and operands exceed L2, so no flush between steps.  Also
    # reported: the same steps run one after another (copies not overlapped).
    from td_benchmark_b200.pipeline import HostPipeline

    x_h = x.cpu().pin_memory()
    ids_h = ids.cpu().pin_memory()
    wts_h = wts.cpu().pin_memory()
    outs_h = [torch.empty(layer.out_local.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    out_h = outs_h[0]
    pipe = HostPipeline(layer)
    cur = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        pipe.submit(x_h, ids_h, wts_h, outs_h[i % 2])
    pipe.drain()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(cur)
    pipe.h2d.wait_stream(cur)
    last = None
    for i in range(args.steps):
        last = pipe.submit(x_h, ids_h, wts_h, outs_h[i % 2])
    cur.wait_event(last)
    p1.record(cur)
    torch.cuda.synchronize()
    barrier()
    e_tot = torch.tensor([p0.elapsed_time(p1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_tot, op=dist.ReduceOp.MAX)
    e_ms = float(e_tot.item()) / args.steps

    x_d, ids_d, wts_d = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(wts)

    def e2e_step():
        x_d.copy_(x_h, non_blocking=True)
        ids_d.copy_(ids_h, non_blocking=True)
        wts_d.copy_(wts_h, non_blocking=True)
        out = layer.forward(x_d, ids_d, wts_d)
        out_h.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        flush.zero_()
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        e_s[i].record()
        e2e_step()
        e_e[i].record()
    torch.cuda.synchronize()
    barrier()
    e_local = torch.tensor([s.elapsed_time(e) for s, e in zip(e_s, e_e)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_local, op=dist.ReduceOp.MAX)
    e_serial_ms = float(e_local.mean().item())
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * 4 + wts_h.numel() * 4
    d2h = out_h.numel() * out_h.element_size()

    # ---- roofline of GEMM1 on this rank
    peaks = _peaks()
    fp8_peak = peaks.get("fp8_tflops")
    peak_src = "measured (profiles/peaks.json)"
    if not fp8_peak:
        fp8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
        peak_src = "2 x measured bf16 (MEASURED_PEAKS.json); no FP8 measurement yet"
    g1_ms = sum(g1) / len(g1)
    f1 = gemm1_flops(ids, layer.expert_map, layer.w.inter, layer.H)
    achieved = f1 / (g1_ms * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get(f"gemm1/{args.workload}/{world}")
    lf = layer_flops(cfg, ids, layer.expert_map, world, spec.parallel)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gold = CpuGolden(bundle)
        n = gold.calibrate(budget_s=15.0)
        cpu = gold.describe(n, 1, gold.run(n))

    if rank == 0:
        s = cfg.shape
        line = {
            "metric": "moe_layer_tokens_per_s", "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3,
            "ms_per_step_min": min(per_step), "ms_per_step_median": statistics.median(per_step),
            "host_enqueue_us_per_step": host_s / args.steps * 1e6,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8-e4m3 (fp32 accum)",
            "data": "synthetic (seeded, BASELINE value distributions)",
            "config": {"workload": label, "tokens": T, "hidden": s.K, "intermediate": s.intermediate,
                       "experts": s.E, "top_k": s.top_k, "parallelism": f"{spec.parallel.lower()}{world}",
                       "scheme": code, "shard_level": level, "routing": cfg.routing.imbalance_kind,
                       "exchange": (f"p2p ag={layer.exchange.ag_mode} rs={args.rs_mode} "
                                    f"chunks={len(layer.exchange.chunk_cols)}"
                                    if getattr(layer.exchange, "name", "") == "p2p" else
                                    getattr(layer.exchange, "name", "none")),
                       "l2": "weights > L2 and 256 MB L2 flush between timed steps"},
            "e2e": {"value": T / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
                    "how": "HostPipeline: pinned-host inputs in and result out every step, double-buffered so the "
                           "copies of steps i+1 / i-1 overlap step i; whole run timed with CUDA events, max over ranks",
                    "serial_ms_per_step": e_serial_ms},
            "gpu_launches": layer.kernel_launches() * args.steps,
            "roofline": {"bound": "tensor", "kernel": "gemm1 (gate/up, tcgen05 kind::f8f6f4)",
                         "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s", "frac": achieved / fp8_peak,
                         "peak_source": peak_src, "traffic": traffic, "gemm1_ms": g1_ms,
                         "layer_tflops": lf / (ms * 1e-3) / 1e12,
                         "layer_frac_of_fp8_peak": lf / (ms * 1e-3) / 1e12 / fp8_peak},
            "clocks": clocks,
            "comm": comm,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
