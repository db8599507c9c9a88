"""Benchmark of the B200 FP8 MoE layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dsv3|mixtral|qwen3|tiny] [--impl reference]

A step is one forward of the MoE FFN layer of the workload: align -> quant ->
all-gather -> dispatch -> GEMM1 (+SiLU*mul+requant) -> GEMM2 (*routed weight) ->
combine (+shared expert) -> reduce-scatter.  Default workload: the DeepSeek-V3
shape of the BASELINE configs (T=8192 tokens, H=7168, I=2048, E=256, top-8, Zipf
1.2 routing, one shared expert of I=2048) with EP=N over the N GPUs (strong
scaling: the layer's T tokens are fixed, T/N per rank); ``--workload mixtral``
is the Mixtral-8x7B TP shape.  Inputs are seeded synthetic tensors with the
config's shapes and value distributions (no dataset); the weights are larger than
L2, and L2 is also flushed (256 MB write) between timed steps, outside the events.

``value``: tokens/s of the whole layer (T / step time, step time = per-step max
over ranks, mean over steps), device-timed with CUDA events on inputs resident
in HBM.  ``e2e``: the same metric with the inputs copied from pinned host memory
and the output copied back every step (``HostPipeline``).  ``roofline``: GEMM1
(gate/up, the dominant kernel) FP8 FLOPs of the routed (unpadded) pairs over its
event-timed duration against the measured FP8 dense peak, and under ``layer`` the
layer's FP8 / NVLink / HBM terms of the most-loaded rank.  ``comm`` (N > 1):
exposed communication and the hidden fraction.  ``parity``: every rank's output of
a forward after the timed runs against the fp32 golden (the reference worker's
gates plus a calibrated max-abs bound).  ``cpu_baseline``: the reference
algorithm (``oracle.golden``, the numpy restatement of ``moe_bench/verify.py:14-47``)
on the whole layer on this host's cores.  ``--impl reference`` times only that CPU
path (rank 0; other ranks exit 0), the same whole-layer run at every N.
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


def rank_work(layer, topk_ids, inter: int, shared_inter: int, rs_fp8: bool = False) -> dict:
    """This rank's algorithmic work in one forward: FP8 FLOPs (routed pairs, unpadded, plus the
    shared expert), the expert weight bytes it must stream from HBM, and its NVLink bytes
    (all-gather received + reduce-scatter sent, bf16 partials) -- the three roofline terms.
    ``inter`` / ``shared_inter``: this rank's unpadded intermediate widths."""
    ids = topk_ids.reshape(-1).long()
    H, I, P = layer.H, inter, layer.P
    if layer.expert_map is None:
        pairs = ids.numel()
        hit = int(torch_unique_count(ids))
    else:
        local = layer.expert_map[ids] >= 0
        pairs = int(local.sum().item())
        hit = int(torch_unique_count(ids[local]))
    flops = 6.0 * H * I * pairs
    wbytes = hit * 3.0 * H * I * (1 + 4.0 / (128 * 128))
    if layer.shared is not None:
        Is = shared_inter
        flops += 6.0 * H * Is * layer.shared.rows
        wbytes += 3.0 * H * Is * (1 + 4.0 / (128 * 128))
    row_fp8 = H + 4 * H // 128
    rows = (P - 1) * layer.T_local          # dense: every other rank's tokens in, every partial out
    ex = layer.exchange
    if getattr(ex, "sparse", False):
        # only the tokens of other ranks that route to one of this rank's experts cross in
        # (all-gather) and their partials out (reduce-scatter)
        r = ex.rank
        tl = layer.T_local
        rk = layer.expert_owner[topk_ids.long()]
        hit = (rk == r).any(dim=1)
        hit[r * tl:(r + 1) * tl] = False
        rows = int(hit.sum().item())
    ag = rows * row_fp8
    rs = rows * (row_fp8 if rs_fp8 else 2 * H)
    if getattr(ex, "rs_mode", None) == "gemm":
        # the down GEMM sends each computed pair row (not a per-token partial) to its token's owner
        tok = torch_arange_like(ids) // layer.top_k
        remote = (tok // layer.T_local) != ex.rank
        if layer.expert_map is not None:
            remote &= layer.expert_map[ids] >= 0
        rs = int(remote.sum().item()) * 2 * H
    return {"flops": flops, "weight_bytes": wbytes, "nvlink_bytes": float(ag + rs), "ag_bytes": ag, "rs_bytes": rs,
            "pairs": pairs, "experts_hit": hit}


def torch_arange_like(t):
    import torch
    return torch.arange(t.numel(), device=t.device)


def torch_unique_count(t) -> int:
    import torch
    return int(torch.unique(t).numel()) if t.numel() else 0


SAMPLE = 2048   # tokens per CPU run: a whole-layer DeepSeek-V3 run takes ~15 s on 16 host cores


class CpuGolden:
    """The numpy restatement of the reference golden (``moe_bench/verify.py:14-47``) on this host.

    Weights are held as bf16 bit patterns and widened per expert inside the loop, as the
    reference golden does (``w1_bf16[expert].float()``).  One run is a fixed sample of the
    layer: its first ``SAMPLE`` tokens (all of them when T is smaller), every expert they
    route to computed -- the same sample at every N and in the main arm's cpu_baseline.  The expert loop runs on every host core the process may use
    (``golden_moe_threads``: whole experts per thread, BLAS single-threaded per thread when
    there are enough experts to go round, else BLAS threads split the cores), whatever
    thread limit the launcher set in the environment (torchrun sets OMP_NUM_THREADS=1).
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
        self.total = bundle.hidden_full.shape[0]
        n = min(SAMPLE, self.total)
        self.hid = bundle.hidden_full[:n].float().cpu().numpy()
        self.ids = bundle.routing.topk_ids_full[:n].cpu().numpy()
        self.wts = bundle.routing.topk_weights_full[:n].cpu().numpy()
        self.cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        hit = len(set(self.ids.reshape(-1).tolist()))
        self.workers = max(1, min(self.cores, hit))
        self.blas_threads = max(1, self.cores // self.workers)

    def run(self) -> float:
        from threadpoolctl import threadpool_limits

        from oracle import golden as ogolden

        with threadpool_limits(limits=self.blas_threads, user_api="blas"):
            t0 = time.perf_counter()
            ogolden.golden_moe_threads(self.hid, self.ids, self.wts, self.w1, self.w2, self.sw1, self.sw2,
                                       workers=self.workers)
            return time.perf_counter() - t0

    def describe(self, runs: int, mean_t: float) -> dict:
        n = self.hid.shape[0]
        return {"value": n / mean_t, "unit": "tokens/s", "cores": self.cores, "kind": "port",
                "sample": f"the first {n} of the layer's {self.total} tokens per run, every expert they route to "
                          f"(numpy fp32 golden of moe_bench/verify.py:14-47, per-expert bf16 widening inside the "
                          f"loop; the same sample at every N); {self.workers} "
                          f"expert threads x {self.blas_threads} BLAS thread(s) on {self.cores} host cores; "
                          f"mean of {runs} run(s), {mean_t:.2f} s each"}


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
    for _ in range(args.warmup):
        gold.run()
    times = [gold.run() for _ in range(args.steps)]
    mean_t = sum(times) / len(times)
    cb = gold.describe(len(times), mean_t)
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


def _timed(fn, steps: int, warmup: int, flush, barrier, events=None):
    """Per-step CUDA-event times (ms) of ``fn`` on the current stream: warm-up steps run
    exactly what a timed step runs, the L2 flush sits between steps outside the events."""
    import torch

    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    s = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        s[i].record()
        fn()
        e[i].record()
    torch.cuda.synchronize()
    barrier()
    return [a.elapsed_time(b) for a, b in zip(s, e)]


def _mean_max_over_ranks(times: list[float], world: int, dev) -> float:
    """Mean over steps of the per-step maximum over ranks (ms)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(times, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.mean().item())


def exchange_split(layer, bundle, x, ids, wts, args, flush, barrier, world, dev, fused_ms: float) -> dict | None:
    """Exposed communication of the fused exchange and the fraction of it that is hidden.

    * compute: this rank's shard of the layer run as a one-GPU layer (every token local,
      no exchange: align, quant + dispatch, GEMM1, GEMM2, combine), plus its shared expert;
    * comm: the exchange kernels of one step with no GEMM between them
      (``P2PExchange.exchange_alone``: quantise + push + dispatch, combine + push + owner reduce);
    * exposed = fused - compute; hidden fraction = 1 - exposed / comm.
    All per-step maxima over ranks, means over steps."""
    import torch

    from td_benchmark_b200.layer import MoELayer, NullExchange

    ex = layer.exchange
    if getattr(ex, "name", "") != "p2p" or world == 1:
        return None
    solo = MoELayer(layer.w, layer.T, layer.top_k, layer.E, expert_map=layer.expert_map, shared=None,
                    exchange=NullExchange(), device=layer.device)
    x_all = bundle.hidden_full.to(dev).contiguous()
    t_solo = _timed(lambda: solo.forward(x_all, ids, wts), args.steps, args.warmup, flush, barrier)
    solo.check()
    del solo
    t_shared = [0.0] * args.steps
    if layer.shared is not None:
        t_shared = _timed(lambda: layer.shared.run(layer.status), args.steps, args.warmup, flush, barrier)
    compute_ms = _mean_max_over_ranks([a + b for a, b in zip(t_solo, t_shared)], world, dev)
    comm_ms = None
    if ex.exchange_alone(layer, x, ids):
        t_comm = _timed(lambda: ex.exchange_alone(layer, x, ids), args.steps, args.warmup, flush, barrier)
        comm_ms = _mean_max_over_ranks(t_comm, world, dev)
    layer.check()
    exposed = fused_ms - compute_ms
    out = {"fused_us": fused_ms * 1e3, "compute_us": compute_ms * 1e3, "exposed_comm_us": exposed * 1e3,
           "comm_alone_us": None if comm_ms is None else comm_ms * 1e3,
           "hidden_frac": None if not comm_ms else 1.0 - exposed / comm_ms,
           "how": "compute = this rank's shard run as a one-GPU layer (no exchange) + its shared expert; comm = "
                  "the exchange kernels of a step alone (P2PExchange.exchange_alone); exposed = fused - compute; "
                  "hidden = 1 - exposed/comm; per-step max over ranks, mean over steps"}
    return out


def check_parity(layer, bundle, x, ids, wts, world, rank, dev, parallel: str, rs_fp8: bool) -> dict:
    """One more regular forward, every rank's rows against the fp32 golden of the same tokens
    (the reference worker's gates + max-abs <= 1.5 x calibrated activation-quant error, plus
    the quantisation error of the ranks' partials when the reduce-scatter payload is FP8)."""
    import torch
    import torch.distributed as dist

    from td_benchmark_b200 import verify

    out = layer.forward(x, ids, wts)
    torch.cuda.synchronize()
    layer.check()
    r0, n = rank * layer.T_local, layer.T_local
    hid = bundle.hidden_full[r0:r0 + n].to(dev)
    extra = 0.0
    if rs_fp8 and world > 1:
        owner = None if layer.expert_owner is None else layer.expert_owner.cpu().tolist()
        extra = verify.rs_fp8_error(verify.rank_partials(hid, ids[r0:r0 + n], wts[r0:r0 + n], bundle.ckpt, world,
                                                         parallel, owner))
    rep = verify.check_layer(out, hid, ids[r0:r0 + n], wts[r0:r0 + n], bundle.ckpt, extra_calib=extra)
    v = torch.tensor([1.0 if rep["pass"] else 0.0, rep["cos_sim"], rep["rel_p99"], rep["max_abs"], rep["calib"],
                      abs(rep["scale"] - 1.0), rep["max_abs"] / max(rep["max_abs_bound"], 1e-30)],
                     dtype=torch.float64, device=dev)
    if world > 1:
        parts = [torch.empty_like(v) for _ in range(world)]
        dist.all_gather(parts, v)
        allv = torch.stack(parts)
    else:
        allv = v[None]
    a = allv.cpu().tolist()
    return {"pass": all(r[0] == 1.0 for r in a), "ranks": world, "cos_min": min(r[1] for r in a),
            "rel_p99_max": max(r[2] for r in a), "max_abs_max": max(r[3] for r in a),
            "calib_min": min(r[4] for r in a), "scale_dev_max": max(r[5] for r in a),
            "max_abs_over_bound_max": max(r[6] for r in a),
            "gates": "cos >= 0.995, masked rel_p99 <= 5, |scale-1| <= 0.05 (moe_bench/worker.py:108-110) and max_abs "
                     "<= 1.5 x calib (calib = max |golden - golden without activation quant| on the same rows)",
            "how": "after the timed runs: one regular forward; each rank's output rows vs the fp32 golden of its "
                   "tokens computed on the device (td_benchmark_b200.verify)"}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="dsv3", choices=sorted(WORKLOADS))
    ap.add_argument("--tokens", type=int, default=None, help="override the workload's token count")
    ap.add_argument("--impl", default="b2m", choices=["b2m", "reference"])
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"],
                    help="exchange of the multi-GPU layer: fused peer memory (default) or NCCL")
    ap.add_argument("--rs-mode", default="auto", choices=["auto", "sm", "gemm", "ce"],
                    help="fused reduce-scatter: rows stored to their owners by the down GEMM (gemm), SM stores from "
                         "the combine (sm), copy-engine push (ce); auto (default): gemm when the pair rows are at most "
                         "twice the partials' bytes (top_k <= 2 TP, <= 2P EP) or with >= 2048 local tokens, else sm")
    ap.add_argument("--ag-mode", default="auto", choices=["auto", "sm", "ce", "push"],
                    help="fused all-gather: SM stores from the quant kernel, copy-engine copies, or by block size")
    ap.add_argument("--rs-dtype", default="bf16", choices=["bf16", "fp8"],
                    help="reduce-scatter payload: bf16 partials, or 1x128 e4m3 codes + scales (the b3 variant)")
    ap.add_argument("--placement", default="auto", choices=["auto", "balanced", "contiguous"],
                    help="expert placement under expert parallelism: the reference's contiguous ranges, experts "
                         "balanced by routed pairs, or auto: balanced from 4 ranks up, contiguous below (measured on "
                         "the DeepSeek-V3 shape: balancing cuts the most-loaded rank's compute at 4 and 8 ranks, "
                         "and costs time at 2)")
    ap.add_argument("--sparse", action="store_true",
                    help="expert parallel: send tokens / partials only to / from the ranks holding their experts")
    ap.add_argument("--chunks", type=int, default=4, help="down-GEMM column chunks of the copy-engine push")
    ap.add_argument("--ce-streams", type=int, default=2, help="side streams carrying the copy-engine push")
    ap.add_argument("--e2e-chunk-mb", type=float, default=1.0,
                    help="host<->device copies of the e2e pipeline in pieces of this many MiB (0: whole tensors)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the post-run check against the fp32 golden")
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
        if args.rs_dtype == "fp8" and args.rs_mode not in ("sm", "auto"):
            raise SystemExit("--rs-dtype fp8 needs --rs-mode sm")
        exchange = P2PExchange(ctx.group, chunks=args.chunks,
                               rs_mode="fp8" if args.rs_dtype == "fp8" else args.rs_mode, ce_streams=args.ce_streams,
                               ag_mode=args.ag_mode, sparse=args.sparse and cfg.parallel == "EP")
    elif world > 1:
        from td_benchmark_b200.layer import NcclExchange
        exchange = NcclExchange(ctx.group, rs_dtype=args.rs_dtype)
    if args.placement == "auto":
        args.placement = "balanced" if world >= 4 else "contiguous"
    layer, level = build_layer(spec, cfg, ctx, bundle, exchange=exchange, placement=args.placement)
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

    # ---- exposed communication and hidden fraction (fused exchange, N > 1)
    comm = exchange_split(layer, bundle, x, ids, wts, args, flush, barrier, world, dev, ms)
    if comm is not None:
        comm["stages_us_max_over_ranks"] = {k: round(v, 1) for k, v in stages.items()}
        barrier()
        layer.forward(x, ids, wts)   # one regular step so every rank's buffers are in step again
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
    chunk = int(args.e2e_chunk_mb * (1 << 20))
    pipe = HostPipeline(layer, chunk_bytes=chunk)
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

    # diagnosis of the pipelined run (not part of the timed number): the same steps traced
    # per stage, and the host<->device copies of a step alone, all ranks copying at once
    tpipe = HostPipeline(layer, trace=True, chunk_bytes=chunk)
    for i in range(args.steps):
        tpipe.submit(x_h, ids_h, wts_h, outs_h[i % 2])
    tpipe.drain()
    spans = tpipe.spans()
    torch.cuda.synchronize()
    barrier()
    x_c, ids_c, wts_c = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(wts)

    def copies_alone():
        with torch.cuda.stream(pipe.h2d):
            x_c.copy_(x_h, non_blocking=True)
            ids_c.copy_(ids_h, non_blocking=True)
            wts_c.copy_(wts_h, non_blocking=True)
        with torch.cuda.stream(pipe.d2h):
            out_h.copy_(layer.out_local, non_blocking=True)
        cur.wait_stream(pipe.h2d)
        cur.wait_stream(pipe.d2h)

    copy_ms = _mean_max_over_ranks(_timed(copies_alone, args.steps, args.warmup, flush, barrier), world, dev)

    x_d, ids_d, wts_d = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(wts)

    def e2e_step():
        x_d.copy_(x_h, non_blocking=True)
        ids_d.copy_(ids_h, non_blocking=True)
        wts_d.copy_(wts_h, non_blocking=True)
        out = layer.forward(x_d, ids_d, wts_d)
        out_h.copy_(out, non_blocking=True)

    e_serial_ms = _mean_max_over_ranks(_timed(e2e_step, args.steps, args.warmup, flush, barrier), world, dev)
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * 4 + wts_h.numel() * 4
    d2h = out_h.numel() * out_h.element_size()

    # ---- roofline: the dominant kernel (GEMM1) and the layer
    peaks = _peaks()
    fp8_peak = peaks.get("fp8_tflops")
    peak_src = "measured cuBLASLt FP8 8192^3 (profiles/peaks.json)"
    if not fp8_peak:
        fp8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
        peak_src = "2 x measured bf16 (MEASURED_PEAKS.json); no FP8 measurement"
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    nvl_peak = peaks.get("nvlink_gbs")
    nvl_src = peaks.get("nvlink_how", "profiles/peaks.json")
    if not nvl_peak:
        nvl_peak, nvl_src = 770.0, "peer copy per direction measured on this pool (profiling recipe figure)"
    g1_ms = sum(g1) / len(g1)
    f1 = gemm1_flops(ids, layer.expert_map, layer.w.inter, layer.H)
    achieved = f1 / (g1_ms * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get(f"gemm1/{args.workload}/{world}")
    s = cfg.shape
    inter_alg = s.intermediate // world if spec.parallel == "TP" else s.intermediate
    sh_alg = s.shared_intermediate // world if spec.parallel == "TP" else s.shared_intermediate
    work = rank_work(layer, ids, inter_alg, sh_alg, rs_fp8=args.rs_dtype == "fp8")
    t_fp8 = work["flops"] / (fp8_peak * 1e12)
    t_nvl = work["nvlink_bytes"] / (nvl_peak * 1e9)
    t_hbm = work["weight_bytes"] / (hbm_peak * 1e9)
    terms = torch.tensor([t_fp8, t_nvl, t_hbm, work["flops"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(terms, op=dist.ReduceOp.MAX)   # the most-loaded rank sets the layer time
    t_fp8, t_nvl, t_hbm, fl_max = terms.tolist()
    bound = max(t_fp8, t_nvl)
    layer_roof = {"t_fp8_us": t_fp8 * 1e6, "t_nvlink_us": t_nvl * 1e6, "t_hbm_weights_us": t_hbm * 1e6,
                  "bound_us": bound * 1e6, "bound_term": "fp8" if t_fp8 >= t_nvl else "nvlink",
                  "frac": bound / (ms * 1e-3), "frac_incl_hbm": max(bound, t_hbm) / (ms * 1e-3),
                  "flops_most_loaded_rank": fl_max, "nvlink_bytes_per_rank": work["nvlink_bytes"],
                  "weight_bytes_per_rank": work["weight_bytes"], "fp8_peak_tflops": fp8_peak,
                  "nvlink_peak_gbs": nvl_peak, "nvlink_peak_source": nvl_src, "hbm_peak_gbs": hbm_peak,
                  "how": "per rank: FP8 FLOPs of routed (unpadded) pairs + shared expert / FP8 peak; all-gather "
                         "received + reduce-scatter sent bytes / NVLink per-direction bandwidth; expert weight "
                         "bytes / HBM; max over ranks; bound = max(fp8, nvlink) (BASELINE definition); frac = "
                         "bound / measured layer time"}

    # ---- parity of the benchmarked layer on every rank
    parity = None if args.no_parity else check_parity(layer, bundle, x, ids, wts, world, rank, dev, spec.parallel,
                                                      args.rs_dtype == "fp8")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gold = CpuGolden(bundle)
        cpu = gold.describe(1, gold.run())

    if rank == 0:
        line = {
            "metric": "moe_layer_tokens_per_s", "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3,
            "ms_per_step_min": min(per_step), "ms_per_step_median": statistics.median(per_step),
            "host_enqueue_us_per_step": host_s / args.steps * 1e6,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8-e4m3 (fp32 accum)",
            "data": "synthetic (seeded, BASELINE value distributions)",
            "config": {"workload": label, "tokens": T, "hidden": s.K, "intermediate": s.intermediate,
                       "experts": s.E, "top_k": s.top_k, "shared_experts": s.shared_experts,
                       "parallelism": f"{spec.parallel.lower()}{world}", "scheme": code, "shard_level": level,
                       "routing": cfg.routing.imbalance_kind,
                       "rs_payload": args.rs_dtype if world > 1 else None,
                       "placement": (args.placement if (spec.parallel == "EP" and world > 1) else None),
                       "exchange": (f"p2p ag={layer.exchange.ag_mode} rs={layer.exchange.rs_mode} "
                                    f"sparse={int(layer.exchange.sparse)} "
                                    f"chunks={len(layer.exchange.chunk_cols)}"
                                    if getattr(layer.exchange, "name", "") == "p2p" else
                                    getattr(layer.exchange, "name", "none")),
                       "l2": "weights > L2 and 256 MB L2 flush between timed steps"},
            "e2e": {"value": T / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
                    "how": "HostPipeline: pinned-host inputs in and result out every step, double-buffered so the "
                           "copies of steps i+1 / i-1 overlap step i; whole run timed with CUDA events, max over ranks",
                    "serial_ms_per_step": e_serial_ms,
                    "diag": {"pipeline_rank0": {k: round(v, 4) if isinstance(v, float) else v for k, v in spans.items()},
                             "copies_alone_ms_per_step": copy_ms,
                             "copies_alone_gbs": (h2d + d2h) / (copy_ms * 1e-3) / 1e9,
                             "how": "traced pipelined steps (rank 0; forward_gap = forward waiting for its inputs); "
                                    "copies alone = one step's h2d and d2h copies on their two streams, no forward, "
                                    "every rank at once, max over ranks"}},
            "gpu_launches": layer.kernel_launches() * args.steps,
            "roofline": {"bound": "tensor", "kernel": "gemm1 (gate/up, tcgen05 kind::f8f6f4)",
                         "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s", "frac": achieved / fp8_peak,
                         "peak_source": peak_src, "traffic": traffic, "gemm1_ms": g1_ms,
                         "gemm1_flops_per_launch": f1, "layer": layer_roof},
            "parity": parity,
            "clocks": clocks,
            "stages_us": {"median_per_step_max_over_ranks": {k: round(v, 1) for k, v in stages.items()},
                          "how": "CUDA events the layer records between its kernels in every timed step; each "
                                 "stage is keyed by the event that closes it"},
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
