"""Measure the roofline denominators this package reports against (one JSON object).

    python -m td_benchmark_b200.peaks [--nvlink-only]      # on a box with >= 1 (FP8) / 2 (NVLink) GPUs

* ``fp8_tflops``: dense FP8 e4m3 x e4m3 -> bf16 GEMM, 8192^3, through cuBLASLt
  (``torch._scaled_mm``), best of 10 CUDA-event timings -- the tensor-core ceiling the
  grouped GEMMs are compared with;
* ``nvlink_gbs``: GPU 0 -> GPU 1 peer copy of 256 MiB by the copy engines (one direction,
  best of 10), and ``nvlink_bidir_gbs`` with both directions at once (per direction) --
  the link term of the layer roofline (bytes that must cross NVLink / this rate);
* ``nvlink_sizes``: the one-direction rate at 1, 4, 16, 64 and 256 MiB.

Read-only with respect to the GPUs' settings: nothing here touches clocks or power.
"""
from __future__ import annotations

import argparse
import json


def _best_ms(fn, reps: int = 10) -> float:
    import torch

    fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return best


def fp8_gemm_tflops(n: int = 8192) -> float:
    import torch

    dev = torch.device("cuda", 0)
    a = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn)
    b = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    ms = _best_ms(lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
    return 2.0 * n ** 3 / (ms * 1e-3) / 1e12


def nvlink_gbs() -> dict:
    import torch

    if torch.cuda.device_count() < 2:
        return {"nvlink_gbs": None, "nvlink_note": "fewer than 2 GPUs visible"}
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    out = {"nvlink_sizes": {}}
    for mib in (1, 4, 16, 64, 256):
        n = mib << 20
        src = torch.empty(n, dtype=torch.uint8, device=d0).fill_(1)
        dst = torch.empty(n, dtype=torch.uint8, device=d1)
        with torch.cuda.device(d0):
            ms = _best_ms(lambda: dst.copy_(src, non_blocking=True))
        out["nvlink_sizes"][f"{mib}MiB"] = n / (ms * 1e-3) / 1e9
    out["nvlink_gbs"] = out["nvlink_sizes"]["256MiB"]
    # both directions at once: one copy per direction on its own stream
    n = 256 << 20
    a0 = torch.empty(n, dtype=torch.uint8, device=d0).fill_(1)
    b1 = torch.empty(n, dtype=torch.uint8, device=d1)
    a1 = torch.empty(n, dtype=torch.uint8, device=d1).fill_(2)
    b0 = torch.empty(n, dtype=torch.uint8, device=d0)
    s0 = torch.cuda.Stream(d0)
    s1 = torch.cuda.Stream(d1)
    best = float("inf")
    for _ in range(10):
        torch.cuda.synchronize(d0)
        torch.cuda.synchronize(d1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s0):
            e0.record(s0)
            b1.copy_(a0, non_blocking=True)
        with torch.cuda.stream(s1):
            b0.copy_(a1, non_blocking=True)
            done = torch.cuda.Event()
            done.record(s1)
        s0.wait_event(done)
        with torch.cuda.stream(s0):
            e1.record(s0)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    out["nvlink_bidir_gbs"] = n / (best * 1e-3) / 1e9
    out["nvlink_how"] = ("copy-engine peer copy GPU0->GPU1 (torch copy_ across devices), best of 10 CUDA-event "
                         "timings, 256 MiB; bidir = both directions at once, rate per direction")
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--nvlink-only", action="store_true")
    args = ap.parse_args(argv)
    res = {}
    if not args.nvlink_only:
        res["fp8_tflops"] = fp8_gemm_tflops()
        res["fp8_how"] = "torch._scaled_mm (cuBLASLt) e4m3 x e4m3 -> bf16, 8192^3, best of 10 CUDA-event timings"
    res.update(nvlink_gbs())
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
