"""Scaling sweep on the DeepSeek-V3 shape, one JSON record per point.

    python -m td_benchmark_b200.sweep [--tokens 512,2048,8192,32768] [--routing uniform,zipf]
                                      [--variants nccl,fused,sparse,fp8rs,ce1,ce2,ce4,ce8] [--steps 10]
    torchrun --nproc-per-node N -m td_benchmark_b200.sweep ...        # N ranks, EP=N

The reference sweeps T x overlap chunk count x world size x routing, fused against its
NCCL scheme (``moe_bench/config.py:250-262`` expands the grid; ``cli.py`` runs one
torchrun per point).  Here one launch covers every (T, routing, variant) point at the
launched world size; the data bundle of a (T, routing) pair is built once and shared by
its variants.  Variants (expert parallel, scheme d2 / d4):

* ``nccl``   NCCL all-gather + NCCL bf16 reduce-scatter (the unfused comparison);
* ``fused``  peer-memory exchange with its default transports (reduce-scatter from the down GEMM);
* ``sm``     the same with the reduce-scatter as SM stores from a combine kernel after the down GEMM;
* ``sparse`` peer-memory exchange sending tokens / partials only to / from the ranks that
             hold their experts;
* ``fp8rs``  peer-memory exchange with the FP8 reduce-scatter payload;
* ``balanced`` / ``balanced-fp8rs``: ``fused`` / ``fp8rs`` with E/P experts per rank placed by
             routed pairs instead of contiguous ranges (the other variants use contiguous);
* ``ceC``    the chunked variant: the down GEMM in C column chunks, each chunk's partials
             pushed by copy engines while the next computes -- the overlap-chunk axis of the
             reference's b2/b3 (``n_chunks_down``).

One GPU runs the single-GPU layer (the variants coincide).  Timing: CUDA events per
step, per-step maximum over ranks, mean over ``--steps`` after ``--warmup`` steps, a
256 MB L2 flush between steps.  Records go to stdout (rank 0) and, with ``--out``, to a
JSONL file.
"""
from __future__ import annotations

import argparse
import json
import sys
import time


def _time_forward(layer, x, ids, wts, steps: int, warmup: int, flush, world: int, dev) -> float:
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(warmup):
        flush.zero_()
        layer.forward(x, ids, wts)
    torch.cuda.synchronize()
    layer.check()
    barrier()
    s = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        s[i].record()
        layer.forward(x, ids, wts)
        e[i].record()
    torch.cuda.synchronize()
    layer.check()
    t = torch.tensor([a.elapsed_time(b) for a, b in zip(s, e)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    barrier()
    return float(t.mean().item())


def _exchange(variant: str, ctx):
    from .layer import NcclExchange, P2PExchange

    if variant == "nccl":
        return NcclExchange(ctx.group)
    if variant == "fused":
        return P2PExchange(ctx.group)
    if variant == "sm":
        return P2PExchange(ctx.group, rs_mode="sm")
    if variant == "sparse":
        return P2PExchange(ctx.group, sparse=True)
    if variant in ("fp8rs", "balanced-fp8rs"):
        return P2PExchange(ctx.group, rs_mode="fp8")
    if variant == "balanced":
        return P2PExchange(ctx.group)
    if variant.startswith("ce"):
        return P2PExchange(ctx.group, rs_mode="ce", chunks=int(variant[2:]))
    raise ValueError(f"unknown variant {variant!r}")


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--preset", default="dsv3")
    ap.add_argument("--tokens", default="512,2048,8192,32768")
    ap.add_argument("--routing", default="uniform,zipf")
    ap.add_argument("--variants", default="nccl,fused,sparse,fp8rs,ce1,ce2,ce4,ce8")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out", default=None, help="also append the records to this JSONL file (rank 0)")
    args = ap.parse_args(argv)

    import torch

    from . import configs, data
    from .context import init_context
    from .schemes import REGISTRY
    from .schemes.b200 import build_layer

    ctx = init_context(backend="nccl", timeout_s=300.0)
    world, dev = ctx.world_size, ctx.device
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    variants = [v for v in args.variants.split(",") if v] if world > 1 else ["single-gpu"]
    out = open(args.out, "a") if (args.out and ctx.rank == 0) else None
    for T in [int(v) for v in args.tokens.split(",") if v]:
        for routing in [r for r in args.routing.split(",") if r]:
            kind = "zipf" if routing == "zipf" else "none"
            cfg = configs.preset(args.preset, M=T, imbalance_kind=kind)
            if T % world:
                continue
            t0 = time.time()
            bundle = data.build_bundle(cfg, rank=ctx.rank, world_size=world, device=dev)
            x = bundle.hidden_local.contiguous()
            ids = bundle.routing.topk_ids_full.contiguous()
            wts = bundle.routing.topk_weights_full.contiguous()
            for variant in variants:
                code = ("d2" if variant == "nccl" else "d4") if cfg.parallel == "EP" else \
                       ("d1" if variant == "nccl" else "d3")
                exchange = None if world == 1 else _exchange(variant, ctx)
                placement = "balanced" if variant.startswith("balanced") else "contiguous"
                layer, _ = build_layer(REGISTRY[code][0], cfg, ctx, bundle, exchange=exchange, placement=placement)
                ms = _time_forward(layer, x, ids, wts, args.steps, args.warmup, flush, world, dev)
                rec = {"preset": args.preset, "tokens": T, "routing": routing, "variant": variant, "scheme": code,
                       "placement": placement if cfg.parallel == "EP" else None,
                       "n_gpus": world, "parallelism": f"{cfg.parallel.lower()}{world}", "us_per_layer": ms * 1e3,
                       "tokens_per_s": T / (ms * 1e-3), "steps": args.steps, "warmup": args.warmup,
                       "exchange": getattr(layer.exchange, "name", "none"),
                       "ag_mode": getattr(layer.exchange, "ag_mode", None),
                       "rs_mode": getattr(layer.exchange, "rs_mode", None),
                       "chunks": len(getattr(layer.exchange, "chunk_cols", [None]))}
                layer.close()
                del layer
                torch.cuda.empty_cache()
                if ctx.rank == 0:
                    line = json.dumps(rec)
                    print(line, flush=True)
                    if out:
                        out.write(line + "\n")
                        out.flush()
            del bundle, x, ids, wts
            torch.cuda.empty_cache()
            if ctx.rank == 0:
                print(f"# T={T} routing={routing}: {time.time() - t0:.1f} s", file=sys.stderr, flush=True)
    if out:
        out.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
