"""Multi-GPU parity check, run under torchrun (one rank per GPU, NCCL).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 tests/dist_gpu_check.py --scheme d3 --preset mixtral --tokens 512

Every rank builds the same seeded data, runs the scheme twice (buffers reused), and
compares its [T/P, H] output slice with the fp32 torch golden of the full layer under
the reference worker's gates plus the calibrated max-abs bound.  Exit status 0 only
if every rank passes; rank 0 prints one JSON line.
"""
import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--scheme", default="d3")
    ap.add_argument("--preset", default="mixtral")
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--zipf", action="store_true")
    ap.add_argument("--ag-mode", default=None, help="d3/d4 tunable ag_mode")
    ap.add_argument("--rs-mode", default=None, help="d3/d4 tunable rs_mode")
    ap.add_argument("--rs-chunks", type=int, default=None, help="d3/d4 tunable rs_chunks")
    ap.add_argument("--rs-dtype", default=None, help="tunable rs_dtype (bf16 | fp8)")
    ap.add_argument("--sparse", action="store_true", help="d4 tunable sparse; also checks it equals the dense exchange")
    ap.add_argument("--placement", default=None, help="d2/d4 tunable placement (contiguous | balanced)")
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    from oracle import golden as ogolden
    from tests import torch_ref
    from td_benchmark_b200 import configs, data
    from td_benchmark_b200.context import init_context
    from td_benchmark_b200.schemes import build_scheme
    from td_benchmark_b200.schemes.base import SchemeCfg

    ctx = init_context(backend="nccl", timeout_s=120.0)
    over = {"M": args.tokens}
    if args.preset == "dsv3" and not args.zipf:
        over["imbalance_kind"] = "none"
    cfg = configs.preset(args.preset, **over)
    bundle = data.build_bundle(cfg, rank=ctx.rank, world_size=ctx.world_size, device=ctx.device)
    tun = {"check_status": True}
    for key, val in (("ag_mode", args.ag_mode), ("rs_mode", args.rs_mode), ("rs_chunks", args.rs_chunks),
                     ("rs_dtype", args.rs_dtype), ("placement", args.placement)):
        if val is not None:
            tun[key] = val
    dense_out = None
    if args.sparse:
        dense = build_scheme(cfg, ctx, bundle, SchemeCfg(args.scheme, dict(tun, ag_mode="sm")))
        dense_out = dense.run().clone()
        torch.cuda.synchronize()
        dense.close()
        tun["sparse"] = True
    inst = build_scheme(cfg, ctx, bundle, SchemeCfg(args.scheme, tun))
    out1 = inst.run().clone()
    out2 = inst.run()
    torch.cuda.synchronize()
    same = bool(torch.equal(out1, out2))
    if dense_out is not None:
        same = same and bool(torch.equal(out2, dense_out))   # sparse sends change no bit of the result
    ck = bundle.ckpt
    sw = None
    if ck.shared_w1 is not None:
        sw = (ck.shared_w1.fp8, ck.shared_w1.scale, ck.shared_w2.fp8, ck.shared_w2.scale)
    g, calib = torch_ref.act_quant_error(bundle.hidden_full, bundle.routing.topk_ids_full,
                                         bundle.routing.topk_weights_full, ck.w1.fp8, ck.w1.scale, ck.w2.fp8,
                                         ck.w2.scale, sw)
    tl = out2.shape[0]
    ref = g[ctx.rank * tl:(ctx.rank + 1) * tl]
    rs_calib = 0.0
    if args.rs_dtype == "fp8":
        # the FP8 reduce-scatter payload adds the quantisation error of every rank's partial
        from td_benchmark_b200 import verify
        r0 = ctx.rank * tl
        owner = None
        if args.placement == "balanced" and cfg.parallel == "EP":
            from td_benchmark_b200.weights import balanced_placement, expert_owner
            owner = expert_owner(balanced_placement(bundle.routing.topk_ids_full, cfg.shape.E,
                                                    ctx.world_size)).tolist()
        parts = verify.rank_partials(bundle.hidden_full[r0:r0 + tl], bundle.routing.topk_ids_full[r0:r0 + tl],
                                     bundle.routing.topk_weights_full[r0:r0 + tl], ck, ctx.world_size, cfg.parallel,
                                     owner)
        rs_calib = verify.rs_fp8_error(parts)
        calib = calib + rs_calib
    rep = ogolden.compare_outputs(out2.float().cpu().numpy(), ref.cpu().numpy(), **ogolden.GATES)
    ok = rep["pass"] and rep["max_abs"] <= 1.5 * calib and same
    inst.close()
    flag = torch.tensor([1.0 if ok else 0.0], device=ctx.device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if ctx.rank == 0:
        print(json.dumps({"scheme": args.scheme, "tunables": tun, "preset": args.preset, "tokens": args.tokens,
                          "world": ctx.world_size,
                          "pass": bool(flag.item() > 0), "rank0": {k: rep[k] for k in ("cos_sim", "rel_p99", "max_abs",
                                                                                         "scale")},
                          "calib_max_abs": calib, "rs_fp8_calib": rs_calib, "repeatable": same}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if flag.item() > 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
