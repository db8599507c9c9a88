"""World-size-2 gloo check of the host-side sharding logic (run under torchrun on CPU).

Each rank takes its TP shard (``weights.tp_views``) or EP shard (``weights.ep_views``)
of the tiny BASELINE layer, computes its partial output on the gathered tokens with
the numpy oracle, and the partials are reduce-scattered with the same collective the
NCCL scheme uses.  Every rank's slice must equal the full-layer oracle output (fp32
reassociation only), and the EP expert map must mark exactly the local experts.
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main() -> int:
    import torch
    import torch.distributed as dist

    from oracle import golden as ogolden
    from oracle import quant as oquant
    from td_benchmark_b200 import configs, data
    from td_benchmark_b200.context import init_context
    from td_benchmark_b200.weights import ep_views, tp_views

    ctx = init_context(backend="gloo", timeout_s=60.0)
    P, r = ctx.world_size, ctx.rank
    cfg = configs.preset("tiny", M=64)
    b = data.build_bundle(cfg, rank=r, world_size=P)
    ck = b.ckpt
    deq = lambda q, s: oquant.dequant_block128(q.view(torch.uint8).numpy(), s.numpy())  # noqa: E731
    h = b.hidden_full.float().numpy()
    ids, wts = b.routing.topk_ids_full.numpy(), b.routing.topk_weights_full.numpy()
    full = ogolden.golden_moe(h, ids, wts, deq(ck.w1.fp8, ck.w1.scale), deq(ck.w2.fp8, ck.w2.scale))
    T, H = full.shape
    ok = True
    for kind in ("TP", "EP"):
        fn = tp_views if kind == "TP" else ep_views
        v = fn(ck.w1.fp8, ck.w1.scale, ck.w2.fp8, ck.w2.scale, r, P)
        w1, w2 = deq(v["w1"], v["w1_scale"]), deq(v["w2"], v["w2_scale"])
        if kind == "TP":
            part = ogolden.golden_moe(h, ids, wts, w1, w2)
        else:
            emap = v["expert_map"].numpy()
            assert set(np.nonzero(emap >= 0)[0]) == set(range(r * cfg.shape.E // P, (r + 1) * cfg.shape.E // P))
            local_ids = np.where(emap[ids] >= 0, emap[ids], -1)
            part = ogolden.golden_moe(h, local_ids, wts, w1, w2)
        out = torch.empty((T // P, H), dtype=torch.float32)
        dist.reduce_scatter_tensor(out, torch.from_numpy(part), group=None)
        ref = full[r * T // P:(r + 1) * T // P]
        err = float(np.abs(out.numpy() - ref).max() / max(np.abs(ref).max(), 1e-12))
        ok = ok and err < 2e-3
        print(f"rank {r} {kind}: max rel err {err:.2e}", flush=True)
    flag = torch.tensor([1.0 if ok else 0.0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    return 0 if flag.item() > 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
