"""B200 schemes: FP8 MoE layer on the b2m kernels behind the reference's builder contract.

``build(cfg, ctx, data, scheme_cfg) -> SchemeInstance`` does all set-up — shard
views (``moe_bench/schemes/runtime.py:27-104``), gate/up interleave, buffers,
exchange — so the timed ``run()`` is only the forward (the reference learned this
the hard way, ``docs/exp/EXP-024-cgroup-perf-rootcause.md:6-9``).  ``run()`` reads
the precomputed full routing (``runtime.py:19-24``) and never the gate weight,
returns bf16 [M/P, K] on ``ctx.device`` ordered on the caller's current stream.

Codes:
  d1  TP, NCCL all-gather (FP8 bytes + scales) -> b2m kernels -> NCCL reduce-scatter (bf16)
  d2  EP, same exchange, local experts only (expert_map), shared expert on local tokens
  d3  TP, fused exchange over NVLink peer memory: the quant kernel stores into every
      rank's gather buffer, the combine kernel stores each partial into its owner's slot
  d4  EP, fused exchange as d3
The NCCL schemes are the unfused comparison for the fused peer-memory schemes.
"""
from __future__ import annotations

from typing import Any

from .base import SchemeConfigError, SchemeInstance, SchemeSpec, TunableSpec, make_lazy_instance, validate_tunables

EXCHANGE = {"d1": "nccl", "d2": "nccl", "d3": "p2p", "d4": "p2p"}

B200_TUNABLES = {
    "check_status": TunableSpec(bool, False, "synchronise after every run() and raise on a device status code"),
    "rs_dtype": TunableSpec(str, "bf16", "reduce-scatter payload: bf16 partials ('bf16') or 1x128-quantised e4m3 "
                                         "codes + fp32 scales dequant-summed by the owner ('fp8', the b3 variant)"),
}
# peer-memory exchange knobs of d3 / d4 (P2PExchange)
P2P_TUNABLES = {
    "ag_mode": TunableSpec(str, "auto", "all-gather by SM stores from the quant kernel ('sm'), copy engines ('ce'), "
                                        "by block size ('auto'), or (TP) straight into the peers' sorted operand "
                                        "under the gate/up GEMM ('push')"),
    "rs_mode": TunableSpec(str, "auto", "reduce-scatter by SM stores from the combine ('sm'), from the down GEMM's "
                                        "epilogue ('gemm'), copy engines ('ce'), or 'auto': 'gemm' when the pair rows are "
                                        "at most twice the partials' bytes (top_k <= 2 TP, <= 2P EP) or with >= "
                                        "2048 local tokens, else 'sm' (also for a tensor-parallel shared expert)"),
    "rs_chunks": TunableSpec(int, 4, "down-GEMM column chunks of the copy-engine reduce-scatter (1..8)"),
}
# expert-parallel schemes (d2, d4)
EP_TUNABLES = {
    "placement": TunableSpec(str, "contiguous", "experts per rank: 'contiguous' (rank r holds [r*E/P, (r+1)*E/P), the "
                                                "reference's layout) or 'balanced' (E/P experts per rank chosen so "
                                                "every rank holds about the same number of routed pairs; same output)"),
}
# expert-parallel peer-memory scheme only
EP_SPARSE = {
    "sparse": TunableSpec(bool, False, "send a token only to the ranks holding one of its experts and its partial only "
                                       "from those ranks (all-gather and reduce-scatter by SM stores; same output as "
                                       "the dense exchange, fewer NVLink bytes)"),
}
_CHOICES = {"ag_mode": ("sm", "ce", "auto", "push"), "rs_mode": ("auto", "sm", "ce", "gemm"), "rs_dtype": ("bf16", "fp8"),
            "placement": ("contiguous", "balanced")}


def _spec(code: str, name: str, parallel: str, comm: str) -> SchemeSpec:
    schema = dict(B200_TUNABLES)
    if parallel == "EP":
        schema.update(EP_TUNABLES)
    if EXCHANGE.get(code) == "p2p":
        schema.update(P2P_TUNABLES)
        if parallel == "EP":
            schema.update(EP_SPARSE)
    return SchemeSpec(code=code, name=name, family="b200", parallel=parallel, comm=comm, weight_dtype="fp8",
                      act_quant="group128", requires_nvshmem=False, tunables_schema=schema)


SPEC_D1 = _spec("d1", "B200-TP-NCCL", "TP", "quantize -> NCCL AG(fp8+scale) -> b2m GEMM1/GEMM2 -> NCCL RS(bf16)")
SPEC_D2 = _spec("d2", "B200-EP-NCCL", "EP", "quantize -> NCCL AG(fp8+scale) -> b2m GEMMs(local experts) -> NCCL RS -> +shared")
SPEC_D3 = _spec("d3", "B200-TP-P2P", "TP", "quantize+push(peer memory) -> b2m GEMM1/GEMM2 -> combine+push -> owner reduce")
SPEC_D4 = _spec("d4", "B200-EP-P2P", "EP", "quantize+push(peer memory) -> b2m GEMMs(local experts) -> combine+push -> owner reduce(+shared)")


def require_data(data: Any) -> Any:
    if data is None:
        raise RuntimeError("Scheme execution requires a DataBundle; build-only tests may pass data=None.")
    return data


def build_layer(spec: SchemeSpec, cfg: Any, ctx: Any, data: Any, exchange: Any = None,
                tunables: dict[str, Any] | None = None, placement: str | None = None):
    """Shard views + prepared weights + MoELayer for this rank.

    ``placement`` (expert parallel; default the ``placement`` tunable, else 'contiguous'):
    'balanced' places E/P experts per rank by the routed pairs of ``data.routing`` (every rank
    computes the same placement from the same routing)."""
    import torch

    from ..layer import ExpertWeights, MoELayer, NcclExchange, P2PExchange
    from ..weights import balanced_placement, ep_views, tp_views

    bundle = require_data(data)
    ckpt = bundle.ckpt
    device = torch.device(ctx.device)
    s = cfg.shape
    T = s.M_aligned(ctx.world_size)
    args = (ckpt.w1.fp8.to(device), ckpt.w1.scale.to(device), ckpt.w2.fp8.to(device), ckpt.w2.scale.to(device),
            ctx.rank, ctx.world_size)
    if placement is None:
        placement = (tunables or {}).get("placement", "contiguous")
    if spec.parallel == "TP":
        views = tp_views(*args)
    elif placement == "balanced" and ctx.world_size > 1:
        views = ep_views(*args, placement=balanced_placement(bundle.routing.topk_ids_full, s.E, ctx.world_size))
    else:
        views = ep_views(*args)
    weights = ExpertWeights.prepare(views["w1"], views["w1_scale"], views["w2"], views["w2_scale"])
    shared = None
    if ckpt.shared_w1 is not None and ckpt.shared_w2 is not None:
        sargs = (ckpt.shared_w1.fp8.to(device), ckpt.shared_w1.scale.to(device), ckpt.shared_w2.fp8.to(device),
                 ckpt.shared_w2.scale.to(device))
        sv = tp_views(*sargs, ctx.rank, ctx.world_size) if spec.parallel == "TP" else tp_views(*sargs, 0, 1)
        shared = ExpertWeights.prepare(sv["w1"], sv["w1_scale"], sv["w2"], sv["w2_scale"])
    rs_dtype = (tunables or {}).get("rs_dtype", "bf16")
    if exchange is None and ctx.world_size > 1:
        if EXCHANGE.get(spec.code) == "p2p":
            t = {k: v.default for k, v in P2P_TUNABLES.items()}
            t.update({k: v for k, v in (tunables or {}).items() if k in P2P_TUNABLES})
            rs_mode = t["rs_mode"]
            if rs_dtype == "fp8":
                if rs_mode not in ("sm", "auto"):
                    raise SchemeConfigError(f"{spec.code}.rs_dtype='fp8' needs rs_mode='sm', got {rs_mode!r}")
                rs_mode = "fp8"
            exchange = P2PExchange(ctx.group, chunks=t["rs_chunks"], rs_mode=rs_mode, ag_mode=t["ag_mode"],
                                   sparse=bool((tunables or {}).get("sparse", False)))
        else:
            exchange = NcclExchange(ctx.group, rs_dtype=rs_dtype)
    expert_map = views.get("expert_map")
    layer = MoELayer(weights, T, s.top_k, s.E, expert_map=expert_map, shared=shared, exchange=exchange,
                     device=device, expert_owner=views.get("expert_owner"))
    return layer, views["shard_level"]


def build_instance(spec: SchemeSpec, cfg: Any, ctx: Any, data: Any, scheme_cfg: Any) -> SchemeInstance:
    import torch

    tunables = validate_tunables(spec, scheme_cfg.tunables)
    for name, allowed in _CHOICES.items():
        if name in tunables and tunables[name] not in allowed:
            raise SchemeConfigError(f"{spec.code}.{name}={tunables[name]!r} violates schema: expected one of {allowed}")
    if tunables.get("rs_dtype") == "fp8" and tunables.get("rs_mode", "auto") not in ("sm", "auto"):
        raise SchemeConfigError(f"{spec.code}.rs_dtype='fp8' violates schema: needs rs_mode='sm', got "
                                f"{tunables['rs_mode']!r}")
    if "rs_chunks" in tunables and not 1 <= tunables["rs_chunks"] <= 8:
        raise SchemeConfigError(f"{spec.code}.rs_chunks={tunables['rs_chunks']} violates schema: expected 1..8")
    bundle = require_data(data)
    layer, level = build_layer(spec, cfg, ctx, bundle, tunables=tunables)
    device = layer.device
    topk_ids = bundle.routing.topk_ids_full.to(device=device, dtype=torch.int32).contiguous()
    topk_weights = bundle.routing.topk_weights_full.to(device=device, dtype=torch.float32).contiguous()
    x = bundle.hidden_local.to(device=device, dtype=torch.bfloat16).contiguous()
    check = tunables["check_status"]

    def run() -> Any:
        out = layer.forward(x, topk_ids, topk_weights)
        if check:
            layer.check()
        return out

    def close() -> None:
        try:
            layer.check()
        finally:
            layer.close()

    diag = {"shard_level": level, "tokens": layer.T, "rows_cap": layer.route.rows_cap,
            "experts_local": layer.w.num_experts, "inter_local": layer.w.inter}
    return make_lazy_instance(spec, tunables, run, diagnostics=diag, close_impl=close)


def build_d1(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any) -> SchemeInstance:
    return build_instance(SPEC_D1, cfg, ctx, data, scheme_cfg)


def build_d2(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any) -> SchemeInstance:
    return build_instance(SPEC_D2, cfg, ctx, data, scheme_cfg)


def build_d3(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any) -> SchemeInstance:
    return build_instance(SPEC_D3, cfg, ctx, data, scheme_cfg)


def build_d4(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any) -> SchemeInstance:
    return build_instance(SPEC_D4, cfg, ctx, data, scheme_cfg)
