"""Layer shapes and run configs.

``ShapeCfg`` / ``RoutingCfg`` keep the field names and helpers of the reference's
``moe_bench/config.py:48-108`` (M tokens, K hidden, E experts, top_k, n_gateup =
2*I, n_down = I, shared expert), so a scheme built here reads a reference
``RunCfg`` unchanged.  ``PRESETS`` are the BASELINE workloads:

* ``tiny``    T=64,   H=256,  I=512,   E=8,   top-2 (CPU-checkable)
* ``mixtral`` T=4096, H=4096, I=14336, E=8,   top-2, TP
* ``dsv3``    T=8192, H=7168, I=2048,  E=256, top-8, EP, Zipf-1.2 routing, 1 shared expert (I=2048)
* ``qwen3``   T=256,  H=2048, I=768,   E=128, top-8, TP (decode; T in {32, 128, 256})
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace


class ConfigError(ValueError):
    """``field=value violates constraint`` (same wording as ``moe_bench/config.py:355-357``)."""


def _require(name: str, value, ok: bool, constraint: str) -> None:
    if not ok:
        raise ConfigError(f"{name}={value!r} violates constraint: {constraint}")


@dataclass(frozen=True)
class ShapeCfg:
    M: int
    K: int
    E: int
    top_k: int
    n_gateup: int
    n_down: int
    shared_experts: int = 0
    shared_intermediate: int | None = None

    def __post_init__(self) -> None:
        shared = self.n_down if self.shared_intermediate is None else self.shared_intermediate
        object.__setattr__(self, "shared_intermediate", shared)
        _require("shape.M", self.M, self.M > 0, "> 0")
        _require("shape.K", self.K, self.K > 0 and self.K % 128 == 0, "> 0 and a multiple of 128")
        _require("shape.E", self.E, self.E > 0, "> 0")
        _require("shape.top_k", self.top_k, 0 < self.top_k <= self.E, "0 < top_k <= E")
        _require("shape.n_gateup", self.n_gateup, self.n_gateup > 0 and self.n_gateup % 2 == 0, "> 0 and even")
        _require("shape.n_down", self.n_down, self.n_down == self.n_gateup // 2, "must equal n_gateup // 2")
        _require("shape.shared_experts", self.shared_experts, self.shared_experts in (0, 1), "must be 0 or 1")

    @property
    def intermediate(self) -> int:
        return self.n_down

    def intermediate_per_tp(self, world_size: int) -> int:
        _require("shape.n_down", self.n_down, self.n_down % world_size == 0, f"divisible by world_size={world_size}")
        return self.n_down // world_size

    def local_E(self, world_size: int) -> int:
        _require("shape.E", self.E, self.E % world_size == 0, f"divisible by world_size={world_size}")
        return self.E // world_size

    def M_aligned(self, world_size: int) -> int:
        return (self.M + world_size - 1) // world_size * world_size


@dataclass(frozen=True)
class RoutingCfg:
    gate_seed: int = 42
    imbalance_kind: str = "none"   # none | zipf
    zipf_s: float = 1.2
    strength: float = 1.0

    def __post_init__(self) -> None:
        _require("routing.imbalance_kind", self.imbalance_kind, self.imbalance_kind in {"none", "zipf"}, "none|zipf")
        _require("routing.zipf_s", self.zipf_s, self.zipf_s > 0, "> 0")


@dataclass(frozen=True)
class RunCfg:
    name: str
    shape: ShapeCfg
    parallel: str = "TP"          # TP | EP
    routing: RoutingCfg = field(default_factory=RoutingCfg)
    seed: int = 42
    weight_std: float = 0.02

    def __post_init__(self) -> None:
        _require("parallel", self.parallel, self.parallel in {"TP", "EP"}, "TP|EP")


PRESETS: dict[str, RunCfg] = {
    "tiny": RunCfg("tiny", ShapeCfg(M=64, K=256, E=8, top_k=2, n_gateup=1024, n_down=512)),
    "mixtral": RunCfg("mixtral", ShapeCfg(M=4096, K=4096, E=8, top_k=2, n_gateup=28672, n_down=14336)),
    "dsv3": RunCfg("dsv3", ShapeCfg(M=8192, K=7168, E=256, top_k=8, n_gateup=4096, n_down=2048, shared_experts=1,
                                    shared_intermediate=2048),
                   parallel="EP", routing=RoutingCfg(imbalance_kind="zipf", zipf_s=1.2)),
    "qwen3": RunCfg("qwen3", ShapeCfg(M=256, K=2048, E=128, top_k=8, n_gateup=1536, n_down=768)),
}


def preset(name: str, **overrides) -> RunCfg:
    """A preset with optional shape/routing overrides, e.g. ``preset('dsv3', M=512, imbalance_kind='none')``."""
    if name not in PRESETS:
        raise ConfigError(f"preset={name!r} violates constraint: one of {sorted(PRESETS)}")
    cfg = PRESETS[name]
    shape_keys = {k: v for k, v in overrides.items() if k in ShapeCfg.__dataclass_fields__}
    routing_keys = {k: v for k, v in overrides.items() if k in RoutingCfg.__dataclass_fields__}
    run_keys = {k: v for k, v in overrides.items() if k in RunCfg.__dataclass_fields__}
    unknown = set(overrides) - set(shape_keys) - set(routing_keys) - set(run_keys)
    if unknown:
        raise ConfigError(f"overrides={sorted(unknown)!r} violates constraint: known shape/routing/run fields")
    return replace(cfg, shape=replace(cfg.shape, **shape_keys), routing=replace(cfg.routing, **routing_keys),
                   **run_keys)
