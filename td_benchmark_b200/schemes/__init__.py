"""Scheme registry — the reference's ``moe_bench/schemes/__init__.py`` contract.

``REGISTRY[code] = (SchemeSpec, build)`` and ``build_scheme(cfg, ctx, data,
scheme_cfg)`` raising ``SchemeConfigError`` for unknown codes (``__init__.py:18-37``).
``register_into_reference()`` adds these codes to a reference ``moe_bench`` install
(its ``REGISTRY`` and ``config._SCHEME_CODES``) so its worker can time them.
"""
from __future__ import annotations

from typing import Any

from . import b200
from .base import BuilderFn, SchemeConfigError, SchemeSpec

REGISTRY: dict[str, tuple[SchemeSpec, BuilderFn]] = {
    b200.SPEC_D1.code: (b200.SPEC_D1, b200.build_d1),
    b200.SPEC_D2.code: (b200.SPEC_D2, b200.build_d2),
    b200.SPEC_D3.code: (b200.SPEC_D3, b200.build_d3),
    b200.SPEC_D4.code: (b200.SPEC_D4, b200.build_d4),
}


def build_scheme(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any):
    try:
        _spec, builder = REGISTRY[scheme_cfg.code]
    except KeyError as exc:
        raise SchemeConfigError(f"scheme {scheme_cfg.code!r} is not registered") from exc
    return builder(cfg, ctx, data, scheme_cfg)


def register_into_reference() -> list[str]:
    """Register the B200 schemes in an importable reference ``moe_bench`` package.

    Each scheme enters the reference ``REGISTRY`` with its spec re-expressed in the
    reference's own ``SchemeSpec`` / ``TunableSpec`` types and a builder whose tunable
    errors are raised as the reference's ``SchemeConfigError``, so the reference worker
    and CLI see nothing foreign (``moe_bench/schemes/__init__.py:18-37``, ``base.py:7-45``);
    the codes are added to ``config._SCHEME_CODES`` so its ``SchemeCfg`` accepts them
    (``moe_bench/config.py:45, 113-114``).  Returns the codes added."""
    import moe_bench.config as ref_config
    import moe_bench.schemes as ref_schemes
    import moe_bench.schemes.base as ref_base

    def as_reference(spec: SchemeSpec):
        schema = {k: ref_base.TunableSpec(t.typ, t.default, t.description) for k, t in spec.tunables_schema.items()}
        return ref_base.SchemeSpec(code=spec.code, name=spec.name, family=spec.family, parallel=spec.parallel,
                                   comm=spec.comm, weight_dtype=spec.weight_dtype, act_quant=spec.act_quant,
                                   requires_nvshmem=spec.requires_nvshmem, tunables_schema=schema)

    def adapt(builder: BuilderFn) -> BuilderFn:
        def build(cfg: Any, ctx: Any, data: Any, scheme_cfg: Any):
            try:
                return builder(cfg, ctx, data, scheme_cfg)
            except SchemeConfigError as exc:
                raise ref_base.SchemeConfigError(str(exc)) from exc
        return build

    added = []
    for code, (spec, builder) in REGISTRY.items():
        ref_schemes.REGISTRY[code] = (as_reference(spec), adapt(builder))
        ref_config._SCHEME_CODES.add(code)
        added.append(code)
    return added


__all__ = ["REGISTRY", "build_scheme", "SchemeConfigError", "SchemeSpec", "register_into_reference"]
