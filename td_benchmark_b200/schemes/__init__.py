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
    """Register the B200 schemes in an importable reference ``moe_bench`` package."""
    import moe_bench.config as ref_config
    import moe_bench.schemes as ref_schemes

    added = []
    for code, (spec, builder) in REGISTRY.items():
        ref_schemes.REGISTRY[code] = (spec, builder)
        ref_config._SCHEME_CODES.add(code)
        added.append(code)
    return added


__all__ = ["REGISTRY", "build_scheme", "SchemeConfigError", "SchemeSpec", "register_into_reference"]
