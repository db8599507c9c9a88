"""Scheme plugin interface — the reference's ``moe_bench/schemes/base.py`` contract.

Names, fields and error behaviour match the reference (``base.py:7-97``) so a
scheme defined here registers in ``moe_bench.schemes.REGISTRY`` unchanged and a
reference ``SchemeSpec`` reads the same way here:

* ``SchemeSpec(code, name, family, parallel, comm, weight_dtype, act_quant,
  requires_nvshmem, tunables_schema)`` (``base.py:18-28``);
* ``SchemeInstance(run, run_staged, diagnostics, close)`` (``base.py:37-42``);
* ``validate_tunables`` raises ``SchemeConfigError`` with ``... violates schema``
  text for unknown keys or wrong types, booleans not accepted as ints (``base.py:48-62``);
* ``make_lazy_instance`` fills the diagnostics dict (``base.py:65-93``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable


class SchemeConfigError(ValueError):
    """Raised when scheme tunables do not match the scheme schema."""


@dataclass(frozen=True)
class TunableSpec:
    typ: type
    default: Any
    description: str


@dataclass(frozen=True)
class SchemeSpec:
    code: str
    name: str
    family: str
    parallel: str
    comm: str
    weight_dtype: str
    act_quant: str
    requires_nvshmem: bool
    tunables_schema: dict[str, TunableSpec]


@dataclass(frozen=True)
class SchemeCfg:
    code: str
    tunables: dict[str, Any] = field(default_factory=dict)


@dataclass
class StageResult:
    output: Any
    stage_ms: dict[str, float]


@dataclass
class SchemeInstance:
    run: Callable[[], Any]
    run_staged: Callable[[], StageResult] | None
    diagnostics: dict[str, Any]
    close: Callable[[], None]


BuilderFn = Callable[[Any, Any, Any, Any], SchemeInstance]


def validate_tunables(spec: SchemeSpec, provided: dict[str, Any]) -> dict[str, Any]:
    unknown = sorted(set(provided) - set(spec.tunables_schema))
    if unknown:
        raise SchemeConfigError(f"{spec.code} tunables {unknown} violate schema: allowed keys are "
                                f"{sorted(spec.tunables_schema)}")
    values = {name: item.default for name, item in spec.tunables_schema.items()}
    values.update(provided)
    for name, value in values.items():
        expected = spec.tunables_schema[name].typ
        ok = isinstance(value, bool) if expected is bool else (isinstance(value, expected) and
                                                                not isinstance(value, bool))
        if not ok:
            raise SchemeConfigError(f"{spec.code}.{name}={value!r} violates schema: expected {expected.__name__}")
    return values


def make_lazy_instance(spec: SchemeSpec, tunables: dict[str, Any], run_impl: Callable[[], Any],
                       diagnostics: dict[str, Any] | None = None,
                       close_impl: Callable[[], None] | None = None,
                       staged_impl: Callable[[], StageResult] | None = None) -> SchemeInstance:
    diag = {
        "scheme": spec.code, "name": spec.name, "family": spec.family, "parallel": spec.parallel,
        "weight_dtype": spec.weight_dtype, "act_quant": spec.act_quant,
        "requires_nvshmem": spec.requires_nvshmem, "tunables": tunables,
    }
    if diagnostics:
        diag.update(diagnostics)

    def run_staged() -> StageResult:
        return StageResult(output=run_impl(), stage_ms={})

    return SchemeInstance(run=run_impl, run_staged=staged_impl or run_staged, diagnostics=diag,
                          close=close_impl or (lambda: None))


def missing_dependency(message: str) -> None:
    raise RuntimeError(message)
