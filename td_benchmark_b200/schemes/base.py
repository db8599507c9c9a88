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


def _conforms(expected: type, value: Any) -> bool:
    """Type rule of a tunable: a bool tunable takes only True/False, and no other type
    takes a bool (``True`` is not a chunk count, although ``bool`` subclasses ``int``)."""
    is_bool = isinstance(value, bool)
    if expected is bool:
        return is_bool
    return not is_bool and isinstance(value, expected)


def validate_tunables(spec: SchemeSpec, provided: dict[str, Any]) -> dict[str, Any]:
    """Schema defaults overlaid with ``provided``, checked key by key in schema order.

    Unknown keys, then the first value of the wrong type, raise ``SchemeConfigError``
    with the message texts of the reference contract (``moe_bench/schemes/base.py:48-62``).
    """
    schema = spec.tunables_schema
    extra = [key for key in provided if key not in schema]
    if extra:
        raise SchemeConfigError(f"{spec.code} tunables {sorted(extra)} violate schema: allowed keys are "
                                f"{sorted(schema)}")
    resolved: dict[str, Any] = {}
    for key, item in schema.items():
        value = provided[key] if key in provided else item.default
        if not _conforms(item.typ, value):
            raise SchemeConfigError(f"{spec.code}.{key}={value!r} violates schema: expected {item.typ.__name__}")
        resolved[key] = value
    return resolved


# SchemeSpec fields copied into every instance's diagnostics (the results row reads them).
_DIAGNOSTIC_FIELDS = ("name", "family", "parallel", "weight_dtype", "act_quant", "requires_nvshmem")


def _no_op() -> None:
    return None


def make_lazy_instance(spec: SchemeSpec, tunables: dict[str, Any], run_impl: Callable[[], Any],
                       diagnostics: dict[str, Any] | None = None,
                       close_impl: Callable[[], None] | None = None,
                       staged_impl: Callable[[], StageResult] | None = None) -> SchemeInstance:
    """Wrap a prepared forward as a ``SchemeInstance``.

    The diagnostics dict carries the scheme code, the spec's descriptive fields and the
    resolved tunables, then any scheme-specific entries (which may override them).
    Without ``staged_impl`` the staged run is the plain run with no stage times.
    """
    diag: dict[str, Any] = {"scheme": spec.code}
    diag.update((f, getattr(spec, f)) for f in _DIAGNOSTIC_FIELDS)
    diag["tunables"] = tunables
    diag.update(diagnostics or {})
    if staged_impl is None:
        def staged_impl() -> StageResult:
            return StageResult(output=run_impl(), stage_ms={})
    return SchemeInstance(run=run_impl, run_staged=staged_impl, diagnostics=diag, close=close_impl or _no_op)


def missing_dependency(message: str) -> None:
    """A scheme whose runtime dependency is absent fails with RuntimeError (the reference's rule)."""
    raise RuntimeError(message)
