"""The drop-in boundary against the reference package itself (CPU; skipped where it is absent).

``register_into_reference()`` must make the B200 codes usable through the reference's own
entry points: ``moe_bench.config.SchemeCfg`` validation (``config.py:45, 113-114``), the
``REGISTRY`` lookup and ``build_scheme`` (``schemes/__init__.py:18-37``), with tunable errors
raised as the reference's ``SchemeConfigError`` and a missing data bundle as ``RuntimeError``
(the contract of ``tests/test_schemes_ab.py`` in the reference).
"""
import sys
from pathlib import Path

import pytest

REF = Path("/root/reference")


@pytest.fixture()
def ref(monkeypatch):
    if not (REF / "moe_bench" / "schemes" / "base.py").exists():
        pytest.skip("reference package not present on this machine")
    monkeypatch.syspath_prepend(str(REF))
    import moe_bench.config as config
    import moe_bench.schemes as schemes
    import moe_bench.schemes.base as base
    saved_reg, saved_codes = dict(schemes.REGISTRY), set(config._SCHEME_CODES)
    yield config, schemes, base
    schemes.REGISTRY.clear()
    schemes.REGISTRY.update(saved_reg)
    config._SCHEME_CODES.clear()
    config._SCHEME_CODES.update(saved_codes)


def _ctx():
    from moe_bench.context import DistContext
    return DistContext(rank=0, world_size=1, local_rank=0, device="cpu", group=None, nvshmem_initialized=False)


def test_reference_rejects_b200_codes_before_registration(ref):
    config, _, _ = ref
    with pytest.raises(config.ConfigError, match="schemes.enabled"):
        config.SchemeCfg("d3", {})


def test_registered_codes_validate_and_resolve_through_the_reference(ref):
    config, schemes, base = ref
    from td_benchmark_b200.schemes import register_into_reference
    added = register_into_reference()
    assert sorted(added) == ["d1", "d2", "d3", "d4"]
    for code, parallel in (("d1", "TP"), ("d2", "EP"), ("d3", "TP"), ("d4", "EP")):
        spec, _ = schemes.REGISTRY[code]
        assert isinstance(spec, base.SchemeSpec) and spec.parallel == parallel
        assert spec.weight_dtype == "fp8" and spec.act_quant == "group128" and not spec.requires_nvshmem
        assert all(isinstance(t, base.TunableSpec) for t in spec.tunables_schema.values())
    cfg = config.SchemeCfg("d3", {"ag_mode": "sm", "rs_mode": "sm"})
    with pytest.raises(RuntimeError, match="DataBundle"):
        schemes.build_scheme(None, _ctx(), None, cfg)
    cfg = config.SchemeCfg("d1", {})
    with pytest.raises(RuntimeError, match="DataBundle"):
        schemes.build_scheme(None, _ctx(), None, cfg)


def test_tunable_errors_surface_as_the_reference_error_type(ref):
    config, schemes, base = ref
    from td_benchmark_b200.schemes import register_into_reference
    register_into_reference()
    with pytest.raises(base.SchemeConfigError, match="violate schema"):
        schemes.build_scheme(None, _ctx(), None, config.SchemeCfg("d3", {"n_chunks": 2}))
    with pytest.raises(base.SchemeConfigError, match="expected one of"):
        schemes.build_scheme(None, _ctx(), None, config.SchemeCfg("d4", {"ag_mode": "nvshmem"}))
    with pytest.raises(base.SchemeConfigError, match="expected bool"):
        schemes.build_scheme(None, _ctx(), None, config.SchemeCfg("d2", {"check_status": 1}))


def test_reference_spec_validation_accepts_b200_specs(ref):
    """The reference's own ``validate_tunables`` reads the re-expressed specs like its own."""
    config, schemes, base = ref
    from td_benchmark_b200.schemes import register_into_reference
    register_into_reference()
    spec, _ = schemes.REGISTRY["d3"]
    vals = base.validate_tunables(spec, {"rs_chunks": 2})
    assert vals["rs_chunks"] == 2 and vals["ag_mode"] == "auto" and vals["check_status"] is False
