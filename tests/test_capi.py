"""The C-ABI library loads without a GPU and exports every symbol the header declares."""
import ctypes
import re
from pathlib import Path

import pytest

from td_benchmark_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b2m.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(b2m_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("b2m_quant_g128", "b2m_align", "b2m_gemm1", "b2m_gemm2", "b2m_combine", "b2m_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.skip("libb2m.so not built (run python -m td_benchmark_b200.build)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    typed = set(_lib.SIGNATURES) | {"b2m_last_error"}
    assert set(_declared()) <= typed


def test_calls_without_gpu_fail_loudly():
    if not _lib.LIB_PATH.exists():
        pytest.skip("libb2m.so not built")
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    lib = _lib.load()
    assert lib.b2m_version() >= 100
    with pytest.raises(_lib.B2MError, match="B2M_ERR"):
        _lib.call("b2m_quant_g128", None, 1, 128, 128, None, 128, None, 1, None)


def test_argument_validation_message():
    if not _lib.LIB_PATH.exists():
        pytest.skip("libb2m.so not built")
    with pytest.raises(_lib.B2MError, match="timeout"):
        _lib.call("b2m_set_timeout_ns", 10)


def test_noalloc_push_validates_before_touching_the_device():
    """Argument errors of the allocation-free push come back without a GPU (nothing is enqueued)."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("libb2m.so not built")
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    with pytest.raises(_lib.B2MError, match="quant_push_noalloc: bad shape"):
        _lib.call("b2m_quant_push_noalloc", 16, 8, 100, 128, 1, None, None, 0, None, 1, None)
