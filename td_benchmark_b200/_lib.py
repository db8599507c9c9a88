"""ctypes binding of the b2m C ABI (``include/b2m.h``).

The library is built in-tree (``python -m td_benchmark_b200.build``) as
``td_benchmark_b200/libb2m.so``.  There is no fallback: if the library is missing
or a call fails, a ``RuntimeError`` carrying ``b2m_last_error()`` is raised.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb2m.so"

_c = ctypes
_i32, _i64, _u64, _p = _c.c_int32, _c.c_int64, _c.c_uint64, _c.c_void_p

# name -> argtypes, in header order.  Every function returns int (B2M_OK == 0).
SIGNATURES: dict[str, list] = {
    "b2m_version": [],
    "b2m_set_timeout_ns": [_u64],
    "b2m_quant_g128": [_p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p],
    "b2m_quant_g128_t": [_p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p],
    "b2m_quant_dispatch": [_p, _i64, _i64, _i64, _p, _i32, _p, _p, _i64, _p, _p, _i64, _p],
    "b2m_dispatch_rows": [_p, _p, _i64, _i64, _p, _i32, _p, _p, _i64, _p],
    "b2m_align": [_p, _i64, _i32, _i32, _p, _p, _i64, _p, _i64, _p, _p, _p, _p],
    "b2m_block_order": [_p, _p, _i64, _i32, _i64, _i32, _i32, _p, _i64, _p, _p],
    "b2m_w1_interleave": [_p, _p, _i32, _i32, _i64, _p, _p, _p],
    "b2m_gemm1": [_p, _p, _i64, _i64, _p, _p, _i32, _i32, _p, _p, _p, _p, _p, _p, _p],
    "b2m_gemm1_wait": [_p, _p, _i64, _i64, _p, _p, _i32, _i32, _p, _p, _p, _p, _i64, _i32, _i64, _p, _c.c_uint32, _p,
                       _i64, _p, _p, _p, _p, _i32, _i32, _p, _p, _p, _p],
    "b2m_gemm2": [_p, _p, _i64, _i32, _p, _p, _i32, _i64, _p, _p, _p, _p, _i64, _p, _p, _i64, _i64, _i32, _p, _p],
    "b2m_gemm2_scatter": [_p, _p, _i64, _i32, _p, _p, _i32, _i64, _p, _p, _p, _p, _i64, _p, _p, _i32, _i64, _i64, _p,
                          _p],
    "b2m_combine": [_p, _i64, _i32, _i64, _p, _p, _p, _p, _i64, _p],
    "b2m_copy_async": [_p, _p, _i64, _p],
    "b2m_copy2d_async": [_p, _i64, _p, _i64, _i64, _i64, _p],
    "b2m_symm_alloc": [_i64, _c.POINTER(_p)],
    "b2m_symm_free": [_p],
    "b2m_ipc_handle": [_p, _p],
    "b2m_ipc_open": [_p, _c.POINTER(_p)],
    "b2m_ipc_close": [_p],
    "b2m_quant_push": [_p, _i64, _i64, _i64, _i32, _p, _p, _i64, _p, _c.c_uint32, _p, _p],
    "b2m_quant_push_noalloc": [_p, _i64, _i64, _i64, _i32, _p, _p, _i64, _p, _c.c_uint32, _p],
    "b2m_quant_dispatch_push": [_p, _i64, _i64, _i64, _p, _i32, _i64, _i32, _i32, _p, _p, _i64, _p, _c.c_uint32, _p,
                                _p],
    "b2m_dispatch_rows_wait": [_p, _p, _i64, _i64, _p, _i32, _p, _p, _i64, _p, _i32, _i32, _c.c_uint32, _p, _p],
    "b2m_combine_push": [_p, _i64, _i32, _i64, _i64, _i64, _p, _p, _p, _i32, _i32, _p, _p, _c.c_uint32, _p, _i32,
                         _i32, _p],
    "b2m_signal": [_p, _i32, _c.c_uint32, _p],
    "b2m_rs_combine": [_p, _i64, _i32, _i64, _i32, _p, _i32, _c.c_uint32, _p, _p, _p, _p],
    "b2m_rs_reduce": [_p, _i64, _i64, _i32, _i32, _p, _c.c_uint32, _p, _p, _p, _i32, _p, _i32, _p, _p],
    "b2m_combine_push_fp8": [_p, _i64, _i32, _i64, _p, _p, _p, _i32, _i32, _p, _p, _p, _c.c_uint32, _p, _i32, _p],
    "b2m_rs_reduce_fp8": [_p, _p, _i64, _i64, _i32, _p, _c.c_uint32, _p, _p, _p, _i32, _p, _i32, _p, _p],
    "b2m_quant_push_sparse": [_p, _i64, _i64, _i64, _i32, _p, _p, _i64, _p, _c.c_uint32, _p, _p, _i32, _p, _i32, _p],
    "b2m_route_topk": [_p, _i64, _i32, _i32, _p, _p, _p, _p],
}

ERROR_NAMES = {1: "B2M_ERR_ARG", 2: "B2M_ERR_CUDA", 3: "B2M_ERR_UNSUPPORTED"}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B2MError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with {ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and type the library; raise if it is absent."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(f"b2m kernel library not built: {p} is missing "
                               "(run `python -m td_benchmark_b200.build` on a machine with nvcc)")
        lib = ctypes.CDLL(str(p))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.b2m_last_error.argtypes = []
        lib.b2m_last_error.restype = ctypes.c_char_p
        if path is None:
            _lib = lib
        return lib


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise B2MError(name, rc, lib.b2m_last_error().decode(errors="replace"))
