"""The allocation-free all-gather push against the regular one, through the C ABI.

Some callers cannot allocate device memory (a runtime that owns every device byte
through its own arena, or code that may not call cudaMalloc), so they cannot pass
b2m_quant_push the completion counter it needs.  b2m_quant_push_noalloc keeps that
counter in the library's static device memory.  This test runs both entry points
on one GPU (world = 1: the push targets this rank's own gather buffer) on two calls
in a row and requires identical codes, scales and published flags (the quantisation
is bit-exact, so the tolerance is zero, as in the other quant tests).
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from td_benchmark_b200 import _lib  # noqa: E402
from td_benchmark_b200.symm import ptr_array  # noqa: E402

DEV = torch.device("cuda", 0)


def _buffers(T, H):
    return (torch.zeros((T, H), dtype=torch.uint8, device=DEV), torch.zeros((T, H // 128), dtype=torch.float32,
                                                                                device=DEV),
            torch.zeros(1, dtype=torch.int32, device=DEV))


def test_noalloc_push_matches_regular_push_on_two_calls():
    T, H = 96, 1024
    stream = torch.cuda.current_stream(DEV).cuda_stream
    qa, sa, fa = _buffers(T, H)
    qb, sb, fb = _buffers(T, H)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    for call, epoch in enumerate((1, 2)):
        x = (torch.randn((T, H), generator=torch.Generator().manual_seed(call)) * 3.0).to(torch.bfloat16).to(DEV)
        _lib.call("b2m_quant_push", x.data_ptr(), T, H, H, 1, ptr_array([qa.data_ptr()]), ptr_array([sa.data_ptr()]),
                  0, ptr_array([fa.data_ptr()]), epoch, counter.data_ptr(), stream)
        _lib.call("b2m_quant_push_noalloc", x.data_ptr(), T, H, H, 1, ptr_array([qb.data_ptr()]),
                  ptr_array([sb.data_ptr()]), 0, ptr_array([fb.data_ptr()]), epoch, stream)
        torch.cuda.synchronize(DEV)
        assert torch.equal(qa, qb), f"codes differ on call {call}"
        assert torch.equal(sa, sb), f"scales differ on call {call}"
        assert int(fa.item()) == epoch and int(fb.item()) == epoch
        assert int(counter.item()) == 0
        assert np.isfinite(sb.cpu().numpy()).all()


def test_noalloc_push_rejects_world_beyond_limit():
    x = torch.zeros((8, 128), dtype=torch.bfloat16, device=DEV)
    ptrs = ptr_array([x.data_ptr()] * 9)
    with pytest.raises(_lib.B2MError, match="world=9"):
        _lib.call("b2m_quant_push_noalloc", x.data_ptr(), 8, 128, 128, 9, ptrs, ptrs, 0, ptrs, 1,
                  torch.cuda.current_stream(DEV).cuda_stream)


def test_noalloc_push_rejects_bad_shape_before_enqueueing():
    """A bad shape is refused by the argument checks, before the scratch counter is cleared."""
    x = torch.zeros((8, 128), dtype=torch.bfloat16, device=DEV)
    ptrs = ptr_array([x.data_ptr()])
    with pytest.raises(_lib.B2MError, match="quant_push_noalloc: bad shape"):
        _lib.call("b2m_quant_push_noalloc", x.data_ptr(), 8, 100, 128, 1, ptrs, ptrs, 0, ptrs, 1,
                  torch.cuda.current_stream(DEV).cuda_stream)
    with pytest.raises(_lib.B2MError, match="null peer pointer"):
        _lib.call("b2m_quant_push_noalloc", x.data_ptr(), 8, 128, 128, 1, ptrs, ptr_array([0]), 0, ptrs, 1,
                  torch.cuda.current_stream(DEV).cuda_stream)
