"""Bounded device waits: a flag that nothing sets makes the wait run out, the kernel records
the site in the status word and returns, and the context stays usable (one GPU, no fault).

The wait limit is lowered to 1 ms for the duration of each test and restored afterwards.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from td_benchmark_b200 import _lib, ops  # noqa: E402

DEV = torch.device("cuda", 0)
TIMEOUT_PEER = 0x104
DEFAULT_NS = 2_000_000_000


@pytest.fixture()
def short_waits():
    torch.cuda.set_device(DEV)
    _lib.call("b2m_set_timeout_ns", 1_000_000)
    try:
        yield
    finally:
        _lib.call("b2m_set_timeout_ns", DEFAULT_NS)


def _stream():
    return torch.cuda.current_stream(DEV).cuda_stream


def test_dispatch_wait_on_a_flag_nobody_sets(short_waits):
    T, H, world = 256, 256, 2
    xq = torch.zeros((T, H), dtype=torch.uint8, device=DEV)
    xs = torch.ones((T, H // 128), dtype=torch.float32, device=DEV)
    pair_pos = torch.arange(T, dtype=torch.int32, device=DEV)
    a = torch.zeros((T, H), dtype=torch.uint8, device=DEV)
    a_t = torch.zeros((H // 128, T), dtype=torch.float32, device=DEV)
    flags = torch.tensor([1, 0], dtype=torch.int32, device=DEV)   # own rows present, rank 1 never arrives
    status = ops.new_status(DEV)
    _lib.call("b2m_dispatch_rows_wait", xq.data_ptr(), xs.data_ptr(), T, H, pair_pos.data_ptr(), 1, a.data_ptr(),
              a_t.data_ptr(), T, flags.data_ptr(), world, 0, 1, status.data_ptr(), _stream())
    torch.cuda.synchronize(DEV)                      # returns: the kernel gave up, nothing faulted
    assert int(status.item()) == TIMEOUT_PEER
    # the own source's rows were dispatched before the wait on rank 1 ran out
    assert torch.equal(a_t[:, :T // 2], xs[:T // 2].T)
    # the context is usable: a regular quant on the same stream succeeds
    x = torch.randn((8, 256), device=DEV).to(torch.bfloat16)
    q, s = ops.quant_g128(x)
    torch.cuda.synchronize(DEV)
    assert torch.isfinite(s).all()


def _gemm_inputs(E=2, inter=128, H=256, T=256):
    w1 = (torch.randn((E, 2 * inter, H), device=DEV) * 0.05).to(ops.FP8)
    w1s = torch.rand((E, 2 * inter // 128, H // 128), device=DEV) + 0.5
    w1i, w1is = ops.w1_interleave(w1, w1s)
    ids = (torch.arange(T, device=DEV, dtype=torch.int32) % E).reshape(T, 1).contiguous()
    cap, nblk = ops.align_sizes(T, E, 128)
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=DEV)
    eids = torch.empty(nblk, dtype=torch.int32, device=DEV)
    ntpp = torch.empty(1, dtype=torch.int32, device=DEV)
    pair_pos = torch.empty(T, dtype=torch.int32, device=DEV)
    ops.moe_align_block_size(ids, 128, E, None, out=(sorted_ids, eids, ntpp), pair_pos=pair_pos)
    rows_cap = nblk * 128
    x = torch.randn((T, H), device=DEV).to(torch.bfloat16)
    a = torch.empty((rows_cap, H), dtype=ops.FP8, device=DEV)
    a_t = torch.empty((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.quant_dispatch(x, pair_pos, 1, a, a_t)
    out_q = torch.empty((rows_cap, inter), dtype=ops.FP8, device=DEV)
    out_s = torch.empty((inter // 128, rows_cap), dtype=torch.float32, device=DEV)
    return dict(a=a, a_t=a_t, w1i=w1i, w1is=w1is, eids=eids, ntpp=ntpp, sorted_ids=sorted_ids, out_q=out_q,
                out_s=out_s, rows_cap=rows_cap, H=H, E=E, inter=inter, T=T, nblk=nblk)


def test_gemm1_wait_on_a_flag_nobody_sets_frees_tmem(short_waits):
    g = _gemm_inputs()
    status = ops.new_status(DEV)
    order = torch.arange(g["nblk"], dtype=torch.int32, device=DEV)
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)          # neither source ever arrives
    _lib.call("b2m_gemm1_wait", g["a"].data_ptr(), g["a_t"].data_ptr(), g["rows_cap"], g["H"], g["w1i"].data_ptr(),
              g["w1is"].data_ptr(), g["E"], g["inter"], g["eids"].data_ptr(), g["ntpp"].data_ptr(), order.data_ptr(),
              g["sorted_ids"].data_ptr(), g["T"], 1, g["T"] // 2, flags.data_ptr(), 1, None, 0, None, None, None,
              None, 2, 0, g["out_q"].data_ptr(), g["out_s"].data_ptr(), status.data_ptr(), _stream())
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == TIMEOUT_PEER
    # TMEM and the CTA's barriers were released: the same GEMM without waits runs clean twice
    status.zero_()
    outs = []
    for _ in range(2):
        ops.gemm1(g["a"], g["a_t"], g["w1i"], g["w1is"], g["eids"], g["ntpp"], g["out_q"], g["out_s"], status)
        torch.cuda.synchronize(DEV)
        outs.append((g["out_q"].view(torch.uint8).clone(), g["out_s"].clone()))
    assert int(status.item()) == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    # and with the flags set the waiting GEMM gives the same result
    flags.fill_(1)
    _lib.call("b2m_gemm1_wait", g["a"].data_ptr(), g["a_t"].data_ptr(), g["rows_cap"], g["H"], g["w1i"].data_ptr(),
              g["w1is"].data_ptr(), g["E"], g["inter"], g["eids"].data_ptr(), g["ntpp"].data_ptr(), order.data_ptr(),
              g["sorted_ids"].data_ptr(), g["T"], 1, g["T"] // 2, flags.data_ptr(), 1, None, 0, None, None, None,
              None, 2, 0, g["out_q"].data_ptr(), g["out_s"].data_ptr(), status.data_ptr(), _stream())
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0
    assert torch.equal(g["out_q"].view(torch.uint8), outs[0][0]) and torch.equal(g["out_s"], outs[0][1])


def test_gemm1_wait_rejects_more_than_eight_sources():
    g = _gemm_inputs()
    order = torch.arange(g["nblk"], dtype=torch.int32, device=DEV)
    flags = torch.zeros(16, dtype=torch.int32, device=DEV)
    status = ops.new_status(DEV)
    with pytest.raises(_lib.B2MError, match="more than 8 source ranks"):
        _lib.call("b2m_gemm1_wait", g["a"].data_ptr(), g["a_t"].data_ptr(), g["rows_cap"], g["H"],
                  g["w1i"].data_ptr(), g["w1is"].data_ptr(), g["E"], g["inter"], g["eids"].data_ptr(),
                  g["ntpp"].data_ptr(), order.data_ptr(), g["sorted_ids"].data_ptr(), g["T"], 1, 16,
                  flags.data_ptr(), 1, None, 0, None, None, None, None, 2, 0, g["out_q"].data_ptr(),
                  g["out_s"].data_ptr(), status.data_ptr(), _stream())
