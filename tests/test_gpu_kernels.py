"""Kernel parity on a B200: CUDA path through the C ABI vs the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import align as oalign
from oracle import fp8 as ofp8
from oracle import quant as oquant

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from td_benchmark_b200 import ops, weights  # noqa: E402

DEV = torch.device("cuda", 0)


def _bf16(shape, seed, scale=1.0):
    return (torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * scale).to(torch.bfloat16)


# ---------------------------------------------------------------- K1 quant
@pytest.mark.parametrize("rows,cols", [(1, 128), (7, 256), (512, 4096), (1024, 7168), (3, 129), (5, 300),
                                       (33, 2048), (0, 256), (2, 384)])
def test_quant_bit_exact(rows, cols):
    x = _bf16((rows, cols), rows * 1000 + cols, 3.0)
    if rows > 2:
        x[1, :128] = 0                     # all-zero group -> scale 1e-12
        x[2, 5] = 3.0e4                    # one huge value in a group
    q, s = ops.quant_g128(x.to(DEV))
    torch.cuda.synchronize()
    qr, sr = oquant.quant_g128(x.float().numpy())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qr)
    assert np.array_equal(s.cpu().numpy(), sr)


@pytest.mark.parametrize("rows,cols,world", [(1, 128, 1), (7, 4096, 2), (33, 7168, 3), (512, 4096, 8),
                                             (1024, 7168, 2)])
def test_quant_push_bit_exact(rows, cols, world):
    """All-gather push (peers emulated by buffers on this GPU): every destination holds the
    oracle's codes and scales at the source's rows, and every flag holds the epoch."""
    from td_benchmark_b200 import _lib
    from td_benchmark_b200.symm import ptr_array

    x = _bf16((rows, cols), rows * 31 + cols, 3.0)
    if rows > 2:
        x[1, :128] = 0
        x[2, 5] = 3.0e4
    xd = x.to(DEV)
    row0 = rows  # the source owns rows [rows, 2 rows) of a 2-rank-tall gather buffer
    qs = [torch.zeros((2 * rows, cols), dtype=torch.uint8, device=DEV) for _ in range(world)]
    ss = [torch.zeros((2 * rows, cols // 128), dtype=torch.float32, device=DEV) for _ in range(world)]
    flags = torch.zeros(world, dtype=torch.int32, device=DEV)
    counter = torch.zeros(4, dtype=torch.int32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("b2m_quant_push", xd.data_ptr(), rows, cols, cols, world, ptr_array([q.data_ptr() for q in qs]),
              ptr_array([s.data_ptr() for s in ss]), row0, ptr_array([flags.data_ptr() + 4 * r for r in range(world)]),
              7, counter.data_ptr(), st)
    torch.cuda.synchronize()
    qr, sr = oquant.quant_g128(x.float().numpy())
    for q, s in zip(qs, ss):
        assert np.array_equal(q[row0:].cpu().numpy(), qr)
        assert np.array_equal(s[row0:].cpu().numpy(), sr)
        assert not q[:row0].any()
    assert flags.tolist() == [7] * world and counter[0].item() == 0


def test_quant_strided_rows_and_offset_output():
    big = _bf16((64, 1024), 5)
    x = big[:, 256:768]                    # row stride 1024
    q = torch.zeros((64, 640), dtype=torch.uint8, device=DEV)
    s = torch.zeros((64, 8), dtype=torch.float32, device=DEV)
    xd = big.to(DEV)[:, 256:768]
    ops.quant_g128(xd, q[:, 64:576].view(torch.float8_e4m3fn), s[:, 2:6])
    qr, sr = oquant.quant_g128(x.float().numpy())
    assert np.array_equal(q[:, 64:576].cpu().numpy(), qr)
    assert np.array_equal(s[:, 2:6].cpu().numpy(), sr)
    assert q[:, :64].abs().sum() == 0 and s[:, :2].abs().sum() == 0


# ---------------------------------------------------------------- K2 align
def _ids(T, k, E, seed, zipf=False):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn((T, E), generator=g)
    if zipf:
        logits += 2.0 * torch.log(torch.arange(1, E + 1, dtype=torch.float32) ** -1.2)
    return torch.topk(logits, k, dim=-1).indices.to(torch.int32).contiguous()


def _inverse(sr, numel, er=None, bs=128):
    pos = np.full(numel, -1, np.int64)
    for p, pair in enumerate(sr):
        if pair < numel and (er is None or er[p // bs] >= 0):
            pos[pair] = p
    return pos


@pytest.mark.parametrize("T,k,E,bs,zipf", [(64, 2, 8, 128, False), (4096, 2, 8, 128, False),
                                           (8192, 8, 256, 128, True), (32, 8, 128, 128, False),
                                           (3, 2, 64, 128, False), (1, 1, 8, 16, False), (1000, 4, 33, 64, True),
                                           (32768, 8, 256, 128, True), (0, 2, 8, 128, False)])
def test_align_bit_exact(T, k, E, bs, zipf):
    ids = _ids(T, k, E, T + E, zipf) if T else torch.zeros((0, k), dtype=torch.int32)
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    s, e, n = ops.moe_align_block_size(ids.to(DEV), bs, E, pair_pos=pp)
    sr, er, nr = oalign.moe_align_block_size(ids.numpy(), bs, E)
    assert int(n.item()) == int(nr[0])
    assert np.array_equal(s.cpu().numpy(), sr)
    assert np.array_equal(e.cpu().numpy(), er)
    assert np.array_equal(pp.cpu().numpy(), _inverse(sr, T * k))


def test_align_expert_map():
    E, P, r = 256, 8, 3
    ids = _ids(2048, 8, E, 11, zipf=True)
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[r * 32:(r + 1) * 32] = torch.arange(32, dtype=torch.int32)
    pp = torch.empty(ids.numel(), dtype=torch.int32, device=DEV)
    s, e, n = ops.moe_align_block_size(ids.to(DEV), 128, E, emap.to(DEV), pair_pos=pp)
    sr, er, nr = oalign.moe_align_block_size(ids.numpy(), 128, E, emap.numpy())
    assert int(n.item()) == int(nr[0]) and np.array_equal(s.cpu().numpy(), sr) and np.array_equal(e.cpu().numpy(), er)
    assert np.array_equal(pp.cpu().numpy(), _inverse(sr, ids.numel(), er))


def test_align_block_pairs():
    E = 16
    ids = _ids(1000, 4, E, 3, zipf=True)
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[4:12] = torch.arange(8, dtype=torch.int32)
    for m in (None, emap):
        nblk = ops.align_sizes(ids.numel(), E, 128)[1]
        bp = torch.full((1 + 2 * nblk,), -7, dtype=torch.int32, device=DEV)
        s, e, n = ops.moe_align_block_size(ids.to(DEV), 128, E, None if m is None else m.to(DEV), block_pairs=bp)
        er = e.cpu().numpy()
        bpn = bp.cpu().numpy()
        got = [(bpn[1 + 2 * i], bpn[2 + 2 * i]) for i in range(bpn[0])]
        exp = []
        nb = int(n.item()) // 128
        b = 0
        while b < nb:
            if er[b] < 0:
                b += 1
                continue
            if b + 1 < nb and er[b + 1] == er[b]:
                exp.append((b, b + 1))
                b += 2
            else:
                exp.append((b, -1))
                b += 1
        assert got == exp


def test_align_rejects_small_buffers():
    from td_benchmark_b200._lib import B2MError
    ids = _ids(64, 2, 8, 1).to(DEV)
    with pytest.raises(B2MError, match="sorted_cap"):
        ops.moe_align_block_size(ids, 128, 8, out=(torch.empty(10, dtype=torch.int32, device=DEV),
                                                   torch.empty(10, dtype=torch.int32, device=DEV),
                                                   torch.empty(1, dtype=torch.int32, device=DEV)))


# ---------------------------------------------------------------- weight interleave
def test_w1_interleave():
    E, I, H = 3, 384, 256
    w = torch.randn((E, 2 * I, H), generator=torch.Generator().manual_seed(2)) * 0.02
    q, s = weights.quantize_block128(w)
    qi, si = ops.w1_interleave(q.to(DEV), s.to(DEV))
    qb = q.view(torch.uint8)
    exp = torch.cat([torch.cat([qb[:, j * 128:(j + 1) * 128], qb[:, I + j * 128:I + (j + 1) * 128]], 1)
                     for j in range(I // 128)], 1)
    exp_s = torch.cat([torch.cat([s[:, j:j + 1], s[:, I // 128 + j:I // 128 + j + 1]], 1) for j in range(I // 128)], 1)
    assert torch.equal(qi.view(torch.uint8).cpu(), exp)
    assert torch.equal(si.cpu(), exp_s)


# ---------------------------------------------------------------- dispatch into expert order
@pytest.mark.parametrize("T,H,k,E,ep", [(64, 256, 2, 8, False), (300, 1024, 4, 16, False), (256, 512, 8, 32, True)])
def test_quant_dispatch_and_dispatch_rows_bit_exact(T, H, k, E, ep):
    x = _bf16((T, H), T + H, 2.0)
    ids = _ids(T, k, E, 5 + T)
    emap = None
    if ep:
        emap = torch.full((E,), -1, dtype=torch.int32)
        emap[8:16] = torch.arange(8, dtype=torch.int32)
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    s, e, n = ops.moe_align_block_size(ids.to(DEV), 128, E, None if emap is None else emap.to(DEV), pair_pos=pp)
    rows_cap = e.numel() * 128
    a = torch.zeros((rows_cap, H), dtype=torch.uint8, device=DEV)
    at = torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    qt = torch.zeros((T + 5, H), dtype=torch.uint8, device=DEV)
    st = torch.zeros((H // 128, T + 5), dtype=torch.float32, device=DEV)
    ops.quant_dispatch(x.to(DEV), pp, k, a.view(torch.float8_e4m3fn), at, qt.view(torch.float8_e4m3fn), st)
    qr, sr = oquant.quant_g128(x.float().numpy())
    assert np.array_equal(qt[:T].cpu().numpy(), qr) and np.array_equal(st[:, :T].cpu().numpy(), sr.T)
    ppn = pp.cpu().numpy().reshape(T, k)
    an, atn = a.cpu().numpy(), at.cpu().numpy()
    written = np.zeros(rows_cap, bool)
    for t in range(T):
        for j in range(k):
            p = ppn[t, j]
            if p < 0:
                continue
            written[p] = True
            assert np.array_equal(an[p], qr[t]) and np.array_equal(atn[:, p], sr[t])
    assert ep or written.sum() == T * k
    # the same layout from already-quantised rows (the all-gather path)
    a2 = torch.zeros_like(a)
    at2 = torch.zeros_like(at)
    xs = torch.from_numpy(sr).to(DEV).contiguous()
    ops.dispatch_rows(torch.from_numpy(qr).to(DEV).view(torch.float8_e4m3fn), xs, pp, k, a2.view(torch.float8_e4m3fn),
                      at2)
    assert torch.equal(a2, a) and torch.equal(at2, at)


# ---------------------------------------------------------------- K3 / K4 GEMMs
def _gemm_problem(T, H, I, E, k, seed, zipf=False):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn((T, H), generator=g)).to(torch.bfloat16)
    w1 = torch.randn((E, 2 * I, H), generator=g) * 0.02
    w2 = torch.randn((E, H, I), generator=g) * 0.02
    w1q, w1s = weights.quantize_block128(w1)
    w2q, w2s = weights.quantize_block128(w2)
    ids = _ids(T, k, E, seed + 1, zipf)
    wts = torch.rand((T, k), generator=g).float()
    wts = wts / wts.sum(-1, keepdim=True)
    return x, w1q, w1s, w2q, w2s, ids, wts


def _deq_rows(codes_u8, scales):
    return ofp8.decode_e4m3(codes_u8).astype(np.float64) * np.repeat(scales, 128, axis=-1)[..., :codes_u8.shape[-1]]


def _deq_w(q, s):
    qn = ofp8.decode_e4m3(q.view(torch.uint8).numpy()).astype(np.float64)
    sn = np.repeat(np.repeat(s.numpy().astype(np.float64), 128, 1), 128, 2)
    return qn * sn


@pytest.mark.parametrize("paired", [True, False], ids=["pair", "single"])
@pytest.mark.parametrize("T,H,I,E,k,zipf", [(200, 512, 256, 4, 2, False), (64, 256, 512, 8, 2, False),
                                            (300, 1024, 384, 16, 4, True), (5, 256, 128, 8, 2, False),
                                            (700, 256, 256, 3, 2, False)])
def test_gemm1_gemm2_against_float64(T, H, I, E, k, zipf, paired):
    x, w1q, w1s, w2q, w2s, ids, wts = _gemm_problem(T, H, I, E, k, T + H, zipf)
    xq, xs = ops.quant_g128(x.to(DEV))
    w1i, w1is = ops.w1_interleave(w1q.to(DEV), w1s.to(DEV))
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    bp = torch.empty(1 + 2 * ops.align_sizes(T * k, E, 128)[1], dtype=torch.int32, device=DEV) if paired else None
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids.to(DEV), 128, E, pair_pos=pp, block_pairs=bp)
    rows_cap = eids.numel() * 128
    a_sorted = torch.empty((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    a_st = torch.empty((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.dispatch_rows(xq, xs, pp, k, a_sorted, a_st)
    status = ops.new_status(DEV)
    hq, hst = ops.gemm1(a_sorted, a_st, w1i, w1is, eids, ntpp, status=status, block_pairs=bp)
    staged = ops.gemm2(hq, hst, w2q.to(DEV), w2s.to(DEV), sorted_ids, eids, ntpp, T * k, wts.reshape(-1).to(DEV),
                       status=status, block_pairs=bp)
    torch.cuda.synchronize()
    ops.check_status(status)
    n = int(ntpp.item())
    srt = sorted_ids.cpu().numpy()[:n]
    valid = srt < T * k
    # float64 reference of GEMM1 + silu*mul on the same quantised activations
    a = _deq_rows(xq.view(torch.uint8).cpu().numpy(), xs.cpu().numpy())           # [T, H]
    W1 = _deq_w(w1q, w1s)
    W2 = _deq_w(w2q, w2s)
    eid_rows = np.repeat(eids.cpu().numpy()[:n // 128], 128)
    rows = np.nonzero(valid)[0]
    toks = srt[rows] // k
    gu = np.einsum("rh,rnh->rn", a[toks], W1[eid_rows[rows]])
    h = gu[:, :I] / (1 + np.exp(-gu[:, :I])) * gu[:, I:]
    hq_np = hq.view(torch.uint8).cpu().numpy()[rows]
    hs_np = hst.cpu().numpy()[:, rows].T
    h_gpu = _deq_rows(hq_np, hs_np)
    # scales: amax/448 of nearly the same values
    sref = np.maximum(np.abs(h).reshape(len(rows), I // 128, 128).max(-1) / 448.0, 1e-12)
    np.testing.assert_allclose(hs_np, sref, rtol=1e-4)
    # codes: within one e4m3 step of the float64 value (quantisation + fp32 accumulation;
    # the epilogue codes h * (1/scale) and uses a fast exp/reciprocal in silu)
    step = np.repeat(hs_np, 128, axis=1) * np.maximum(2.0 ** (np.floor(np.log2(np.maximum(np.abs(h) / np.repeat(hs_np, 128, axis=1), 2.0 ** -6))) - 3), 2.0 ** -9)
    assert np.all(np.abs(h_gpu - h) <= step * 1.01 + 1e-30)
    # GEMM2 on the GPU's own intermediate, float64 reference
    pairs = srt[rows]
    y = np.einsum("ri,rni->rn", h_gpu, W2[eid_rows[rows]]) * wts.reshape(-1).numpy()[pairs][:, None]
    got = staged.float().cpu().numpy()[pairs]
    np.testing.assert_allclose(got, y, rtol=2 ** -7, atol=1e-3 * np.abs(y).max())


@pytest.mark.parametrize("paired", [True, False], ids=["pair", "single"])
def test_gemm_skips_non_local_experts(paired):
    T, H, I, E, k = 128, 256, 128, 8, 2
    x, w1q, w1s, w2q, w2s, ids, wts = _gemm_problem(T, H, I, E, k, 77)
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[2:4] = torch.tensor([0, 1], dtype=torch.int32)
    w1i, w1is = ops.w1_interleave(w1q[2:4].contiguous().to(DEV), w1s[2:4].contiguous().to(DEV))
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    bp = torch.empty(1 + 2 * ops.align_sizes(T * k, E, 128)[1], dtype=torch.int32, device=DEV) if paired else None
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids.to(DEV), 128, E, emap.to(DEV), pair_pos=pp, block_pairs=bp)
    rows_cap = eids.numel() * 128
    a_sorted = torch.empty((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    a_st = torch.empty((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.quant_dispatch(x.to(DEV), pp, k, a_sorted, a_st)
    staged = torch.full((T * k, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    hq, hst = ops.gemm1(a_sorted, a_st, w1i, w1is, eids, ntpp, block_pairs=bp)
    ops.gemm2(hq, hst, w2q[2:4].contiguous().to(DEV), w2s[2:4].contiguous().to(DEV), sorted_ids, eids, ntpp, T * k,
              wts.reshape(-1).to(DEV), out=staged, block_pairs=bp)
    out = ops.combine(staged, k, ids.to(DEV), emap.to(DEV))
    torch.cuda.synchronize()
    local = ((ids == 2) | (ids == 3)).reshape(-1)
    st = staged.float().cpu()
    assert torch.isfinite(st[local]).all() and torch.isnan(st[~local]).all()
    assert torch.isfinite(out.float()).all()


# ---------------------------------------------------------------- combine
@pytest.mark.parametrize("T,k,H,shared", [(64, 2, 256, False), (100, 8, 1024, True), (1, 1, 128, True)])
def test_combine_bit_exact(T, k, H, shared):
    st = _bf16((T * k, H), 3)
    sh = _bf16((T, H), 4) if shared else None
    out = ops.combine(st.to(DEV), k, shared=None if sh is None else sh.to(DEV))
    acc = np.zeros((T, H), np.float32)
    s3 = st.float().numpy().reshape(T, k, H)
    for j in range(k):
        acc = (acc + s3[:, j]).astype(np.float32)
    if sh is not None:
        acc = (acc + sh.float().numpy()).astype(np.float32)
    exp = ofp8.f32_to_bf16_bits(acc)
    assert np.array_equal(out.view(torch.int16).cpu().numpy().astype(np.uint16), exp)


@pytest.mark.parametrize("k", [8, 40])
def test_combine_expert_map_bit_exact(k):
    """Only local pairs count (expert map >= 0), summed in ascending j, then the shared row;
    k = 40 takes the kernel instantiation that tests pairs j >= 32 one by one."""
    T, H, E = 96, 512, 64
    g = torch.Generator().manual_seed(k)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[::3] = torch.arange(len(emap[::3]), dtype=torch.int32)
    st = _bf16((T * k, H), 11)
    sh = _bf16((T, H), 12)
    out = ops.combine(st.to(DEV), k, ids.to(DEV), emap.to(DEV), sh.to(DEV))
    local = (emap[ids.long()] >= 0).numpy()
    s3 = st.float().numpy().reshape(T, k, H)
    acc = np.zeros((T, H), np.float32)
    for j in range(k):
        acc = np.where(local[:, j:j + 1], (acc + s3[:, j]).astype(np.float32), acc)
    acc = (acc + sh.float().numpy()).astype(np.float32)
    assert np.array_equal(out.view(torch.int16).cpu().numpy().astype(np.uint16), ofp8.f32_to_bf16_bits(acc))


@pytest.mark.parametrize("world,src,paired,H", [(2, 1, False, 512), (4, 0, False, 640), (4, 3, True, 512),
                                                 (2, 0, False, 384)])
def test_gemm2_scatter_and_rs_combine(world, src, paired, H):
    """Down GEMM storing into owner buffers (owners emulated by buffers on this GPU): every
    pair row lands bit-identical to b2m_gemm2's row at owner p // ppo, row row0 + p - q*ppo;
    the owner combine equals a sequential fp32 sum over sources and top-k rows.  H = 640 and
    384 end on a half column tile (a 256-byte row piece instead of 512)."""
    from td_benchmark_b200 import _lib
    from td_benchmark_b200.symm import ptr_array

    T, I, E, k = 256, 256, 4, 2
    x, w1q, w1s, w2q, w2s, ids, wts = _gemm_problem(T, H, I, E, k, 77 + world, False)
    xq, xs = ops.quant_g128(x.to(DEV))
    w1i, w1is = ops.w1_interleave(w1q.to(DEV), w1s.to(DEV))
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    bp = torch.empty(1 + 2 * ops.align_sizes(T * k, E, 128)[1], dtype=torch.int32, device=DEV) if paired else None
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids.to(DEV), 128, E, pair_pos=pp, block_pairs=bp)
    rows_cap = eids.numel() * 128
    a_sorted = torch.empty((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    a_st = torch.empty((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.dispatch_rows(xq, xs, pp, k, a_sorted, a_st)
    status = ops.new_status(DEV)
    hq, hst = ops.gemm1(a_sorted, a_st, w1i, w1is, eids, ntpp, status=status, block_pairs=bp)
    w2d, w2sd, wd = w2q.to(DEV), w2s.to(DEV), wts.reshape(-1).to(DEV).contiguous()
    staged = ops.gemm2(hq, hst, w2d, w2sd, sorted_ids, eids, ntpp, T * k, wd, status=status, block_pairs=bp)
    ppo = T * k // world
    recv = [torch.zeros((world * ppo, H), dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    _lib.call("b2m_gemm2_scatter", hq.data_ptr(), hst.data_ptr(), rows_cap, I, w2d.data_ptr(), w2sd.data_ptr(), E, H,
              sorted_ids.data_ptr(), eids.data_ptr(), ntpp.data_ptr(), None if bp is None else bp.data_ptr(), T * k,
              wd.data_ptr(), ptr_array([r.data_ptr() for r in recv]), world, ppo, src * ppo, status.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ops.check_status(status)
    for q in range(world):
        assert torch.equal(recv[q][src * ppo:(src + 1) * ppo], staged[q * ppo:(q + 1) * ppo])
        assert not recv[q][:src * ppo].any() and not recv[q][(src + 1) * ppo:].any()
    # owner combine over `world` sources of top-k rows (+ an added row), flags already at the epoch
    q = world - 1
    for s in range(world):                        # fill the other sources' blocks with distinct rows
        if s != src:
            recv[q][s * ppo:(s + 1) * ppo] = (staged[q * ppo:(q + 1) * ppo].float() * (0.5 + s)).to(torch.bfloat16)
    rows = T // world
    add = _bf16((rows, H), 5)
    flags = torch.full((world,), 3, dtype=torch.int32, device=DEV)
    out = torch.empty((rows, H), dtype=torch.bfloat16, device=DEV)
    _lib.call("b2m_rs_combine", recv[q].data_ptr(), rows, k, H, world, flags.data_ptr(), world, 3,
              add.to(DEV).data_ptr(), out.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ops.check_status(status)
    r = recv[q].float().cpu().numpy().reshape(world, rows, k, H)
    acc = np.zeros((rows, H), dtype=np.float32)
    for s in range(world):
        for j in range(k):
            acc = acc + r[s, :, j]
    acc = acc + add.float().numpy()
    assert torch.equal(out.cpu(), torch.from_numpy(acc).to(torch.bfloat16))


def _route(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)


@pytest.mark.parametrize("T,H,k,E,world,src", [(512, 1024, 2, 8, 4, 2), (256, 2048, 8, 16, 2, 0), (96, 512, 3, 5, 3, 1)])
def test_quant_dispatch_push_bit_exact(T, H, k, E, world, src):
    """All-gather into the sorted operand (destinations emulated by buffers on this GPU): each
    destination holds exactly the source's rows and scales that b2m_quant_dispatch writes."""
    from td_benchmark_b200 import _lib
    from td_benchmark_b200.symm import ptr_array

    x = _bf16((T, H), T + H + k, 2.0).to(DEV)
    ids = _route(T, k, E, 3).to(DEV)
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids, 128, E, pair_pos=pp)
    rows_cap = eids.numel() * 128
    a_ref = torch.zeros((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    s_ref = torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.quant_dispatch(x, pp, k, a_ref, s_ref)
    Tl = T // world
    a_d = [torch.zeros((rows_cap, H), dtype=torch.uint8, device=DEV) for _ in range(world)]
    s_d = [torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV) for _ in range(world)]
    flags = torch.zeros(world, dtype=torch.int32, device=DEV)
    counters = torch.zeros(world, dtype=torch.int32, device=DEV)
    xs = x[src * Tl:(src + 1) * Tl].contiguous()
    for epoch in (5, 6):                            # second call: counters must have been re-armed
        _lib.call("b2m_quant_dispatch_push", xs.data_ptr(), Tl, H, H, pp.data_ptr(), k, src * Tl, world, src,
                  ptr_array([a.data_ptr() for a in a_d]), ptr_array([s.data_ptr() for s in s_d]), rows_cap,
                  ptr_array([flags.data_ptr() + 4 * d for d in range(world)]), epoch, counters.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert flags.tolist() == [epoch] * world and not counters.any()
    pos = pp.view(T, k)[src * Tl:(src + 1) * Tl].reshape(-1).long().cpu()
    pos = pos[pos >= 0]
    mask = torch.zeros(rows_cap, dtype=torch.bool)
    mask[pos] = True
    for a, s in zip(a_d, s_d):
        assert torch.equal(a.cpu()[mask], a_ref.view(torch.uint8).cpu()[mask])
        assert not a.cpu()[~mask].any()
        assert torch.equal(s.cpu()[:, mask], s_ref.cpu()[:, mask])


@pytest.mark.parametrize("T,k,E,world,rank", [(512, 2, 8, 8, 3), (256, 8, 128, 4, 0), (1000, 2, 8, 5, 4)])
def test_block_order(T, k, E, world, rank):
    from td_benchmark_b200 import _lib

    ids = _route(T, k, E, T + world).to(DEV)
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids, 128, E)
    Tl = (T + world - 1) // world
    order = torch.full((eids.numel(),), -7, dtype=torch.int32, device=DEV)
    status = ops.new_status(DEV)
    _lib.call("b2m_block_order", sorted_ids.data_ptr(), ntpp.data_ptr(), T * k, k, Tl, world, rank, order.data_ptr(),
              order.numel(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ops.check_status(status)
    nblk = int(ntpp.item()) // 128
    srt = sorted_ids.cpu().numpy()[:nblk * 128].reshape(nblk, 128)
    keys = []
    for b in range(nblk):
        v = srt[b][srt[b] < T * k]
        keys.append(int((((v // k) // Tl - rank) % world).max()) if v.size else 0)
    want = sorted(range(nblk), key=lambda b: (keys[b], b))
    assert order.cpu().tolist()[:nblk] == want


@pytest.mark.parametrize("world,rank", [(2, 1), (8, 5)])
def test_gemm1_wait_matches_gemm1(world, rank):
    """The gate/up GEMM in block order with its source waits satisfied equals b2m_gemm1."""
    from td_benchmark_b200 import _lib

    T, H, I, E, k = 512, 512, 256, 8, 2
    x, w1q, w1s, w2q, w2s, ids, wts = _gemm_problem(T, H, I, E, k, 99 + world, False)
    xq, xs = ops.quant_g128(x.to(DEV))
    w1i, w1is = ops.w1_interleave(w1q.to(DEV), w1s.to(DEV))
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids.to(DEV), 128, E, pair_pos=pp)
    rows_cap = eids.numel() * 128
    a_sorted = torch.zeros((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    a_st = torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.dispatch_rows(xq, xs, pp, k, a_sorted, a_st)
    status = ops.new_status(DEV)
    hq, hst = ops.gemm1(a_sorted, a_st, w1i, w1is, eids, ntpp, status=status)
    order = torch.empty(eids.numel(), dtype=torch.int32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    Tl = T // world
    _lib.call("b2m_block_order", sorted_ids.data_ptr(), ntpp.data_ptr(), T * k, k, Tl, world, rank, order.data_ptr(),
              order.numel(), status.data_ptr(), st)
    flags = torch.full((world,), 9, dtype=torch.int32, device=DEV)
    hq2 = torch.zeros_like(hq)
    hst2 = torch.zeros_like(hst)
    _lib.call("b2m_gemm1_wait", a_sorted.data_ptr(), a_st.data_ptr(), rows_cap, H, w1i.data_ptr(), w1is.data_ptr(), E,
              I, eids.data_ptr(), ntpp.data_ptr(), order.data_ptr(), sorted_ids.data_ptr(), T * k, k, Tl,
              flags.data_ptr(), 9, None, 0, None, None, None, None, 0, 0, hq2.data_ptr(), hst2.data_ptr(),
              status.data_ptr(), st)
    torch.cuda.synchronize()
    ops.check_status(status)
    n = int(ntpp.item())
    assert torch.equal(hq2.view(torch.uint8)[:n].cpu(), hq.view(torch.uint8)[:n].cpu())
    assert torch.equal(hst2[:, :n].cpu(), hst[:, :n].cpu())


@pytest.mark.parametrize("world,rank", [(2, 0), (4, 2)])
def test_gemm1_pushes_own_rows_to_peers(world, rank):
    """The gate/up GEMM's pusher warps (peers emulated by buffers on this GPU, their waits
    already satisfied): every peer gets exactly this rank's pair rows and scales, the flag of
    every peer is published, counters are re-armed, and the GEMM output is unchanged."""
    from td_benchmark_b200 import _lib
    from td_benchmark_b200.symm import ptr_array

    T, H, I, E, k = 512, 1024, 256, 8, 2
    x, w1q, w1s, w2q, w2s, ids, wts = _gemm_problem(T, H, I, E, k, 7 * world + rank, False)
    xq, xs = ops.quant_g128(x.to(DEV))
    w1i, w1is = ops.w1_interleave(w1q.to(DEV), w1s.to(DEV))
    pp = torch.empty(T * k, dtype=torch.int32, device=DEV)
    sorted_ids, eids, ntpp = ops.moe_align_block_size(ids.to(DEV), 128, E, pair_pos=pp)
    rows_cap = eids.numel() * 128
    a_sorted = torch.zeros((rows_cap, H), dtype=torch.float8_e4m3fn, device=DEV)
    a_st = torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV)
    ops.dispatch_rows(xq, xs, pp, k, a_sorted, a_st)
    status = ops.new_status(DEV)
    hq, hst = ops.gemm1(a_sorted, a_st, w1i, w1is, eids, ntpp, status=status)
    st = torch.cuda.current_stream().cuda_stream
    Tl = T // world
    order = torch.empty(eids.numel(), dtype=torch.int32, device=DEV)
    _lib.call("b2m_block_order", sorted_ids.data_ptr(), ntpp.data_ptr(), T * k, k, Tl, world, rank, order.data_ptr(),
              order.numel(), status.data_ptr(), st)
    wait_flags = torch.full((world,), 4, dtype=torch.int32, device=DEV)
    peers_a = [a_sorted.view(torch.uint8) if d == rank else torch.zeros((rows_cap, H), dtype=torch.uint8, device=DEV)
               for d in range(world)]
    peers_s = [a_st if d == rank else torch.zeros((H // 128, rows_cap), dtype=torch.float32, device=DEV)
               for d in range(world)]
    push_flags = torch.zeros(world, dtype=torch.int32, device=DEV)
    counters = torch.zeros(world, dtype=torch.int32, device=DEV)
    own_pos = pp[rank * Tl * k:(rank + 1) * Tl * k].contiguous()
    hq2, hst2 = torch.zeros_like(hq), torch.zeros_like(hst)
    for _ in range(2):                              # second call: counters re-armed by the first
        _lib.call("b2m_gemm1_wait", a_sorted.data_ptr(), a_st.data_ptr(), rows_cap, H, w1i.data_ptr(),
                  w1is.data_ptr(), E, I, eids.data_ptr(), ntpp.data_ptr(), order.data_ptr(), sorted_ids.data_ptr(),
                  T * k, k, Tl, wait_flags.data_ptr(), 4, own_pos.data_ptr(), Tl * k,
                  ptr_array([a.data_ptr() for a in peers_a]), ptr_array([s.data_ptr() for s in peers_s]),
                  ptr_array([push_flags.data_ptr() + 4 * d for d in range(world)]), counters.data_ptr(), world, rank,
                  hq2.data_ptr(), hst2.data_ptr(), status.data_ptr(), st)
        torch.cuda.synchronize()
        ops.check_status(status)
        assert not counters.any()
    want_flags = [0 if d == rank else 4 for d in range(world)]
    assert push_flags.tolist() == want_flags
    n = int(ntpp.item())
    assert torch.equal(hq2.view(torch.uint8)[:n].cpu(), hq.view(torch.uint8)[:n].cpu())
    assert torch.equal(hst2[:, :n].cpu(), hst[:, :n].cpu())
    pos = own_pos.long().cpu()
    pos = pos[pos >= 0]
    mask = torch.zeros(rows_cap, dtype=torch.bool)
    mask[pos] = True
    for d in range(world):
        if d == rank:
            continue
        assert torch.equal(peers_a[d].cpu()[mask], a_sorted.view(torch.uint8).cpu()[mask])
        assert not peers_a[d].cpu()[~mask].any()
        assert torch.equal(peers_s[d].cpu()[:, mask], a_st.cpu()[:, mask])


# ---------------------------------------------------------------- reduce-scatter push + owner reduce
@pytest.mark.parametrize("payload,sparse,world,k,H,shared,ep,perm", [
    ("fp8", False, 2, 2, 256, False, False, False), ("fp8", False, 4, 8, 384, True, False, False),
    ("fp8", False, 4, 2, 1024, False, True, False), ("fp8", False, 8, 1, 128, False, False, False),
    ("fp8", True, 4, 2, 1024, False, True, False), ("fp8", True, 8, 8, 256, False, True, True),
    ("bf16", False, 4, 8, 384, True, False, False), ("bf16", True, 4, 2, 512, False, True, False),
    ("bf16", True, 8, 8, 256, False, True, True), ("bf16", True, 4, 8, 256, False, True, True)])
def test_reduce_scatter_emulated_bit_exact(payload, sparse, world, k, H, shared, ep, perm):
    """Every source rank pushes its partials (bf16, or FP8 codes + scales: the b3 payload) to
    the owners, then every owner sums its slots in rank order: all ranks emulated on one GPU,
    each with its own buffers; pushed slots, flags and outputs bit-exact against the oracle.
    Sparse (expert parallel): a token's partial goes only from ranks holding one of its
    experts, and the owner reads only those slots -- the others are prefilled with NaN here,
    so reading one would show.  ``perm``: experts spread over the ranks by a permutation
    (an arbitrary placement through the owner table) instead of contiguous ranges."""
    from oracle import rs as ors
    from td_benchmark_b200 import _lib
    from td_benchmark_b200.symm import ptr_array

    Tl = 24
    T = world * Tl
    E = 16
    epr = E // world
    st = [_bf16((T * k, H), 50 + r, 0.5) for r in range(world)]
    sh = [_bf16((T, H), 70 + r) if shared else None for r in range(world)]
    ids = torch.stack([torch.randperm(E, generator=torch.Generator().manual_seed(900 + t))[:k] for t in range(T)])
    ids = ids.to(torch.int32).contiguous()
    order = torch.randperm(E, generator=torch.Generator().manual_seed(11)) if perm else torch.arange(E)
    owner = torch.empty(E, dtype=torch.int32)
    emaps = []
    for r in range(world):
        mine = torch.sort(order[r * epr:(r + 1) * epr]).values
        owner[mine] = r
        m = torch.full((E,), -1, dtype=torch.int32)
        m[mine] = torch.arange(epr, dtype=torch.int32)
        emaps.append(m)
    owner_d = owner.to(DEV)
    fp8 = payload == "fp8"
    if fp8:
        slots = [torch.full((T, H), 0x7F, dtype=torch.uint8, device=DEV) for _ in range(world)]   # NaN codes
        scales = [torch.full((T, H // 128), float("nan"), dtype=torch.float32, device=DEV) for _ in range(world)]
    else:
        slots = [torch.full((T, H), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=DEV) for _ in range(world)]
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    ids_d = ids.to(DEV)
    for r in range(world):
        sd, shd, em = st[r].to(DEV), None if sh[r] is None else sh[r].to(DEV), emaps[r].to(DEV)
        fl = ptr_array([f.data_ptr() + 4 * r for f in flags])
        idp, emp, shp = ids_d.data_ptr() if ep else None, em.data_ptr() if ep else None, \
            None if shd is None else shd.data_ptr()
        if fp8:
            _lib.call("b2m_combine_push_fp8", sd.data_ptr(), T, k, H, idp, emp, shp, world, r,
                      ptr_array([c.data_ptr() for c in slots]), ptr_array([s.data_ptr() for s in scales]), fl, 7,
                      counter.data_ptr(), int(sparse), stream)
        else:
            _lib.call("b2m_combine_push", sd.data_ptr(), T, k, H, 0, H, idp, emp, shp, world, r,
                      ptr_array([c.data_ptr() for c in slots]), fl, 7, counter.data_ptr(), 0, int(sparse), stream)
        torch.cuda.synchronize(DEV)
    outs = []
    status = ops.new_status(DEV)
    for o in range(world):
        out = torch.empty((Tl, H), dtype=torch.bfloat16, device=DEV)
        own_ids = ids_d[o * Tl:(o + 1) * Tl].contiguous()
        sp = (own_ids.data_ptr(), k, owner_d.data_ptr(), E) if sparse else (None, 0, None, 0)
        if fp8:
            _lib.call("b2m_rs_reduce_fp8", slots[o].data_ptr(), scales[o].data_ptr(), Tl, H, world,
                      flags[o].data_ptr(), 7, None, out.data_ptr(), *sp, status.data_ptr(), stream)
        else:
            _lib.call("b2m_rs_reduce", slots[o].data_ptr(), Tl, H, world, 1, flags[o].data_ptr(), 7, None,
                      out.data_ptr(), *sp, status.data_ptr(), stream)
        outs.append(out)
    torch.cuda.synchronize(DEV)
    assert int(status.item()) == 0 and int(counter.item()) == 0
    assert all(torch.equal(f.cpu(), torch.full((world,), 7, dtype=torch.int32)) for f in flags)
    # oracle: each source's combined partials; with sparse, only the rows it holds a pair of
    parts = []
    sent = []
    for r in range(world):
        mask = (emaps[r][ids.long()] >= 0).numpy() if ep else None
        parts.append(ors.combine_rows(st[r].float().numpy(), k, None if sh[r] is None else sh[r].float().numpy(),
                                      mask))
        sent.append(mask.any(1) if (sparse and mask is not None) else np.ones(T, bool))
    for o in range(world):
        rows_o = slice(o * Tl, (o + 1) * Tl)
        if fp8:
            qs = [ors.rs_fp8_push(parts[r][rows_o]) for r in range(world)]
            got_q, got_s = slots[o].cpu().numpy(), scales[o].cpu().numpy()
            for r in range(world):
                m = sent[r][rows_o]
                assert np.array_equal(got_q[r * Tl:(r + 1) * Tl][m], qs[r][0][m])
                assert np.array_equal(got_s[r * Tl:(r + 1) * Tl][m], qs[r][1][m])
                assert sparse or m.all()
            exp = ors.rs_fp8_reduce(np.stack([q[0] for q in qs]), np.stack([q[1] for q in qs]))
        else:
            got = slots[o].view(torch.int16).cpu().numpy().astype(np.uint16)
            for r in range(world):
                m = sent[r][rows_o]
                assert np.array_equal(got[r * Tl:(r + 1) * Tl][m], parts[r][rows_o][m])
            acc = np.zeros((Tl, H), np.float32)
            for r in range(world):
                acc = (acc + ofp8.bf16_bits_to_f32(parts[r][rows_o])).astype(np.float32)
            exp = ofp8.f32_to_bf16_bits(acc)
        assert np.array_equal(outs[o].view(torch.int16).cpu().numpy().astype(np.uint16), exp)
