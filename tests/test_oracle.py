"""The CPU oracle against the reference's own outputs (fixtures from tests/golden/make_golden.py)."""
import numpy as np
import pytest

from oracle import align as oalign
from oracle import fp8, golden, quant


def _load(golden_dir, name):
    return np.load(golden_dir / name)


def test_fp8_encode_matches_torch_cast(golden_dir):
    d = _load(golden_dir, "fp8_cast.npz")
    codes = fp8.encode_e4m3(d["x"])
    mism = np.nonzero(codes != d["codes"])[0]
    assert mism.size == 0, f"{mism.size} mismatches, first x={d['x'][mism[:5]]}"


def test_fp8_decode_roundtrip_all_codes():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    vals = fp8.decode_e4m3(codes)
    back = fp8.encode_e4m3(vals)
    # -0 and +0 both decode to zero; encode keeps the sign bit
    assert np.array_equal(back, codes)
    assert fp8.decode_e4m3(np.array([0x7E], dtype=np.uint8))[0] == 448.0
    assert fp8.decode_e4m3(np.array([0x01], dtype=np.uint8))[0] == 2.0 ** -9


def test_fp8_encode_rejects_out_of_range():
    with pytest.raises(ValueError):
        fp8.encode_e4m3(np.array([500.0], dtype=np.float32))


def test_quant_block128_bit_exact(golden_dir):
    d = _load(golden_dir, "quant_block128.npz")
    for w, q, s in (("w_a", "q_a", "s_a"), ("w_b", "q_b", "s_b")):
        codes, scale = quant.quant_block128(d[w])
        assert np.array_equal(codes, d[q]), w
        assert np.array_equal(scale, d[s]), w
    assert d["s_a"].shape == (2, 2, 1)
    assert d["s_b"][1, 0, 1] == np.float32(1e-12)


def test_group_quant_dequant_bit_exact(golden_dir):
    d = _load(golden_dir, "group_qdq.npz")
    for x, y in (("x1", "y1"), ("x2", "y2"), ("x3", "y3")):
        got = quant.quant_dequant_g128(d[x])
        assert got.shape == d[y].shape
        assert np.array_equal(got.view(np.uint32), d[y].view(np.uint32)), x


def test_group_quant_small_values_error_bound(golden_dir):
    # tests/test_golden.py:29-35 of the reference: QDQ error < 2e-3 for 0.01-scale inputs
    d = _load(golden_dir, "group_qdq.npz")
    assert np.abs(quant.quant_dequant_g128(d["x1"]) - d["x1"]).max() < 2e-3


def _tiny_weights(d):
    w1 = quant.dequant_block128(d["w1_q"], d["w1_s"])
    w2 = quant.dequant_block128(d["w2_q"], d["w2_s"])
    sw1 = quant.dequant_block128(d["sw1_q"], d["sw1_s"])
    sw2 = quant.dequant_block128(d["sw2_q"], d["sw2_s"])
    return w1, w2, sw1, sw2


def test_dequant_block128_matches_reference_bf16_view(golden_dir):
    d = _load(golden_dir, "golden_tiny.npz")
    w1 = quant.dequant_block128(d["w1_q"], d["w1_s"])
    ref_bits = d["w1_bf16_bits"].astype(np.uint16)
    assert np.array_equal(fp8.f32_to_bf16_bits(w1[:, :8]), ref_bits)


@pytest.mark.parametrize("hidden_key,out_key", [("hidden", "out"), ("hidden_bf16", "out_bf16in")])
def test_golden_moe_matches_reference(golden_dir, hidden_key, out_key):
    d = _load(golden_dir, "golden_tiny.npz")
    w1, w2, sw1, sw2 = _tiny_weights(d)
    hidden = d["hidden"] if hidden_key == "hidden" else fp8.bf16_round(d["hidden"])
    out = golden.golden_moe(hidden, d["topk_ids"], d["topk_weights"], w1, w2, sw1, sw2)
    ref = d[out_key]
    # fp32 matmuls in a different BLAS differ by round-off, which moves a few
    # intermediate FP8 codes across a rounding boundary (one e4m3 ulp each): most
    # elements agree to round-off, the rest by far less than the activation-quant error.
    close = np.isclose(out, ref, rtol=1e-4, atol=1e-6 * np.abs(ref).max())
    assert close.mean() > 0.97, close.mean()
    assert np.abs(out - ref).max() <= 2e-3 * np.abs(ref).max()
    rep = golden.compare_outputs(out, ref, **golden.GATES)
    assert rep["pass"] and rep["cos_sim"] > 0.99999


def test_compare_outputs_gate_sentinels():
    # reference tests/test_verify_gate.py:8-45
    rng = np.random.default_rng(0)
    g = rng.standard_normal((256, 64)).astype(np.float32)
    assert not golden.compare_outputs(np.zeros_like(g), g, cos_threshold=0.99, rel_p99_threshold=0.05)["pass"]
    assert golden.compare_outputs(g * 1.0001, g, cos_threshold=0.999, rel_p99_threshold=0.05)["pass"]
    rep = golden.compare_outputs(g * 0.5, g, cos_threshold=0.99, rel_p99_threshold=5.0, scale_tolerance=0.05)
    assert not rep["pass"] and abs(rep["scale"] - 0.5) < 0.01
    assert golden.compare_outputs(np.ones((8, 8)) * 1.01, np.ones((8, 8)), atol=0.2)["pass"]


# ---------------------------------------------------------------- align
def _align_loop(ids, bs, E, emap=None):
    """Pure-Python restatement of the vLLM contract for small cases (independent of the numpy one)."""
    flat = [int(v) for v in np.asarray(ids).reshape(-1)]
    numel = len(flat)
    cap, nblk = oalign.buffer_sizes(numel, E, bs)
    out, eids = [], []
    for e in range(E):
        seg = [i for i, v in enumerate(flat) if v == e]
        if not seg:
            continue
        padded = -(-len(seg) // bs) * bs
        out += seg + [numel] * (padded - len(seg))
        eids += [e if emap is None else int(emap[e])] * (padded // bs)
    ntpp = len(out)
    out += [numel] * (cap - ntpp)
    eids += [-1] * (nblk - len(eids))
    return np.array(out, np.int32), np.array(eids, np.int32), ntpp


def test_align_docstring_example():
    # vLLM moe_align_block_size.py:57-71 (its ids are 1-based; shifted to 0-based experts 0..3 here)
    ids = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]]) - 1
    s, e, n = oalign.moe_align_block_size(ids, 4, 4)
    assert n[0] == 16
    assert s[:16].tolist() == [3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12]
    assert e[:4].tolist() == [0, 1, 2, 3]
    assert s.size == 12 + 4 * 3 and e.size == 6


@pytest.mark.parametrize("T,k,E,bs,seed", [(64, 2, 8, 16, 0), (3, 2, 8, 4, 1), (100, 8, 64, 128, 2),
                                           (1, 1, 4, 128, 3), (0, 2, 8, 128, 4), (37, 3, 5, 7, 5)])
def test_align_matches_loop_restatement(T, k, E, bs, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32) if T else np.zeros((0, k), np.int32)
    s, e, n = oalign.moe_align_block_size(ids, bs, E)
    s2, e2, n2 = _align_loop(ids, bs, E)
    assert n[0] == n2 and np.array_equal(s, s2) and np.array_equal(e, e2)


def test_align_expert_map_marks_non_local():
    rng = np.random.default_rng(7)
    E = 16
    ids = np.stack([rng.permutation(E)[:4] for _ in range(50)]).astype(np.int32)
    emap = np.full(E, -1, np.int32)
    emap[4:8] = np.arange(4)
    s, e, n = oalign.moe_align_block_size(ids, 8, E, emap)
    s2, e2, n2 = _align_loop(ids, 8, E, emap)
    assert np.array_equal(e, e2) and np.array_equal(s, s2)
    assert set(e[e >= 0].tolist()) <= {0, 1, 2, 3}


def test_threaded_golden_equals_serial_golden():
    """The threaded expert loop (used to time the CPU baseline) computes the same layer."""
    from oracle import golden as og
    rng = np.random.default_rng(5)
    T, H, I, E, k = 48, 256, 256, 6, 2
    h = rng.standard_normal((T, H)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    w1 = (0.05 * rng.standard_normal((E, 2 * I, H))).astype(np.float32)
    w2 = (0.05 * rng.standard_normal((E, H, I))).astype(np.float32)
    a = og.golden_moe(h, ids, w, w1, w2)
    b = og.golden_moe_threads(h, ids, w, w1, w2, workers=4)
    np.testing.assert_allclose(b, a, rtol=1e-5, atol=1e-6)
