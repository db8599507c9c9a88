"""The on-device verification step (``td_benchmark_b200.verify``) against the numpy oracle, on CPU."""
import numpy as np
import torch

from oracle import golden as ogolden
from oracle import quant as oquant
from td_benchmark_b200 import configs, data, verify


def _tiny():
    cfg = configs.preset("tiny")
    return cfg, data.build_bundle(cfg, device="cpu")


def _oracle(b, act_quant=True):
    ck = b.ckpt
    w1 = oquant.dequant_block128(ck.w1.fp8.view(torch.uint8).numpy(), ck.w1.scale.numpy())
    w2 = oquant.dequant_block128(ck.w2.fp8.view(torch.uint8).numpy(), ck.w2.scale.numpy())
    return ogolden.golden_moe(b.hidden_full.float().numpy(), b.routing.topk_ids_full.numpy(),
                              b.routing.topk_weights_full.numpy(), w1, w2, act_quant=act_quant)


def test_golden_rows_matches_numpy_oracle():
    _, b = _tiny()
    g = verify.golden_rows(b.hidden_full, b.routing.topk_ids_full, b.routing.topk_weights_full, b.ckpt)
    ref = _oracle(b)
    rep = ogolden.compare_outputs(g.numpy(), ref, **ogolden.GATES)
    assert rep["pass"] and rep["cos_sim"] > 0.99999, rep


def test_golden_rows_of_a_slice_equal_the_slice_of_the_full_golden():
    _, b = _tiny()
    ids, wts, h = b.routing.topk_ids_full, b.routing.topk_weights_full, b.hidden_full
    full = verify.golden_rows(h, ids, wts, b.ckpt)
    part = verify.golden_rows(h[16:48], ids[16:48], wts[16:48], b.ckpt)
    assert torch.allclose(part, full[16:48], rtol=1e-5, atol=1e-6)


def test_compare_outputs_agrees_with_the_oracle_metrics():
    rng = np.random.default_rng(3)
    e = rng.standard_normal((64, 256)).astype(np.float32)
    a = e + 0.01 * rng.standard_normal(e.shape).astype(np.float32)
    mine = verify.compare_outputs(torch.from_numpy(a), torch.from_numpy(e), **verify.GATES)
    ref = ogolden.compare_outputs(a, e, **ogolden.GATES)
    for k in ("max_abs", "cos_sim", "rel_p99", "scale"):
        assert abs(mine[k] - ref[k]) <= 1e-9 * max(1.0, abs(ref[k])), (k, mine[k], ref[k])
    assert mine["pass"] == ref["pass"]


def test_check_layer_rejects_a_zero_output_and_accepts_the_golden():
    _, b = _tiny()
    ids, wts, h = b.routing.topk_ids_full, b.routing.topk_weights_full, b.hidden_full
    g = verify.golden_rows(h, ids, wts, b.ckpt)
    assert verify.check_layer(g.to(torch.bfloat16), h, ids, wts, b.ckpt)["pass"]
    bad = verify.check_layer(torch.zeros_like(g), h, ids, wts, b.ckpt)
    assert not bad["pass"] and bad["cos_sim"] == 0.0


def test_rank_partials_sum_to_the_golden_ep_and_tp():
    cfg = configs.preset("tiny", M=64)
    b = data.build_bundle(cfg, device="cpu")
    ids, wts, h = b.routing.topk_ids_full, b.routing.topk_weights_full, b.hidden_full
    g = verify.golden_rows(h, ids, wts, b.ckpt)
    for world, par in ((2, "EP"), (4, "EP"), (2, "TP"), (4, "TP")):
        parts = verify.rank_partials(h, ids, wts, b.ckpt, world, par)
        assert parts.shape == (world, 64, 256)
        assert torch.allclose(parts.sum(0), g, rtol=1e-4, atol=1e-5), (world, par)
        err = verify.rs_fp8_error(parts)
        assert 0.0 < err < 0.1 * float(g.abs().max())
