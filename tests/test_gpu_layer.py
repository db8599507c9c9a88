"""Layer parity on a B200: the full b2m forward against the fp32 golden.

Gates are the reference worker's (cos >= 0.995, masked rel_p99 <= 5.0,
|scale - 1| <= 0.05, ``moe_bench/worker.py:108-110``) plus a max-abs bound:
max |out - golden| <= 1.5 x (max |golden_fp8act - golden_bf16act|), the
calibration rule of ``tests/calibrate_tolerance.py:17-25`` re-run at each shape.
"""
import numpy as np
import pytest
import torch

from oracle import golden as ogolden
from oracle import quant as oquant

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from tests import torch_ref  # noqa: E402
from td_benchmark_b200 import configs, data  # noqa: E402
from td_benchmark_b200.context import DistContext  # noqa: E402
from td_benchmark_b200.layer import ExpertWeights, MoELayer  # noqa: E402
from td_benchmark_b200.schemes import build_scheme  # noqa: E402
from td_benchmark_b200.schemes.base import SchemeCfg  # noqa: E402

DEV = torch.device("cuda", 0)


def _gates(out, ref, calib):
    rep = ogolden.compare_outputs(out, ref, **ogolden.GATES)
    assert rep["pass"], rep
    assert rep["max_abs"] <= 1.5 * calib, (rep["max_abs"], calib)
    return rep


def test_tiny_layer_vs_reference_fixture(golden_dir):
    """The reference's own data bundle and golden output (BASELINE tiny shape + shared expert)."""
    d = np.load(golden_dir / "golden_tiny.npz")
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    fp8 = lambda a: t(a).view(torch.float8_e4m3fn)  # noqa: E731
    w = ExpertWeights.prepare(fp8(d["w1_q"]), t(d["w1_s"]), fp8(d["w2_q"]), t(d["w2_s"]))
    sw = ExpertWeights.prepare(fp8(d["sw1_q"]), t(d["sw1_s"]), fp8(d["sw2_q"]), t(d["sw2_s"]))
    layer = MoELayer(w, 64, 2, 8, shared=sw)
    x = torch.from_numpy(d["hidden"]).to(torch.bfloat16).to(DEV)
    out = layer.forward(x, t(d["topk_ids"]), t(d["topk_weights"]))
    torch.cuda.synchronize()
    layer.check()
    got = out.float().cpu().numpy()
    w1 = oquant.dequant_block128(d["w1_q"], d["w1_s"])
    w2 = oquant.dequant_block128(d["w2_q"], d["w2_s"])
    sw1 = oquant.dequant_block128(d["sw1_q"], d["sw1_s"])
    sw2 = oquant.dequant_block128(d["sw2_q"], d["sw2_s"])
    hb = x.float().cpu().numpy()
    g_fp8 = ogolden.golden_moe(hb, d["topk_ids"], d["topk_weights"], w1, w2, sw1, sw2, act_quant=True)
    g_none = ogolden.golden_moe(hb, d["topk_ids"], d["topk_weights"], w1, w2, sw1, sw2, act_quant=False)
    calib = float(np.abs(g_fp8 - g_none).max())
    _gates(got, d["out_bf16in"], calib)
    # against the reference golden on the unrounded fp32 hidden states, as the worker verifies
    rep = ogolden.compare_outputs(got, d["out"], **ogolden.GATES)
    assert rep["pass"], rep


def _run_scheme(cfg, code="d1"):
    bundle = data.build_bundle(cfg, device=DEV)
    ctx = DistContext(rank=0, world_size=1, local_rank=0, device=DEV)
    inst = build_scheme(cfg, ctx, bundle, SchemeCfg(code, {"check_status": True}))
    out = inst.run()
    out2 = inst.run()                                 # second call reuses every buffer
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    inst.close()
    return bundle, out


def test_tiny_config_vs_numpy_oracle():
    cfg = configs.preset("tiny")
    bundle, out = _run_scheme(cfg)
    ck = bundle.ckpt
    w1 = oquant.dequant_block128(ck.w1.fp8.view(torch.uint8).cpu().numpy(), ck.w1.scale.cpu().numpy())
    w2 = oquant.dequant_block128(ck.w2.fp8.view(torch.uint8).cpu().numpy(), ck.w2.scale.cpu().numpy())
    h = bundle.hidden_full.float().cpu().numpy()
    ids, wts = bundle.routing.topk_ids_full.cpu().numpy(), bundle.routing.topk_weights_full.cpu().numpy()
    g = ogolden.golden_moe(h, ids, wts, w1, w2, act_quant=True)
    gn = ogolden.golden_moe(h, ids, wts, w1, w2, act_quant=False)
    _gates(out.float().cpu().numpy(), g, float(np.abs(g - gn).max()))


@pytest.mark.parametrize("name,over", [
    ("qwen3", {"M": 32}), ("qwen3", {"M": 256}),
    ("mixtral", {"M": 512}),
    ("dsv3", {"M": 512}), ("dsv3", {"M": 2048, "imbalance_kind": "none"}),
])
def test_baseline_shapes_vs_torch_golden(name, over):
    cfg = configs.preset(name, **over)
    bundle, out = _run_scheme(cfg)
    ck = bundle.ckpt
    sw = None
    if ck.shared_w1 is not None:
        sw = (ck.shared_w1.fp8, ck.shared_w1.scale, ck.shared_w2.fp8, ck.shared_w2.scale)
    g, calib = torch_ref.act_quant_error(bundle.hidden_full, bundle.routing.topk_ids_full,
                                         bundle.routing.topk_weights_full, ck.w1.fp8, ck.w1.scale, ck.w2.fp8,
                                         ck.w2.scale, sw)
    _gates(out.float().cpu().numpy(), g.cpu().numpy(), calib)


def test_host_pipeline_matches_direct_forward():
    """Double-buffered host pipeline: each step's pinned-host result equals a direct forward
    of that step's inputs (different inputs per step, slots reused)."""
    from td_benchmark_b200.pipeline import HostPipeline
    from td_benchmark_b200.schemes import REGISTRY
    from td_benchmark_b200.schemes.b200 import build_layer

    cfg = configs.preset("mixtral", M=256)
    bundle = data.build_bundle(cfg, device=DEV)
    ctx = DistContext(rank=0, world_size=1, local_rank=0, device=DEV)
    layer, _ = build_layer(REGISTRY["d1"][0], cfg, ctx, bundle)
    ids = bundle.routing.topk_ids_full.contiguous()
    wts = bundle.routing.topk_weights_full.contiguous()
    xs = [(bundle.hidden_local * (1.0 + 0.25 * i)).to(torch.bfloat16).contiguous() for i in range(5)]
    want = [layer.forward(x, ids, wts).clone() for x in xs]
    torch.cuda.synchronize()
    pipe = HostPipeline(layer)
    outs = [torch.empty(want[0].shape, dtype=torch.bfloat16).pin_memory() for _ in xs]
    for x, o in zip(xs, outs):
        pipe.submit(x.cpu().pin_memory(), ids.cpu().pin_memory(), wts.cpu().pin_memory(), o)
    pipe.drain()
    layer.check()
    for w, o in zip(want, outs):
        assert torch.equal(w.cpu(), o)
    # whole-tensor copies (chunk_bytes=0) and traced steps give the same results
    for kw in ({"chunk_bytes": 0}, {"trace": True, "chunk_bytes": 64 << 10}):
        pipe2 = HostPipeline(layer, **kw)
        outs2 = [torch.empty(want[0].shape, dtype=torch.bfloat16).pin_memory() for _ in xs]
        for x, o in zip(xs, outs2):
            pipe2.submit(x.cpu().pin_memory(), ids.cpu().pin_memory(), wts.cpu().pin_memory(), o)
        pipe2.drain()
        assert all(torch.equal(w.cpu(), o) for w, o in zip(want, outs2))
        if kw.get("trace"):
            sp = pipe2.spans()
            assert sp["steps"] == len(xs) and sp["forward_ms"] > 0 and sp["h2d_ms"] > 0 and sp["d2h_ms"] > 0
    out_dev = torch.empty_like(want[0])
    assert layer.forward(xs[2], ids, wts, out=out_dev) is out_dev and torch.equal(out_dev, want[2])
    with pytest.raises(ValueError):
        layer.forward(xs[0], ids, wts, out=torch.empty(3, dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("name", ["mixtral", "dsv3"])
def test_benchmarked_full_shapes_vs_golden(name):
    """The shapes bench.py times at N=1: Mixtral T=4096 (TP1) and DeepSeek-V3 T=8192 with Zipf
    routing and the shared expert (EP1), against the device fp32 golden of the package's
    verification step (the worker's gates + max-abs <= 1.5 x calibrated act-quant error)."""
    from td_benchmark_b200 import verify

    cfg = configs.preset(name)
    bundle, out = _run_scheme(cfg, "d2" if cfg.parallel == "EP" else "d1")
    rep = verify.check_layer(out, bundle.hidden_full, bundle.routing.topk_ids_full, bundle.routing.topk_weights_full,
                             bundle.ckpt)
    assert rep["pass"], rep
