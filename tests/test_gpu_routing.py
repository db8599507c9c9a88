"""On-device routing (``b2m_route_topk`` + ``Router``) against the reference's routing.

The committed fixture ``tests/golden/routing.npz`` holds the reference's own
``build_routing`` output (uniform and Zipf-1.2, top-8 of 64 experts) for given hidden
states and gate weights.  Given the same fp32 logits (the gate product computed on the
host as the reference did), the kernel's expert ids must be identical and its weights
equal to within a few fp32 ulps (the softmax and renormalisation sums are accumulated in
a different order from torch's).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from td_benchmark_b200 import configs, data, ops, verify  # noqa: E402
from td_benchmark_b200.routing import Router, log_prior  # noqa: E402

DEV = torch.device("cuda", 0)
W_RTOL = 1e-6   # ~8 fp32 ulps: softmax and renormalisation sums in another order


@pytest.mark.parametrize("kind", ["uniform", "zipf"])
def test_route_kernel_matches_reference_fixture(golden_dir, kind):
    d = np.load(golden_dir / "routing.npz")
    hid = torch.from_numpy(d["hidden_bits"]).view(torch.bfloat16)
    gate = torch.from_numpy(d["gate_bits"]).view(torch.bfloat16)
    logits = (hid.float() @ gate.float().T).contiguous()          # the reference's fp32 product, on the host
    cfg = configs.RoutingCfg() if kind == "uniform" else configs.RoutingCfg(imbalance_kind="zipf", zipf_s=1.2,
                                                                             gate_seed=42)
    ids, w = ops.route_topk(logits.to(DEV), 8, log_prior(cfg, 64, DEV))
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), d[f"ids_{kind}"])
    np.testing.assert_allclose(w.cpu().numpy(), d[f"w_{kind}"], rtol=W_RTOL, atol=0)


@pytest.mark.parametrize("T,E,k,zipf", [(8192, 256, 8, True), (4096, 8, 2, False), (333, 128, 8, False),
                                        (64, 1000, 4, False), (17, 32, 32, False)])
def test_route_kernel_matches_torch(T, E, k, zipf):
    g = torch.Generator(device=DEV).manual_seed(T + E)
    logits = torch.randn((T, E), device=DEV, generator=g)
    cfg = configs.RoutingCfg(imbalance_kind="zipf") if zipf else configs.RoutingCfg()
    bias = log_prior(cfg, E, DEV)
    ids, w = ops.route_topk(logits, k, bias)
    ref_ids, ref_w = data.route(logits, k, cfg)
    torch.cuda.synchronize()
    assert torch.equal(ids, ref_ids)
    torch.testing.assert_close(w, ref_w, rtol=W_RTOL, atol=0)
    assert torch.allclose(w.sum(-1), torch.ones(T, device=DEV), atol=1e-6)


def test_router_feeds_the_layer():
    """Gate GEMM + routing kernel on the device, then the layer: same ids as the host-side
    route of the same product, and the layer output passes the golden gates on that routing."""
    from td_benchmark_b200.context import DistContext
    from td_benchmark_b200.schemes import REGISTRY
    from td_benchmark_b200.schemes.b200 import build_layer

    cfg = configs.preset("dsv3", M=1024)
    b = data.build_bundle(cfg, device=DEV)
    gate = (torch.randn((cfg.shape.E, cfg.shape.K), generator=torch.Generator().manual_seed(3)) * 0.01).to(DEV)
    router = Router(gate, 1024, cfg.shape.top_k, log_prior(cfg.routing, cfg.shape.E, DEV), device=DEV)
    x = b.hidden_local
    ids, w = router(x)
    # the gate product is the fp32 GEMM of the reference (another cuBLAS call may sum in another
    # order, so compare it loosely); the routing of that product is compared tightly
    torch.testing.assert_close(router.logits, x.float() @ gate.float().T, rtol=1e-5, atol=1e-5)
    ref_ids, ref_w = data.route(router.logits, cfg.shape.top_k, cfg.routing)
    torch.cuda.synchronize()
    assert torch.equal(ids, ref_ids)
    torch.testing.assert_close(w, ref_w, rtol=W_RTOL, atol=0)
    layer, _ = build_layer(REGISTRY["d2"][0], cfg, DistContext(device=DEV), b)
    out = layer.forward(x, ids, w)
    torch.cuda.synchronize()
    layer.check()
    rep = verify.check_layer(out, b.hidden_full, ids, w, b.ckpt)
    assert rep["pass"], rep
    layer.close()


def test_route_rejects_bad_shapes():
    with pytest.raises(Exception, match="top_k"):
        ops.route_topk(torch.zeros((4, 8), device=DEV), 9)
    with pytest.raises(Exception, match="E"):
        ops.route_topk(torch.zeros((4, 2000), device=DEV), 8)
