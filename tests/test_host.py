"""Host-side logic on CPU: weight prep, routing, configs, scheme plumbing."""
import numpy as np
import pytest
import torch

from oracle import quant as oquant
from td_benchmark_b200 import configs, data, weights
from td_benchmark_b200.schemes import REGISTRY, SchemeConfigError, build_scheme
from td_benchmark_b200.schemes.base import SchemeCfg, SchemeSpec, TunableSpec, make_lazy_instance, validate_tunables


def test_torch_block_quant_matches_oracle():
    w = torch.randn((3, 384, 256), generator=torch.Generator().manual_seed(0)) * 0.02
    w[0, :128, :128] = 0
    q, s = weights.quantize_block128(w)
    q2, s2 = oquant.quant_block128(w.numpy())
    assert np.array_equal(q.view(torch.uint8).numpy(), q2)
    assert np.array_equal(s.numpy(), s2)
    deq = weights.dequantize_block128(q, s)
    assert np.array_equal(deq.float().numpy(), oquant.dequant_block128(q2, s2))


def test_route_matches_reference_fixture(golden_dir):
    d = np.load(golden_dir / "routing.npz")
    hid = torch.from_numpy(d["hidden_bits"]).view(torch.bfloat16)
    gate = torch.from_numpy(d["gate_bits"]).view(torch.bfloat16)
    logits = hid.float() @ gate.float().T
    ids, w = data.route(logits, 8, configs.RoutingCfg())
    assert np.array_equal(ids.numpy(), d["ids_uniform"]) and np.array_equal(w.numpy(), d["w_uniform"])
    ids, w = data.route(logits, 8, configs.RoutingCfg(imbalance_kind="zipf", zipf_s=1.2, gate_seed=42))
    assert np.array_equal(ids.numpy(), d["ids_zipf"]) and np.array_equal(w.numpy(), d["w_zipf"])


def test_bundle_deterministic_and_rank_sliced():
    cfg = configs.preset("tiny")
    b0 = data.build_bundle(cfg, rank=0, world_size=2)
    b1 = data.build_bundle(cfg, rank=1, world_size=2)
    full = data.build_bundle(cfg, rank=0, world_size=1)
    assert torch.equal(torch.cat([b0.hidden_local, b1.hidden_local]), full.hidden_local)
    assert torch.equal(b0.routing.topk_ids_full, full.routing.topk_ids_full)
    assert torch.equal(b1.ckpt.w1.fp8.view(torch.uint8), full.ckpt.w1.fp8.view(torch.uint8))
    assert full.routing.topk_ids_full.dtype == torch.int32
    assert torch.allclose(full.routing.topk_weights_full.sum(-1), torch.ones(64))


def test_zipf_routing_is_skewed():
    cfg = configs.preset("dsv3", M=2048)
    b = data.build_bundle(cfg, with_weights=False)
    counts = torch.bincount(b.routing.topk_ids_full.flatten().long(), minlength=256).float()
    assert counts.max() / counts.mean() > 5


def test_presets_and_validation():
    assert configs.PRESETS["mixtral"].shape.intermediate_per_tp(8) == 1792
    assert configs.PRESETS["dsv3"].shape.local_E(8) == 32
    with pytest.raises(configs.ConfigError, match="violates constraint"):
        configs.ShapeCfg(M=8, K=100, E=4, top_k=2, n_gateup=256, n_down=128)
    with pytest.raises(configs.ConfigError):
        configs.preset("nope")
    assert configs.preset("qwen3", M=32).shape.M == 32


def _full_weights(E=4, I=256, H=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    w1q, w1s = weights.quantize_block128(torch.randn((E, 2 * I, H), generator=g) * 0.02)
    w2q, w2s = weights.quantize_block128(torch.randn((E, H, I), generator=g) * 0.02)
    return w1q, w1s, w2q, w2s


def test_tp_views_aligned_slices_codes():
    w1q, w1s, w2q, w2s = _full_weights(I=512)
    v = weights.tp_views(w1q, w1s, w2q, w2s, rank=1, world_size=2)
    assert v["shard_level"] == "L0" and v["inter"] == 256
    assert torch.equal(v["w1"][:, :256].view(torch.uint8), w1q[:, 256:512].view(torch.uint8))
    assert torch.equal(v["w1"][:, 256:].view(torch.uint8), w1q[:, 768:].view(torch.uint8))
    assert torch.equal(v["w2"].view(torch.uint8), w2q[:, :, 256:].view(torch.uint8))
    assert v["w1_scale"].shape == (4, 4, 2) and v["w2_scale"].shape == (4, 2, 2)


def test_tp_views_ragged_pads_to_128():
    # Qwen3 at TP=8: I/P = 96 -> zero padded to 128 ("L2", runtime.py:46-55)
    w1q, w1s, w2q, w2s = _full_weights(E=2, I=768, H=256)
    v = weights.tp_views(w1q, w1s, w2q, w2s, rank=3, world_size=8)
    assert v["shard_level"] == "L2" and v["inter"] == 128
    assert v["w1"].shape == (2, 256, 256) and v["w2"].shape == (2, 256, 128)
    assert v["w1"][:, 96:128].float().abs().sum() == 0 and v["w2"][:, :, 96:].float().abs().sum() == 0


def test_ep_views_expert_map():
    w1q, w1s, w2q, w2s = _full_weights(E=8)
    v = weights.ep_views(w1q, w1s, w2q, w2s, rank=2, world_size=4)
    assert v["expert_map"].tolist() == [-1, -1, -1, -1, 0, 1, -1, -1]
    assert torch.equal(v["w1"].view(torch.uint8), w1q[4:6].view(torch.uint8))


def test_scheme_registry_and_tunables():
    assert {"d1", "d2"} <= set(REGISTRY)
    spec, _ = REGISTRY["d1"]
    assert spec.weight_dtype == "fp8" and spec.act_quant == "group128" and not spec.requires_nvshmem
    assert validate_tunables(spec, {}) == {"check_status": False, "rs_dtype": "bf16"}
    with pytest.raises(SchemeConfigError, match="violate schema"):
        validate_tunables(spec, {"nope": 1})
    with pytest.raises(SchemeConfigError, match="expected bool"):
        validate_tunables(spec, {"check_status": 1})
    with pytest.raises(SchemeConfigError, match="not registered"):
        build_scheme(None, None, None, SchemeCfg("zz", {}))
    with pytest.raises(RuntimeError, match="requires a DataBundle"):
        build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d1", {}))


def test_p2p_exchange_tunables():
    spec, _ = REGISTRY["d3"]
    assert validate_tunables(spec, {}) == {"check_status": False, "rs_dtype": "bf16", "ag_mode": "auto", "rs_mode": "auto",
                                           "rs_chunks": 4}
    with pytest.raises(SchemeConfigError, match="violate schema"):
        validate_tunables(REGISTRY["d1"][0], {"ag_mode": "ce"})   # NCCL schemes have no exchange knobs
    with pytest.raises(SchemeConfigError, match="one of"):
        build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d4", {"ag_mode": "dma"}))
    with pytest.raises(SchemeConfigError, match="1..8"):
        build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d3", {"rs_chunks": 9}))
    with pytest.raises(SchemeConfigError, match="rs_dtype"):
        build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d3", {"rs_dtype": "fp8", "rs_mode": "gemm"}))
    with pytest.raises(SchemeConfigError, match="one of"):
        build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d1", {"rs_dtype": "fp16"}))
    for ok in ({"ag_mode": "push"}, {"ag_mode": "ce", "rs_mode": "gemm"}, {"rs_mode": "ce", "rs_chunks": 8},
               {"rs_dtype": "fp8"}):
        with pytest.raises(RuntimeError, match="requires a DataBundle"):   # accepted; fails later for lack of data
            build_scheme(configs.preset("tiny"), None, None, SchemeCfg("d3", ok))


def test_p2p_exchange_rejects_unknown_modes():
    import torch.distributed as dist
    from td_benchmark_b200.layer import P2PExchange

    own = not dist.is_initialized()
    if own:
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:0", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="rs_mode"):
            P2PExchange(rs_mode="dma")
        with pytest.raises(ValueError, match="ag_mode"):
            P2PExchange(ag_mode="ring")
        ex = P2PExchange(ag_mode="push", rs_mode="gemm")
        assert ex.world_size == 1 and ex.chunks_req == 1 and ex.extra_launches() == 0
    finally:
        if own:
            dist.destroy_process_group()


def test_int_tunable_rejects_bool():
    spec = SchemeSpec("x", "x", "f", "TP", "c", "fp8", "group128", False, {"n": TunableSpec(int, 2, "d")})
    with pytest.raises(SchemeConfigError):
        validate_tunables(spec, {"n": True})
    inst = make_lazy_instance(spec, {"n": 2}, lambda: 7)
    assert inst.run() == 7 and inst.run_staged().output == 7 and inst.diagnostics["scheme"] == "x"


def test_balanced_placement_evens_routed_pairs():
    from td_benchmark_b200 import weights
    cfg = configs.preset("dsv3")
    b = data.build_bundle(cfg, device="cpu", with_weights=False)
    ids = b.routing.topk_ids_full
    E, P = cfg.shape.E, 8
    pl = weights.balanced_placement(ids, E, P)
    assert sorted(e for es in pl for e in es) == list(range(E)) and all(len(es) == E // P for es in pl)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    per_rank = [int(counts[es].sum()) for es in pl]
    contiguous = [int(counts[r * E // P:(r + 1) * E // P].sum()) for r in range(P)]
    mean = ids.numel() / P
    assert max(per_rank) <= 1.05 * mean < max(contiguous)      # Zipf routing: contiguous is skewed
    assert weights.balanced_placement(ids, E, P) == pl            # deterministic
    owner = weights.expert_owner(pl)
    assert all(int(owner[e]) == r for r, es in enumerate(pl) for e in es)


def test_ep_views_with_a_placement_gather_the_rank_experts():
    from td_benchmark_b200 import weights
    E = 8
    w1 = torch.arange(E * 256 * 128, dtype=torch.float32).view(E, 256, 128).to(torch.float8_e4m3fn)
    s1 = torch.arange(E * 2, dtype=torch.float32).view(E, 2, 1)
    w2 = torch.zeros((E, 128, 128), dtype=torch.float8_e4m3fn)
    s2 = torch.arange(E, dtype=torch.float32).view(E, 1, 1)
    pl = [[1, 6], [0, 7], [2, 5], [3, 4]]
    v = weights.ep_views(w1, s1, w2, s2, 2, 4, placement=pl)
    assert torch.equal(v["w1_scale"], s1[[2, 5]]) and torch.equal(v["w2_scale"], s2[[2, 5]])
    assert v["expert_map"].tolist() == [-1, -1, 0, -1, -1, 1, -1, -1]
    assert v["expert_owner"].tolist() == [1, 0, 2, 3, 3, 2, 0, 1]
    c = weights.ep_views(w1, s1, w2, s2, 1, 4)
    assert torch.equal(c["w1_scale"], s1[2:4]) and c["expert_owner"].tolist() == [0, 0, 1, 1, 2, 2, 3, 3]


def test_sweep_and_peaks_modules_parse_their_arguments():
    """The user-facing measurement modules start and print their usage without a GPU."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    for mod in ("td_benchmark_b200.sweep", "td_benchmark_b200.peaks"):
        res = subprocess.run([sys.executable, "-m", mod, "--help"], capture_output=True, text=True, cwd=root)
        assert res.returncode == 0 and "usage" in res.stdout, (mod, res.stderr[-500:])


def test_sweep_variant_table():
    import torch.distributed as dist
    from td_benchmark_b200 import sweep
    from td_benchmark_b200.context import DistContext

    own = not dist.is_initialized()
    if own:
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:0", rank=0, world_size=1)
    try:
        ctx = DistContext()
        assert sweep._exchange("nccl", ctx).name == "nccl"
        ex = sweep._exchange("ce4", ctx)
        assert ex.rs_mode == "ce" and ex.chunks_req == 4
        assert sweep._exchange("sm", ctx).rs_mode == "sm" and sweep._exchange("fused", ctx).rs_mode == "auto"
        assert sweep._exchange("sparse", ctx).sparse and sweep._exchange("fp8rs", ctx).rs_mode == "fp8"
        with pytest.raises(ValueError):
            sweep._exchange("ring", ctx)
    finally:
        if own:
            dist.destroy_process_group()


def test_auto_reduce_scatter_choice():
    """rs_mode='auto' follows the measured break-even: DeepSeek-V3 (top-8) EP2 takes the down GEMM's
    stores at 4096 local tokens but SM stores at 1024 and 256; EP4/EP8 (pair rows <= 2x the
    partials) and Mixtral TP (top-2) take them at any size; a TP shared expert never does."""
    from td_benchmark_b200.layer import P2PExchange as X
    assert X.auto_rs_mode(True, 8, 2, 4096, True) == "gemm"
    assert X.auto_rs_mode(True, 8, 2, 1024, True) == "sm"
    assert X.auto_rs_mode(True, 8, 2, 256, False) == "sm"
    assert X.auto_rs_mode(True, 8, 4, 2048, True) == "gemm"
    assert X.auto_rs_mode(True, 8, 8, 64, True) == "gemm"
    assert X.auto_rs_mode(False, 2, 8, 512, False) == "gemm"
    assert X.auto_rs_mode(False, 8, 4, 64, False) == "sm"
    assert X.auto_rs_mode(False, 2, 2, 4096, True) == "sm"
