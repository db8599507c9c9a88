"""The overlap-level plug point (``moe_forward_overlap_fp8ag``) on one B200 against the golden.

Same signature as ``moe_bench/overlap/overlap_forward.py:348-366``: weights in the
reference layout (w1 [E, 2I, H] gate-then-up with 128x128 block scales), full routing,
an optional shared expert given as an object with ``w1_fp8/w1_scale/w2_fp8/w2_scale``
(``moe_bench/schemes/shared_expert.py:15-30``).
"""
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

from td_benchmark_b200 import configs, data, verify  # noqa: E402
from td_benchmark_b200.overlap import MoEOverlapState, moe_forward_overlap_fp8ag  # noqa: E402

DEV = torch.device("cuda", 0)


def _call(state, b, shared=None):
    ck, s = b.ckpt, None
    return moe_forward_overlap_fp8ag(state, b.hidden_local, ck.w1.fp8, ck.w2.fp8, b.routing.topk_weights_full,
                                     b.routing.topk_ids_full, b.routing.topk_ids_full.shape[1], ck.w1.fp8.shape[0],
                                     shared_mlp=shared, w1_scale=ck.w1.scale, w2_scale=ck.w2.scale,
                                     block_shape=[128, 128])


@pytest.mark.parametrize("name,over", [("tiny", {}), ("mixtral", {"M": 512}), ("dsv3", {"M": 512})])
def test_overlap_entry_point_vs_golden(name, over):
    cfg = configs.preset(name, **over)
    b = data.build_bundle(cfg, device=DEV)
    shared = None
    if b.ckpt.shared_w1 is not None:
        shared = SimpleNamespace(w1_fp8=b.ckpt.shared_w1.fp8, w1_scale=b.ckpt.shared_w1.scale,
                                 w2_fp8=b.ckpt.shared_w2.fp8, w2_scale=b.ckpt.shared_w2.scale)
    state = MoEOverlapState()
    out = _call(state, b, shared)
    again = _call(state, b, shared)        # the prepared layer is cached and reused
    torch.cuda.synchronize()
    assert len(state._layers) == 1 and torch.equal(out, again)
    rep = verify.check_layer(out, b.hidden_full, b.routing.topk_ids_full, b.routing.topk_weights_full, b.ckpt)
    assert rep["pass"], rep
    state.release()


def test_overlap_entry_point_rejects_what_the_contract_excludes():
    b = data.build_bundle(configs.preset("tiny"), device=DEV)
    ck = b.ckpt
    args = (MoEOverlapState(), b.hidden_local, ck.w1.fp8, ck.w2.fp8, b.routing.topk_weights_full,
            b.routing.topk_ids_full, 2, 8)
    with pytest.raises(ValueError, match="w1_scale"):
        moe_forward_overlap_fp8ag(*args)
    with pytest.raises(ValueError, match="block_shape"):
        moe_forward_overlap_fp8ag(*args, w1_scale=ck.w1.scale, w2_scale=ck.w2.scale, block_shape=[64, 64])
    with pytest.raises(ValueError, match="exchange"):
        MoEOverlapState(exchange="nvshmem")
