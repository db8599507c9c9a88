"""Cross-check of the align and quant kernels against vLLM's compiled ops on the same GPU.

The reference calls vLLM's ``moe_align_block_size`` (``overlap_forward.py:420-422``) and
``per_token_group_fp8_quant`` (via ``moe_kernel_quantize_input``, ``:427-429``); both are
compiled CUDA ops.  Where vLLM imports on the box, the b2m kernels are compared with them
directly (skipped otherwise):

* align: ``num_tokens_post_padded`` and ``expert_ids`` identical; inside each expert's
  segment the same pairs and the same number of pad slots (vLLM's in-segment order is not
  ascending, the b2m order is, so the segments are compared as multisets);
* quant: e4m3 codes identical everywhere; scales identical except in groups whose amax
  is below vLLM's floor (vLLM floors amax at 1e-10 before dividing by 448, the reference
  oracle floors the scale at 1e-12 -- ``moe_bench/verify.py:115``).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from tests.conftest import cuda_ok  # noqa: E402

if not cuda_ok():
    pytest.skip("needs an sm_100 GPU", allow_module_level=True)

try:
    from vllm.model_executor.layers.fused_moe.moe_align_block_size import moe_align_block_size as v_align
    from vllm.model_executor.layers.quantization.utils.fp8_utils import per_token_group_quant_fp8 as v_quant
except Exception as exc:  # noqa: BLE001
    pytest.skip(f"vllm not importable here: {type(exc).__name__}", allow_module_level=True)

from td_benchmark_b200 import configs, data, ops  # noqa: E402

DEV = torch.device("cuda", 0)


def _ids(T, k, E, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.stack([torch.randperm(E, device=DEV, generator=g)[:k] for _ in range(T)]).to(torch.int32).contiguous()


@pytest.mark.parametrize("T,k,E", [(64, 2, 8), (4096, 2, 8), (256, 8, 128), (3, 2, 8), (1000, 8, 256)])
def test_align_matches_vllm(T, k, E):
    _check_align(_ids(T, k, E, T * 31 + E), E)


def test_align_matches_vllm_on_zipf_routing():
    cfg = configs.preset("dsv3")
    b = data.build_bundle(cfg, device=DEV, with_weights=False)
    _check_align(b.routing.topk_ids_full.contiguous(), cfg.shape.E)


def _check_align(ids, E):
    s_v, e_v, n_v = v_align(ids, 128, E)
    s_m, e_m, n_m = ops.moe_align_block_size(ids, 128, E)
    torch.cuda.synchronize()
    assert s_v.numel() == s_m.numel() and e_v.numel() == e_m.numel()
    n = int(n_v.item())
    assert n == int(n_m.item())
    nb = n // 128
    assert torch.equal(e_v[:nb], e_m[:nb])
    numel = ids.numel()
    ev = e_v[:nb].cpu().tolist()
    start = 0
    while start < nb:
        end = start
        while end < nb and ev[end] == ev[start]:
            end += 1
        a = torch.sort(s_v[start * 128:end * 128]).values
        b = torch.sort(s_m[start * 128:end * 128]).values
        assert torch.equal(a, b), f"expert {ev[start]} segment differs"
        assert int((b == numel).sum()) == int((a == numel).sum())
        start = end


@pytest.mark.parametrize("rows,cols,scale", [(512, 4096, 1.0), (1024, 7168, 3.0), (64, 256, 1e-3), (7, 2048, 40.0)])
def test_group_quant_matches_vllm(rows, cols, scale):
    g = torch.Generator(device=DEV).manual_seed(rows + cols)
    x = (torch.randn((rows, cols), device=DEV, generator=g) * scale).to(torch.bfloat16)
    x[0, :128] = 0
    if rows > 1:
        x[1, :128] = 1e-30
    q_v, s_v = v_quant(x, 128, eps=1e-10, dtype=torch.float8_e4m3fn, use_ue8m0=False)
    q_m, s_m = ops.quant_g128(x)
    torch.cuda.synchronize()
    assert torch.equal(q_v.view(torch.uint8), q_m.view(torch.uint8))
    floored = x.float().view(rows, cols // 128, 128).abs().amax(-1) <= 1e-10 * 448
    assert torch.equal(s_v[~floored], s_m[~floored])
