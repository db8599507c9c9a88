"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in the build container, where the reference package is importable:

    PYTHONPATH=/path/to/td_benchmark python tests/golden/make_golden.py

It imports the reference's own functions (``moe_bench.data.checkpoint``,
``moe_bench.verify``, ``moe_bench.data.routing``) and records their outputs on
seeded inputs.  The fixtures are small ``.npz`` files committed next to this
script; the tests never import the reference.

Fixtures
  fp8_cast.npz        torch ``.to(float8_e4m3fn)`` of every bf16 value in [-448, 448]
                      plus 200k random fp32 values (the cast both quant rules use)
  quant_block128.npz  ``quantize_block128`` on the reference test's ragged (2,130,65)
                      input (``tests/test_quantize.py:27-36``) and on a (3,256,384) block
  group_qdq.npz       ``_group_quant_dequant(x, 128)`` (``verify.py:108-117``) on ragged,
                      zero-group and large-magnitude inputs
  golden_tiny.npz     reference data bundle pieces and ``golden_moe`` output for the
                      BASELINE tiny shape (T=64, H=256, I=512, E=8, top-2, + shared expert)
  routing.npz         ``build_routing`` ids/weights (uniform and Zipf-1.2) for given
                      hidden states and gate weights
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main() -> int:
    from moe_bench.config import RoutingCfg, ShapeCfg
    from moe_bench.context import DistContext
    from moe_bench.data.checkpoint import build_checkpoint, quantize_block128
    from moe_bench.data.routing import build_routing
    from moe_bench.verify import _group_quant_dequant, golden_moe

    # fp8 cast table
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()
    vals = bits[torch.isfinite(bits) & (bits.abs() <= 448.0)]
    rnd = torch.randn(200_000, generator=torch.Generator().manual_seed(1)) * torch.logspace(-4, 2.6, 200_000)
    vals = torch.cat([vals, rnd.clamp(-448, 448), torch.tensor([0.0, -0.0, 448.0, -448.0, 2.0 ** -10, 2.0 ** -9,
                                                                1.5 * 2.0 ** -9, 2.5 * 2.0 ** -9, 464.0 - 1e-3])])
    vals = vals.clamp(-448, 448).contiguous()
    codes = vals.to(torch.float8_e4m3fn).view(torch.uint8)
    np.savez_compressed(HERE / "fp8_cast.npz", x=vals.numpy(), codes=codes.numpy())

    # weight block quant
    g = torch.Generator(device="cpu").manual_seed(7)
    w_a = torch.randn((2, 130, 65), generator=g, dtype=torch.float32) * 0.01
    q_a, s_a = quantize_block128(w_a)
    w_b = torch.randn((3, 256, 384), generator=torch.Generator().manual_seed(8), dtype=torch.float32) * 0.02
    w_b[1, :128, 128:256] = 0.0   # an all-zero block -> scale 1e-12
    q_b, s_b = quantize_block128(w_b)
    np.savez_compressed(HERE / "quant_block128.npz", w_a=w_a.numpy(), q_a=q_a.view(torch.uint8).numpy(),
                        s_a=s_a.numpy(), w_b=w_b.numpy(), q_b=q_b.view(torch.uint8).numpy(), s_b=s_b.numpy())

    # activation group quant-dequant
    x1 = torch.randn((3, 129), generator=torch.Generator().manual_seed(6), dtype=torch.float32) * 0.01
    x2 = torch.randn((16, 512), generator=torch.Generator().manual_seed(9), dtype=torch.bfloat16).float()
    x3 = torch.randn((5, 300), generator=torch.Generator().manual_seed(10), dtype=torch.float32) * 50.0
    x3[2, :128] = 0.0
    x3[4, 5] = 1.0e4
    np.savez_compressed(HERE / "group_qdq.npz", x1=x1.numpy(), y1=_group_quant_dequant(x1, 128).numpy(),
                        x2=x2.numpy(), y2=_group_quant_dequant(x2, 128).numpy(), x3=x3.numpy(),
                        y3=_group_quant_dequant(x3, 128).numpy())

    # tiny golden layer (reference data generators)
    shape = ShapeCfg(M=64, K=256, E=8, top_k=2, n_gateup=1024, n_down=512, shared_experts=1)
    ckpt = build_checkpoint(shape, seed=42, device="cpu")
    hidden = torch.randn((64, 256), generator=torch.Generator().manual_seed(42 + 17), dtype=torch.float32)
    routing = build_routing(hidden.to(torch.bfloat16), ckpt.gate_weight, RoutingCfg(), shape, DistContext())
    out = golden_moe(hidden, routing, ckpt.w1.bf16, ckpt.w2.bf16, ckpt.shared_w1.bf16, ckpt.shared_w2.bf16,
                     "group128")
    out_bf16in = golden_moe(hidden.to(torch.bfloat16).float(), routing, ckpt.w1.bf16, ckpt.w2.bf16,
                            ckpt.shared_w1.bf16, ckpt.shared_w2.bf16, "group128")
    np.savez_compressed(
        HERE / "golden_tiny.npz", hidden=hidden.numpy(),
        w1_q=ckpt.w1.fp8.view(torch.uint8).numpy(), w1_s=ckpt.w1.scale.numpy(),
        w2_q=ckpt.w2.fp8.view(torch.uint8).numpy(), w2_s=ckpt.w2.scale.numpy(),
        sw1_q=ckpt.shared_w1.fp8.view(torch.uint8).numpy(), sw1_s=ckpt.shared_w1.scale.numpy(),
        sw2_q=ckpt.shared_w2.fp8.view(torch.uint8).numpy(), sw2_s=ckpt.shared_w2.scale.numpy(),
        w1_bf16_bits=ckpt.w1.bf16.view(torch.int16).numpy()[:, :8],   # a slice to pin the dequant rounding
        topk_ids=routing.topk_ids_full.numpy(), topk_weights=routing.topk_weights_full.numpy(),
        out=out.numpy(), out_bf16in=out_bf16in.numpy())

    # routing
    hid = torch.randn((256, 128), generator=torch.Generator().manual_seed(3), dtype=torch.bfloat16)
    gate = (torch.randn((64, 128), generator=torch.Generator().manual_seed(4)) * 0.01).to(torch.bfloat16)
    shape_r = ShapeCfg(M=256, K=128, E=64, top_k=8, n_gateup=256, n_down=128)
    r_uni = build_routing(hid, gate, RoutingCfg(), shape_r, DistContext())
    r_zipf = build_routing(hid, gate, RoutingCfg(imbalance_kind="zipf", zipf_s=1.2, gate_seed=42), shape_r,
                           DistContext())
    np.savez_compressed(HERE / "routing.npz", hidden_bits=hid.view(torch.int16).numpy(),
                        gate_bits=gate.view(torch.int16).numpy(), ids_uniform=r_uni.topk_ids_full.numpy(),
                        w_uniform=r_uni.topk_weights_full.numpy(), ids_zipf=r_zipf.topk_ids_full.numpy(),
                        w_zipf=r_zipf.topk_weights_full.numpy())
    print("wrote fixtures to", HERE)
    return 0


if __name__ == "__main__":
    sys.exit(main())
