"""fp32 torch restatement of the reference layer oracle for large shapes on the GPU (test-only).

Same steps as ``moe_bench/verify.py:14-47`` (and ``oracle/golden.py``): per expert,
group-128 QDQ of the routed rows, gate/up matmul, silu*up, QDQ, down matmul,
routing weight, scatter-add; plus the dense shared expert.  Used where the numpy
oracle would take minutes (the GEMMs are floating-point kernels, so a torch fp32
reference is the stated comparison for them).
"""
import torch


def qdq128(x: torch.Tensor) -> torch.Tensor:
    r, c = x.shape
    cp = (c + 127) // 128 * 128
    xp = torch.nn.functional.pad(x.float(), (0, cp - c)).view(r, cp // 128, 128)
    s = (xp.abs().amax(-1, keepdim=True) / 448.0).clamp(min=1e-12)
    q = (xp / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float() * s
    return q.view(r, cp)[:, :c]


def dequant_block(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    e, n, k = q.shape
    w = q.float().view(e, n // 128, 128, k // 128, 128) * s[:, :, None, :, None].float()
    return w.view(e, n, k).to(torch.bfloat16).float()


def ffn(x, w1, w2):
    gu = qdq128(x) @ w1.T
    i = gu.shape[1] // 2
    h = torch.nn.functional.silu(gu[:, :i]) * gu[:, i:]
    return qdq128(h) @ w2.T


def golden_moe(hidden, topk_ids, topk_weights, w1q, w1s, w2q, w2s, sw=None):
    """hidden [T, H] (any float dtype); w*q/w*s block-FP8 codes/scales -> fp32 [T, H]."""
    hidden = hidden.float()
    out = torch.zeros((hidden.shape[0], w2q.shape[1]), dtype=torch.float32, device=hidden.device)
    for e in range(w1q.shape[0]):
        rows, slots = torch.nonzero(topk_ids == e, as_tuple=True)
        if rows.numel() == 0:
            continue
        w1 = dequant_block(w1q[e:e + 1], w1s[e:e + 1])[0]
        w2 = dequant_block(w2q[e:e + 1], w2s[e:e + 1])[0]
        y = ffn(hidden[rows], w1, w2)
        out.index_add_(0, rows, y * topk_weights[rows, slots].float()[:, None])
    if sw is not None:
        sw1q, sw1s, sw2q, sw2s = sw
        out += ffn(hidden, dequant_block(sw1q, sw1s)[0], dequant_block(sw2q, sw2s)[0])
    return out


def act_quant_error(hidden, topk_ids, topk_weights, w1q, w1s, w2q, w2s, sw=None):
    """max |golden(fp8 activations) - golden(no activation quant)| — the calibrate_tolerance.py measure."""
    global qdq128
    fq = golden_moe(hidden, topk_ids, topk_weights, w1q, w1s, w2q, w2s, sw)
    saved = qdq128
    try:
        qdq128 = lambda x: x.float()  # noqa: E731
        fn = golden_moe(hidden, topk_ids, topk_weights, w1q, w1s, w2q, w2s, sw)
    finally:
        qdq128 = saved
    return fq, float((fq - fn).abs().max())
