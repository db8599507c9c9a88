"""CPU oracle for the FP8 MoE layer path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms of the path that
stmoonar/td_benchmark measures (scheme b2, ``moe_bench/overlap/overlap_forward.py:348-622``):

* ``fp8``     — fp32 -> float8_e4m3fn round-to-nearest-even encode / decode, the
                cast ``torch.Tensor.to(torch.float8_e4m3fn)`` performs in
                ``moe_bench/verify.py:116`` and ``moe_bench/data/checkpoint.py:46``.
* ``quant``   — 1x128 activation group quant (``moe_bench/verify.py:108-117``) and
                128x128 weight block quant (``moe_bench/data/checkpoint.py:28-52``).
* ``align``   — ``moe_align_block_size`` (vLLM contract,
                ``vllm/model_executor/layers/fused_moe/moe_align_block_size.py:11-104``).
* ``golden``  — the fp32 per-expert layer oracle ``golden_moe``
                (``moe_bench/verify.py:14-47``) and ``compare_outputs`` gates
                (``moe_bench/verify.py:50-105``, ``moe_bench/worker.py:108-110``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg may import this package, and only as the checker or the
timed CPU baseline.  The product path (``td_benchmark_b200``) never imports it.

Parity pins: ``tests/golden/make_golden.py`` imports the reference package in the
build container and writes fixtures under ``tests/golden/``; ``tests/test_oracle.py``
checks this oracle against them (fp8 bytes and scales bit-exact; golden layer output
to fp32 round-off).  ``moe_align_block_size`` is a compiled vLLM op with no source
and no reference test: it is pinned only by the worked example of its docstring
(``moe_align_block_size.py:57-71``) and by its documented buffer sizing.
"""
