"""``moe_align_block_size`` restated in numpy (test oracle).

Contract (vLLM 0.22, ``vllm/model_executor/layers/fused_moe/moe_align_block_size.py``;
called by the reference at ``moe_bench/overlap/overlap_forward.py:420-422``):

* flatten ``topk_ids`` (``numel`` (token, slot) pairs, flat index ``t*top_k + j``);
* count pairs per expert, pad each count up to a multiple of ``block_size``
  (an expert with no pairs gets no block);
* lay the padded segments out in expert order; inside a segment write the flat
  pair indices, then the pad id ``numel`` (docstring example ``:57-71``);
* ``expert_ids[b]`` = expert owning block ``b``; with ``expert_map`` the ids are
  remapped global -> local and non-local experts become ``-1`` (``:100-101``);
* buffer sizes: ``numel + E*(block_size-1)`` entries, capped at
  ``numel*block_size`` when ``numel < E`` (``:74-80``); ``cdiv(len, block_size)``
  expert ids; one ``num_tokens_post_padded`` value.

vLLM's compiled op documents no order inside a segment.  This build fixes it to
ascending flat pair index (deterministic); entries past ``num_tokens_post_padded``
are ``numel`` in ``sorted_token_ids`` and ``-1`` in ``expert_ids``.
"""
from __future__ import annotations

import numpy as np


def buffer_sizes(numel: int, num_experts: int, block_size: int) -> tuple[int, int]:
    max_padded = numel + num_experts * (block_size - 1)
    if numel < num_experts:
        max_padded = min(numel * block_size, max_padded)
    return max_padded, (max_padded + block_size - 1) // block_size


def moe_align_block_size(topk_ids: np.ndarray, block_size: int, num_experts: int,
                         expert_map: np.ndarray | None = None
                         ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    flat = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    numel = flat.size
    max_padded, max_blocks = buffer_sizes(numel, num_experts, block_size)
    counts = np.bincount(flat, minlength=num_experts)[:num_experts]
    padded = (counts + block_size - 1) // block_size * block_size
    starts = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.int64)
    ntpp = int(padded.sum())
    sorted_ids = np.full(max_padded, numel, dtype=np.int32)
    expert_ids = np.full(max_blocks, -1, dtype=np.int32)
    order = np.argsort(flat, kind="stable")          # ascending pair index inside each expert
    seg_pos = 0
    for e in range(num_experts):
        c = int(counts[e])
        if c:
            sorted_ids[starts[e]:starts[e] + c] = order[seg_pos:seg_pos + c]
            seg_pos += c
            b0 = starts[e] // block_size
            expert_ids[b0:b0 + padded[e] // block_size] = e
    if expert_map is not None:
        em = np.asarray(expert_map, dtype=np.int32)
        valid = expert_ids >= 0
        expert_ids[valid] = em[expert_ids[valid]]
    return sorted_ids, expert_ids, np.array([ntpp], dtype=np.int32)
