"""moe_align_block_size's contract, restated in numpy (test infrastructure only).

Follows the vLLM 0.22.0 wrapper and its docstring (vllm/model_executor/layers/fused_moe/moe_align_block_size.py:
11-103), the call the kit makes (files/mbx_moek.py:266, ``ignore_invalid_experts=True``, no expert_map) and what the
kit's kernel relies on (files/mbx_moek.cu:309-314: the valid rows of a block are a prefix of it).

- The flat (token, slot) indices ``i = token * top_k + slot`` are grouped by expert, experts in ascending order,
  indices ascending inside an expert (the docstring example, :59-72). Ids outside [0, num_experts) are skipped.
- Each expert's group is padded to a multiple of ``block_size`` with the sentinel ``numel``; an expert with no rows
  has no block. ``num_tokens_post_pad`` is the padded total.
- ``sorted_ids`` has ``numel + E * (block_size - 1)`` entries (``min(numel * block_size, ...)`` when numel < E,
  :74-80); entries past the padded total hold the sentinel.
- ``expert_ids[b]`` is the expert of block b for b < num_tokens_post_pad / block_size, and -1 after that.

The compiled kernel's order inside an expert cannot be observed here (no GPU); the docstring example is the only
pin, and this restatement fixes stable ascending order.
"""
import numpy as np


def sizes(numel: int, num_experts: int, block_size: int):
    """(len(sorted_ids), len(expert_ids)) as the wrapper allocates them (:74-87)."""
    n = numel + num_experts * (block_size - 1)
    if numel < num_experts:
        n = min(numel * block_size, n)
    return n, (n + block_size - 1) // block_size


def moe_align(topk_ids: np.ndarray, num_experts: int, block_size: int):
    """topk_ids int [M, top_k] -> (sorted_ids int32, expert_ids int32, num_tokens_post_pad int32 [1])."""
    flat = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    numel = flat.size
    ls, lb = sizes(numel, num_experts, block_size)
    sorted_ids = np.full(ls, numel, dtype=np.int32)
    expert_ids = np.full(lb, -1, dtype=np.int32)
    pos = 0
    for e in range(num_experts):
        rows = np.nonzero(flat == e)[0]
        if rows.size == 0:
            continue
        sorted_ids[pos:pos + rows.size] = rows
        nblk = (rows.size + block_size - 1) // block_size
        expert_ids[pos // block_size:pos // block_size + nblk] = e
        pos += nblk * block_size
    return sorted_ids, expert_ids, np.array([pos], dtype=np.int32)
