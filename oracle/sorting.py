"""moe_sorting restated in numpy (test infrastructure only).

Follows `moe_sorting_native` (op_tests/test_moe_sorting.py:15-70) and the layout
documented in csrc/include/moe_sorting_opus.h:274-322:

* experts in ascending id order; an expert with no tokens takes no block
  (SkipExpertsWithZeroTokens, moe_sorting_opus.h:313-322);
* inside an expert, entries in ascending (token, slot) order -- the row-major
  order of `torch.where(topk_ids == e)`;
* entry = token | slot << 24 (MOCK_ID, moe_sorting_opus.h:266-267);
* each expert's segment is padded to a multiple of `block_size` with
  `M | topk << 24` and weight 0 (moe_sorting_opus.h:1040-1057);
* `sorted_expert_ids[b]` = expert id of block b (local id under expert_mask);
* `num_valid_ids = [padded total, tokens]`;
* `moe_buf[:tokens]` is zeroed (moe_sorting_opus.h:1061-1080).
"""
import numpy as np


def max_num_tokens_padded(M, topk, num_experts, block_size):
    """`aiter/fused_moe.py:41`."""
    return M * topk + num_experts * block_size - topk


def moe_sorting(topk_ids, topk_weights, num_experts, block_size,
                expert_mask=None, num_local_tokens=None):
    """Returns (sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids)."""
    topk_ids = np.asarray(topk_ids, dtype=np.int32)
    topk_weights = np.asarray(topk_weights, dtype=np.float32)
    M, topk = topk_ids.shape
    max_pad = max_num_tokens_padded(M, topk, num_experts, block_size)
    max_blocks = (max_pad + block_size - 1) // block_size
    init_val = np.int32((topk << 24) | M)
    sorted_ids = np.full(max_pad, init_val, dtype=np.int32)
    sorted_weights = np.zeros(max_pad, dtype=np.float32)
    sorted_expert_ids = np.full(max_blocks, -1, dtype=np.int32)
    tokens = M if num_local_tokens is None else int(num_local_tokens)
    ids = topk_ids[:tokens]
    pos = 0
    blk = 0
    skipped = 0
    for e in range(num_experts):
        if expert_mask is not None and int(expert_mask[e]) == 0:
            skipped += 1
            continue
        tok, slot = np.nonzero(ids == e)          # row-major -> ascending (token, slot)
        n = tok.size
        nblk = (n + block_size - 1) // block_size
        sorted_ids[pos:pos + n] = (slot.astype(np.int64) << 24 | tok).astype(np.int32)
        sorted_weights[pos:pos + n] = topk_weights[tok, slot]
        sorted_expert_ids[blk:blk + nblk] = e - skipped
        pos += nblk * block_size
        blk += nblk
    num_valid = np.array([pos, tokens], dtype=np.int32)
    return sorted_ids, sorted_weights, sorted_expert_ids, num_valid
