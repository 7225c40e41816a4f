"""MXFP4 activation quant and MoE scale sorting (test infrastructure only).

* `e8m0_shuffle` restates `e8m0_shuffle` (aiter/utility/fp4_utils.py:72-92): the
  e8m0 scale matrix, padded to a multiple of 256 rows and 8 columns, viewed as
  [rows/32, 2, 16, cols/8, 2, 4] and permuted to (0, 3, 5, 2, 4, 1).  The padding
  is `torch.empty` in the reference (undefined); here it is 0.
* `moe_mxfp4_sort` restates the torch reference of the sorted-scale layout,
  `run_torch` (op_tests/test_moe_sorting_mxfp4.py:20-43): row p of the sorted
  matrix takes the scales of token `sorted_ids[p] & 0xFFFFFF` (stage 1, scales
  [tokens, cols]) or of row token * topk + slot (stage 2, scales [tokens, topk,
  cols]; slot = sorted_ids[p] >> 24); padding slots (token == token_num) and every
  row from num_valid_ids on are 0; rows are padded to a multiple of 32 and the
  result is shuffled like e8m0_shuffle.  The HIP kernel `mxfp4_moe_sort_hip` and the
  fused quant + sort (`fused_dynamic_mxfp4_quant_moe_sort`, aiter/ops/quant.py:
  584-652) produce the same matrix.
* `per_1x32_f4_quant` lives in oracle/quant.py.
"""
import numpy as np


def shuffle_index(rows, cols):
    """(src_row, src_col) of every element of the shuffled [rows, cols] matrix, in
    output order (rows % 32 == 0, cols % 8 == 0)."""
    a, b, c, d, e, f = np.meshgrid(np.arange(rows // 32), np.arange(cols // 8), np.arange(4), np.arange(16),
                                   np.arange(2), np.arange(2), indexing="ij")
    src_row = a * 32 + f * 16 + d
    src_col = b * 8 + e * 4 + c
    return src_row.reshape(-1), src_col.reshape(-1)


def shuffle(m):
    """The (0, 3, 5, 2, 4, 1) permutation of a [rows, cols] matrix viewed as
    [rows/32, 2, 16, cols/8, 2, 4], returned as [rows, cols]."""
    rows, cols = m.shape
    r, c = shuffle_index(rows, cols)
    return m[r, c].reshape(rows, cols)


def e8m0_shuffle(scale):
    s = np.asarray(scale, dtype=np.uint8)
    m, n = s.shape
    pad = np.zeros(((m + 255) // 256 * 256, (n + 7) // 8 * 8), dtype=np.uint8)
    pad[:m, :n] = s
    return shuffle(pad)


def moe_mxfp4_sort(scale, sorted_ids, num_valid, token_num):
    """Sorted, shuffled e8m0 scales: [ceil(len(sorted_ids) / 32) * 32, cols] uint8."""
    s = np.asarray(scale, dtype=np.uint8)
    topk = 1
    if s.ndim == 3:
        topk = s.shape[1]
        s = s.reshape(-1, s.shape[-1])
    ids = np.asarray(sorted_ids, dtype=np.int64).copy()
    ids[int(num_valid):] = token_num
    slot = ids >> 24
    tok = ids & 0xFFFFFF
    pad = tok == token_num
    src = tok * topk + slot if topk > 1 else tok
    src = np.where(pad, 0, src)
    g = s[src]
    g[pad] = 0
    rows = (g.shape[0] + 31) // 32 * 32
    full = np.zeros((rows, g.shape[1]), dtype=np.uint8)
    full[:g.shape[0]] = g
    return shuffle(full)
