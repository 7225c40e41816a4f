"""Allreduce semantics of the tensor-parallel path (test infrastructure only).

* `allreduce_rank_order`: the IPC allreduce of aiter_b200 -- every rank's input
  accumulated in fp32 in rank order 0..W-1, rounded once to the input dtype;
  identical bits on every rank.
* `allreduce_fp8_quant`: the reference's fp8-quantised two-shot allreduce,
  `allReduceQuantFp8` (csrc/include/custom_all_reduce.cuh:1018-1088), dispatched by
  `runFp8QuantKernel` (:2177-2232) for fp16 inputs of at least 128 * 2048 elements
  when `open_fp8_quant` is set (csrc/kernels/custom_all_reduce.cu:90-96):
    - the input is cut into W segments of `size // W` 16-byte packs (8 halves),
      the last rank taking the remainder (:1029-1033);
    - owner rank r sums its segment over the ranks in the rotated order
      r, r+1, ..., r-1 in fp32 and rounds to fp16 (`multiGPUPackReduce`,
      :1001-1013, ptrs[i] = rank (r + i) % W, :1038-1042); that is r's result;
    - it quantises the sum in groups of G elements (G = 128, 64, 32, 16 or 8, the
      largest dividing numel // W, :2209-2229), aligned to the segment start:
      scale = fp16(amax / 448) (:1049-1053), code = e4m3(x / scale) in fp32
      (`packQuant`, :957-976);
    - every other rank dequantises the owner's codes: fp16(float(code) * scale)
      (`packDequant`, :978-999, :1062-1087).
  So each rank's own segment is the exact sum and the other segments carry fp8
  rounding: ranks do not agree bit for bit.  One deviation: a group whose scale
  is 0 (all zeros, or amax below 448 * 2^-25) would divide 0 by 0 in the
  reference and decode to NaN; here, as in aiter_b200, its codes are 0.
"""
import numpy as np

from .codecs import fp8_e4m3_decode, fp8_e4m3_encode

FP8_QUANT_MIN_NUMEL = 128 * 2048


def allreduce_rank_order(xs, dtype):
    """fp32 sum of the per-rank arrays in rank order, rounded to `dtype`."""
    acc = np.zeros(np.asarray(xs[0]).shape, dtype=np.float32)
    for x in xs:
        acc += np.asarray(x).astype(np.float32)
    return acc.astype(dtype)


def fp8_quant_group(numel, world):
    """Quant group size of runFp8QuantKernel for `numel` elements on `world` ranks."""
    single = numel // world
    for g in (128, 64, 32, 16):
        if single % g == 0:
            return g
    return 8


def fp8_quant_segments(numel, world):
    """[(lo, hi)] pack ranges (8 elements per pack) owned by each rank."""
    size = numel // 8
    part = size // world
    return [(r * part, size if r == world - 1 else (r + 1) * part) for r in range(world)]


def allreduce_fp8_quant(xs):
    """Per-rank results of the fp8-quantised allreduce of fp16 arrays `xs`."""
    world = len(xs)
    xs = [np.asarray(x, dtype=np.float16).reshape(-1) for x in xs]
    numel = xs[0].size
    G = fp8_quant_group(numel, world)
    segs = fp8_quant_segments(numel, world)
    exact, deq = [], []
    for r, (lo, hi) in enumerate(segs):
        acc = np.zeros((hi - lo) * 8, dtype=np.float32)
        for i in range(world):
            acc += xs[(r + i) % world][lo * 8:hi * 8].astype(np.float32)
        s16 = acc.astype(np.float16)
        groups = s16.astype(np.float32).reshape(-1, G)
        amax = np.abs(groups).max(axis=1)
        scale = (amax / np.float32(448.0)).astype(np.float16).astype(np.float32)
        safe = np.where(scale == 0, np.float32(1.0), scale)
        q = fp8_e4m3_encode(np.where(scale[:, None] == 0, np.float32(0.0), groups / safe[:, None]))
        d = (fp8_e4m3_decode(q) * scale[:, None]).astype(np.float16).reshape(-1)
        exact.append(s16)
        deq.append(d)
    outs = []
    for p in range(world):
        parts = [exact[s] if s == p else deq[s] for s in range(world)]
        outs.append(np.concatenate(parts))
    return outs
