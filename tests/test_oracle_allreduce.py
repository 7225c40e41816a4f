"""CPU checks of the allreduce oracle (oracle/allreduce.py): the rank-order sum and
the restatement of the reference's fp8-quantised two-shot allreduce
(allReduceQuantFp8, csrc/include/custom_all_reduce.cuh:1018-1088).  The reference
kernel is HIP-only and ships no vectors, so these are known-answer cases worked by
hand from its source and structural properties."""
import numpy as np
import pytest

from oracle.allreduce import (allreduce_fp8_quant, allreduce_rank_order, fp8_quant_group,
                              fp8_quant_segments)
from oracle.codecs import round_fp8


def test_quant_group_follows_the_dispatch_rule():
    # runFp8QuantKernel: the largest of 128/64/32/16 dividing numel / world, else 8
    assert fp8_quant_group(128 * 2048, 8) == 128
    assert fp8_quant_group(8 * 64 * 3, 8) == 64
    assert fp8_quant_group(2 * 48, 2) == 16
    assert fp8_quant_group(2 * 40, 2) == 8


def test_segments_cover_every_pack_once_last_rank_takes_the_remainder():
    segs = fp8_quant_segments(8 * 1003, 4)
    assert segs[0] == (0, 250) and segs[-1] == (750, 1003)
    assert all(a[1] == b[0] for a, b in zip(segs, segs[1:]))


def test_known_answer_constant_inputs():
    # every rank holds 1.0: each owner sums to W exactly, amax = W,
    # scale = fp16(W / 448), code = e4m3(W / scale), decoded = fp16(code * scale)
    W, n = 4, 128 * 2048
    outs = allreduce_fp8_quant([np.ones(n, np.float16)] * W)
    scale = np.float32(np.float16(np.float32(W) / np.float32(448.0)))
    dec = np.float16(round_fp8(np.float32(W) / scale)[()] * scale)
    segs = fp8_quant_segments(n, W)
    for p, o in enumerate(outs):
        for s, (lo, hi) in enumerate(segs):
            want = np.float16(W) if s == p else dec
            assert np.all(o[lo * 8:hi * 8] == want), (p, s)


def test_own_segment_exact_others_within_fp8_rounding():
    rng = np.random.default_rng(3)
    W, n = 8, 128 * 2048
    xs = [rng.standard_normal(n).astype(np.float16) for _ in range(W)]
    outs = allreduce_fp8_quant(xs)
    exact = allreduce_rank_order(xs, np.float32)
    segs = fp8_quant_segments(n, W)
    for p, o in enumerate(outs):
        for s, (lo, hi) in enumerate(segs):
            got = o[lo * 8:hi * 8].astype(np.float32)
            ref = exact[lo * 8:hi * 8]
            if s == p:
                # rotated summation order vs rank order: a few fp16 ulps at most
                assert np.allclose(got, ref, rtol=2e-3, atol=2e-3)
            else:
                # e4m3 keeps 3 mantissa bits: half a step is 2^-4 relative, plus the
                # subnormal quantum 2^-9 of the group's scale
                g = got.reshape(-1, 128)
                r = ref.reshape(-1, 128)
                amax = np.abs(r).max(axis=1, keepdims=True)
                assert np.all(np.abs(g - r) <= np.abs(r) * 2.0 ** -4 + amax / 448 * 2.0 ** -9 + 2e-3 * np.abs(r) + 1e-3)
    # ranks disagree outside their own segment, agree on nothing bit for bit overall
    assert not np.array_equal(outs[0], outs[1])


def test_zero_group_decodes_to_zero_not_nan():
    W, n = 2, 128 * 2048
    xs = [np.zeros(n, np.float16) for _ in range(W)]
    xs[0][:128] = 0  # a whole zero group, amax 0 -> scale 0
    xs[0][128:] = 1
    outs = allreduce_fp8_quant(xs)
    assert not np.isnan(outs[1].astype(np.float32)).any()
    assert np.all(outs[1][:128] == 0)


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_rank_order_sum(dtype):
    xs = [np.full(16, v, dtype) for v in (1e4, 1.0, -1e4)]
    # fp32 accumulation in rank order: (1e4 + 1) - 1e4 = 1 exactly in fp32
    assert np.all(allreduce_rank_order(xs, dtype) == dtype(1.0))
