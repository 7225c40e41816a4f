"""CPU checks of the quick allreduce oracle (oracle/quick_reduce.py) against what the
reference's own test demands (op_tests/multigpu_tests/test_quick_all_reduce.py):

* random inputs: |out - sum| <= 1.25 W + 0.5 W |sum| (:114-121);
* the variable-input loop (:128-170): all-zero inputs reduce to 0 and all-one
  inputs to exactly W with INT4 on fp16 (cast_bf2half) -- and so do the other levels
  and dtypes, except FP8 on bf16 without the cast, whose bf16 scale factor T(1/240)
  is too coarse (hand trace below);
* codec properties: a group's scale depends on its own 32 values only; the group
  extreme of the INT levels decodes exactly; level FP is the rank-order T sum.
"""
import numpy as np
import pytest

from oracle import quick_reduce as q
from oracle.codecs import round_bf16

MODES = [("fp16", False), ("bf16", False), ("bf16", True)]


def _inputs(world, n, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal(n) * scale).astype(np.float32) for _ in range(world)]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("level", q.LEVELS)
@pytest.mark.parametrize("dtype,cast", MODES)
def test_reference_tolerance(world, level, dtype, cast):
    xs = _inputs(world, 4 * 16384 + 8 * 5, seed=world * 10 + level)
    rnd = (lambda a: a.astype(np.float16).astype(np.float32)) if dtype == "fp16" else round_bf16
    xs = [rnd(x) for x in xs]
    out = q.quick_allreduce(xs, level, dtype, cast)
    ref = np.sum(np.stack(xs).astype(np.float64), axis=0)
    atol, rtol = q.reference_test_tolerance(world)
    assert np.all(np.abs(out - ref) <= atol + rtol * np.abs(ref))
    # much tighter in practice: the INT4 error is a fraction of the group scale
    assert np.sqrt(np.mean((out - ref) ** 2)) < 0.1 * world


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("level", q.LEVELS)
@pytest.mark.parametrize("dtype,cast", MODES)
def test_zeros_and_ones(world, level, dtype, cast):
    n = 2048 * 3
    zeros = q.quick_allreduce([np.zeros(n, np.float32)] * world, level, dtype, cast)
    assert np.all(zeros == 0)
    ones = q.quick_allreduce([np.ones(n, np.float32)] * world, level, dtype, cast)
    if level == q.FP8 and dtype == "bf16" and not cast:
        # bf16: dec = T(1 * 0.004150390625) ; enc = T(1 / dec) = 241 ; 1 * 241 -> e4m3 240 ;
        # 240 * dec = 0.99609375.  W = 2: sum 1.9921875 ; dec = 0.008239746 ; enc = 121.5 ;
        # 242 -> e4m3 240 ; 240 * dec -> 1.9765625
        if world == 2:
            assert np.all(ones == np.float32(1.9765625))
        assert np.all(np.abs(ones - world) <= 0.02 * world)
    else:
        assert np.all(ones == world)


@pytest.mark.parametrize("level", [q.FP8, q.INT6, q.INT4])
@pytest.mark.parametrize("t", ["fp16", "bf16"])
def test_groups_are_independent(level, t):
    rng = np.random.default_rng(3)
    x = q.to_t(rng.standard_normal(64 * 6).astype(np.float32), t)
    base = q.qdq(x, level, t)
    y = x.copy()
    y[64 * 2 + 10] = q.to_t(np.float32(50.0), t).reshape(-1)[0]  # an even element of span 2
    got = q.qdq(y, level, t)
    changed = np.nonzero(got != base)[0]
    assert changed.size > 0
    # only the even elements of span 2 may change
    assert np.all((changed // 64 == 2) & (changed % 2 == 0))


@pytest.mark.parametrize("level", [q.INT6, q.INT4])
def test_int_extreme_is_exact(level):
    rng = np.random.default_rng(5)
    x = q.to_t(rng.standard_normal(64 * 8).astype(np.float32), "fp16")
    out = q.qdq(x, level, "fp16").reshape(-1, 32, 2)
    xg = x.reshape(-1, 32, 2)
    for g in range(xg.shape[0]):
        for p in range(2):
            v = xg[g, :, p]
            mx, mn = v.max(), v.min()
            m = mx if abs(mx) > abs(mn) else mn
            i = int(np.nonzero(v == m)[0][0])
            assert out[g, i, p] == m


def test_fp_level_is_rank_order_sum():
    xs = [q.to_t(x, "fp16") for x in _inputs(4, 16384 + 64, seed=9, scale=200.0)]
    acc = np.zeros_like(xs[0])
    for x in xs:
        acc = (acc + x).astype(np.float16).astype(np.float32)
    assert np.array_equal(q.quick_allreduce(xs, q.FP, "fp16"), acc)


def test_fp16_overflow_saturates():
    xs = [np.full(64, 40000.0, np.float32)] * 2
    out = q.quick_allreduce(xs, q.FP, "fp16")
    assert np.all(out == 65504.0)
    # a true infinity stays infinite
    assert np.isinf(q.to_t(np.float32(np.inf), "fp16"))


def test_cast_bf16_rounds_through_fp16():
    x = round_bf16(np.array([1.0 + 2.0 ** -7] * 64, dtype=np.float32))  # exact in bf16 and fp16
    out = q.quick_allreduce([x, x], q.FP, "bf16", cast_bf2half=True)
    assert np.all(out == round_bf16(np.float32(2.0 + 2.0 ** -6)))


def test_message_must_be_16_byte_multiple():
    with pytest.raises(ValueError):
        q.quick_allreduce([np.zeros(12, np.float32)] * 2, q.INT4)
