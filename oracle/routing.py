"""Routing restated in numpy (test infrastructure only).

* `topk_softmax` follows the torch reference `test_nofuse`
  (op_tests/test_moeTopkSoftmax.py:21-41): softmax over all experts in fp32,
  top-k of the softmax values, optional renormalisation over the k kept weights.
* `grouped_topk` follows `grouped_topk_torch` (aiter/ops/topk.py:161-197) and
  `biased_grouped_topk` follows `biased_grouped_topk_torch` (aiter/ops/topk.py:
  116-158); both multiply by `routed_scaling_factor` after renormalisation as the
  device kernel does (csrc/kernels/topk_softmax_kernels_group.cu:596-611).

Arithmetic contract shared with the device kernels (aiter_b200/csrc/routing.cu),
which reproduce it bit for bit:

* exp is `rexp` below: Cody & Waite's additive range reduction
  (x = n ln2 + r, |r| <= ln2/2, ln 2 split into a 21-bit head and a tail so that
  n * head is exact) and the degree-13 Taylor polynomial of e^r, evaluated in
  IEEE double with separately rounded multiplies and adds (no fused multiply-add),
  scaled by 2^n and rounded once to fp32.  The double result is within a few
  double ulps of e^x, so the fp32 result is the correctly rounded one except when
  e^x lies within about 2^-50 relative of an fp32 rounding boundary.
* softmax follows torch's AVX-512 CPU kernel order (the one the reference test's
  torch path takes on the host that produced the golden vectors): max; e_i =
  exp(x_i - max); the sum of 16-lane vectors accumulated in order (lane j adds
  elements j, j+16, j+32, ...; a partial last vector adds only its first E mod 16
  lanes), then a butterfly over the lanes (lane j plus lane j^8, then ^4, ^2, ^1);
  with E < 16 the sum runs element by element from e_0; p_i = e_i * (1 / sum).
* the k kept weights are summed in the order torch's CPU sum kernel uses for a
  contiguous row of k floats (`ksum`), then each weight is divided by the sum.
* selection: the k largest softmax values, the lower expert index first among
  equal values (torch's own order among equal values is unspecified).
* sigmoid(x) = 1 / (1 + exp(-x)), each step rounded to fp32.

torch's own softmax uses a faster exp of lower accuracy, and its grouped top-k
returns its picks in an unspecified order (sorted=False), which changes the order
of the renormalising sum; so the weights here can differ from the reference's
torch outputs by a few fp32 ulps (measured per golden case in the tests), while
ids, which the tests compare exactly, agree.
"""
import numpy as np

_LOG2E = float.fromhex("0x1.71547652b82fep+0")
_LN2_HI = float.fromhex("0x1.62e42p-1")            # ln 2 with 21 significant bits
_LN2_LO = float.fromhex("0x1.fdf473de6af28p-22")    # ln 2 - _LN2_HI, rounded to double
_INV_FACT = [float.fromhex(h) for h in (
    "0x1p+0", "0x1p+0", "0x1p-1", "0x1.5555555555555p-3", "0x1.5555555555555p-5", "0x1.1111111111111p-7",
    "0x1.6c16c16c16c17p-10", "0x1.a01a01a01a01ap-13", "0x1.a01a01a01a01ap-16", "0x1.71de3a556c734p-19",
    "0x1.27e4fb7789f5cp-22", "0x1.ae64567f544e4p-26", "0x1.1eed8eff8d898p-29", "0x1.6124613a86d09p-33")]


def rexp(x):
    """exp of fp32 values, returned as fp32 (the contract above)."""
    x = np.asarray(x, dtype=np.float32)
    d = np.clip(np.nan_to_num(x.astype(np.float64)), -110.0, 100.0)
    n = np.rint(d * _LOG2E)
    r = (d - n * _LN2_HI) - n * _LN2_LO
    p = np.full_like(r, _INV_FACT[13])
    for c in _INV_FACT[12::-1]:
        p = p * r + c
    with np.errstate(over="ignore"):
        y = (p * np.ldexp(1.0, n.astype(np.int32))).astype(np.float32)
    y = np.where(x > 100.0, np.float32(np.inf), y)
    y = np.where(x < -110.0, np.float32(0.0), y)
    return np.where(np.isnan(x), x, y).astype(np.float32)


def softmax_sum(e):
    """Row sums of e [M, E] fp32 in torch's AVX-512 CPU softmax order."""
    e = np.asarray(e, dtype=np.float32)
    M, E = e.shape
    if E < 16:
        acc = e[:, 0].copy()
        for j in range(1, E):
            acc = (acc + e[:, j]).astype(np.float32)
        return acc
    full = E // 16
    acc = e[:, :16].copy()
    for t in range(1, full):
        acc = (acc + e[:, 16 * t:16 * t + 16]).astype(np.float32)
    rem = E % 16
    if rem:
        acc[:, :rem] = (acc[:, :rem] + e[:, 16 * full:]).astype(np.float32)
    for o in (8, 4, 2, 1):
        lanes = np.arange(16)
        acc = (acc + acc[:, lanes ^ o]).astype(np.float32)
    return acc[:, 0]


def softmax(x):
    x = np.asarray(x, dtype=np.float32)
    mx = x.max(axis=-1, keepdims=True)
    e = rexp((x - mx).astype(np.float32))
    rz = (np.float32(1.0) / softmax_sum(e)).astype(np.float32)
    return (e * rz[:, None]).astype(np.float32)


def ksum(w):
    """Row sums of w [M, k] fp32 in the order of torch's CPU sum over a contiguous
    row of k floats: k < 8 -- four accumulators take elements 4i+j, the tail
    elements go to the first, then acc0 + acc1 + acc2 + acc3; k >= 8 -- 8-lane
    vectors added lane-wise in order, the tail elements (from 8 * (k // 8)) summed
    from zero, then the 8 lanes added to that one by one."""
    w = np.asarray(w, dtype=np.float32)
    M, k = w.shape
    f = lambda a: np.asarray(a, dtype=np.float32)
    if k < 8:
        nil = k // 4
        acc = [np.zeros(M, np.float32) for _ in range(4)]
        for i in range(nil):
            for j in range(4):
                acc[j] = f(acc[j] + w[:, 4 * i + j])
        for i in range(4 * nil, k):
            acc[0] = f(acc[0] + w[:, i])
        r = acc[0]
        for j in range(1, 4):
            r = f(r + acc[j])
        return r
    nv = k // 8
    lanes = w[:, :8].copy()
    for v in range(1, nv):
        lanes = f(lanes + w[:, 8 * v:8 * v + 8])
    r = np.zeros(M, np.float32)
    for i in range(8 * nv, k):
        r = f(r + w[:, i])
    for j in range(8):
        r = f(r + lanes[:, j])
    return r


def _topk_lowest_index(scores, k):
    # stable sort on -score: among equal scores the lower index comes first
    order = np.argsort(-scores, axis=-1, kind="stable")
    return order[:, :k]


def _renorm(w):
    return (w / ksum(w)[:, None]).astype(np.float32)


def topk_softmax(gating, topk, renormalize):
    """gating: [M, E] (any float dtype; converted to fp32).
    Returns weights f32 [M,k], ids i32 [M,k], token_expert_indices i32 [M,k]."""
    x = np.asarray(gating, dtype=np.float32)
    M, E = x.shape
    p = softmax(x)
    ids = _topk_lowest_index(p, topk)
    w = np.take_along_axis(p, ids, axis=-1)
    if renormalize:
        w = _renorm(w)
    tei = (np.arange(topk, dtype=np.int32)[None, :] * M + np.arange(M, dtype=np.int32)[:, None])
    return w.astype(np.float32), ids.astype(np.int32), tei.astype(np.int32)


def _sigmoid(x):
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + rexp(-x)).astype(np.float32)).astype(np.float32)


def grouped_topk(gating, topk, num_expert_group, topk_group, renormalize,
                 is_softmax=True, routed_scaling_factor=1.0):
    x = np.asarray(gating, dtype=np.float32)
    M, E = x.shape
    if is_softmax:
        scores = softmax(x)
    else:
        scores = _sigmoid(x)
    g = scores.reshape(M, num_expert_group, -1).max(axis=-1)
    gidx = _topk_lowest_index(g, topk_group)
    gmask = np.zeros_like(g)
    np.put_along_axis(gmask, gidx, 1.0, axis=-1)
    smask = np.repeat(gmask, E // num_expert_group, axis=-1).astype(bool)
    tmp = np.where(smask, scores, np.float32(0.0))
    ids = _topk_lowest_index(tmp, topk)
    w = np.take_along_axis(tmp, ids, axis=-1)
    if renormalize:
        w = _renorm(w)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return w, ids.astype(np.int32)


def biased_grouped_topk(gating, correction_bias, topk, num_expert_group, topk_group,
                        renormalize, routed_scaling_factor=1.0):
    x = np.asarray(gating, dtype=np.float32)
    M, E = x.shape
    scores = _sigmoid(x)
    choice = (scores + np.asarray(correction_bias, dtype=np.float32)[None, :]).astype(np.float32)
    per_group = choice.reshape(M, num_expert_group, -1)
    top2 = -np.sort(-per_group, axis=-1)[..., :2]
    g = (top2[..., 0] + top2[..., 1]).astype(np.float32)
    gidx = _topk_lowest_index(g, topk_group)
    gmask = np.zeros_like(g)
    np.put_along_axis(gmask, gidx, 1.0, axis=-1)
    smask = np.repeat(gmask, E // num_expert_group, axis=-1).astype(bool)
    tmp = np.where(smask, choice, np.float32(0.0))
    ids = _topk_lowest_index(tmp, topk)
    w = np.take_along_axis(scores, ids, axis=-1)
    if renormalize:
        w = _renorm(w)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return w, ids.astype(np.int32)


def topk_sigmoid(logits, topk):
    """`topk_sigmoid` (aiter/ops/moe_op.py:40-42; torch reference
    op_tests/test_moe_topk_sigmoid.py:30-35): the topk largest logits per row in
    descending order (equal values: lower index first) and sigmoid of each in fp32.
    Returns (weights f32 [M, k], ids i32 [M, k])."""
    x = np.asarray(logits, dtype=np.float32)
    ids = np.argsort(-x, axis=-1, kind="stable")[:, :topk].astype(np.int32)
    v = np.take_along_axis(x, ids.astype(np.int64), axis=-1)
    w = _sigmoid(v)
    return w, ids
