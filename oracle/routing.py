"""Routing restated in numpy (test infrastructure only).

* `topk_softmax` follows the torch reference `test_nofuse`
  (op_tests/test_moeTopkSoftmax.py:21-41): softmax over all experts in fp32,
  top-k, optional renormalisation over the k kept weights.  Selection is made on
  the fp32 logits with the lower expert index winning a tie, the rule of the
  device kernel's arg-max (csrc/kernels/topk_softmax_kernels.cu:356-362);
  softmax is monotonic, so on distinct logits this is torch's top-k set.
* `grouped_topk` follows `grouped_topk_torch` (aiter/ops/topk.py:161-197) and
  `biased_grouped_topk` follows `biased_grouped_topk_torch` (aiter/ops/topk.py:
  116-158); both multiply by `routed_scaling_factor` after renormalisation as the
  device kernel does (csrc/kernels/topk_softmax_kernels_group.cu:596-611).
"""
import numpy as np


def _topk_lowest_index(scores, k):
    # stable sort on -score: among equal scores the lower index comes first
    order = np.argsort(-scores, axis=-1, kind="stable")
    return order[:, :k]


def topk_softmax(gating, topk, renormalize):
    """gating: [M, E] (any float dtype; converted to fp32).
    Returns weights f32 [M,k], ids i32 [M,k], token_expert_indices i32 [M,k]."""
    x = np.asarray(gating, dtype=np.float32)
    M, E = x.shape
    mx = x.max(axis=-1, keepdims=True)
    e = np.exp(x - mx).astype(np.float32)
    z = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    p = (e * (np.float32(1.0) / z)).astype(np.float32)
    ids = _topk_lowest_index(x, topk)
    w = np.take_along_axis(p, ids, axis=-1)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    tei = (np.arange(topk, dtype=np.int32)[None, :] * M + np.arange(M, dtype=np.int32)[:, None])
    return w.astype(np.float32), ids.astype(np.int32), tei.astype(np.int32)


def _sigmoid(x):
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def grouped_topk(gating, topk, num_expert_group, topk_group, renormalize,
                 is_softmax=True, routed_scaling_factor=1.0):
    x = np.asarray(gating, dtype=np.float32)
    M, E = x.shape
    if is_softmax:
        mx = x.max(axis=-1, keepdims=True)
        e = np.exp(x - mx).astype(np.float32)
        scores = (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
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
        w = w / w.sum(axis=-1, keepdims=True, dtype=np.float32)
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
        w = w / w.sum(axis=-1, keepdims=True, dtype=np.float32)
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
    w = (np.float32(1.0) / (np.float32(1.0) + np.exp(-v))).astype(np.float32)
    return w, ids
