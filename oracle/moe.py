"""Fused-MoE math restated in numpy (test infrastructure only).

The pipeline is the reference's 2-stage torch path as its test drives it
(op_tests/test_moe_2stage.py:187-231):

1. activations quantised 1x128 to fp8 (`pertoken_quant`, aiter/ops/quant.py:42);
2. `torch_moe_stage1` (aiter/fused_moe.py:1483-1585): dequantise, per-expert
   `x @ w1[e].T`, then act(gate) * up with gate = first I columns (:1578-1582),
   cast to bf16;
3. 1x128 requant of the bf16 intermediate (op_tests/test_moe_2stage.py:203-207);
4. `torch_moe_stage2` (aiter/fused_moe.py:1588-1666): dequantise, per-expert
   `a2 @ w2[e].T`, multiply by the top-k weight, sum over the k slots, cast to bf16.

Weights are either fp8 with 128x128 fp32 block scales (QuantType.per_1x128) or
MXFP4 with e8m0 scales per 32 along K (the A8W4 contract: fp8 1x128 activations
and intermediate, MXFP4 weights).
"""
import numpy as np

from . import codecs, quant

F32 = np.float32


def silu(x):
    x = np.asarray(x, dtype=F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def gelu(x):
    from math import sqrt
    import numpy as _np
    x = _np.asarray(x, dtype=_np.float64)
    from scipy.special import erf  # exact-erf gelu, torch F.gelu default
    return (0.5 * x * (1.0 + erf(x / sqrt(2.0)))).astype(F32)


def swiglu(gate, up, alpha=1.702, limit=7.0):
    """`swiglu` (aiter/fused_moe.py:1473-1480): clamp(gate, max=7) * sigmoid(1.702 *
    that) * (clamp(up, -7, 7) + 1), in fp32."""
    g = np.minimum(np.asarray(gate, dtype=F32), F32(limit))
    u = np.clip(np.asarray(up, dtype=F32), F32(-limit), F32(limit))
    return (g * (F32(1.0) / (F32(1.0) + np.exp(-F32(alpha) * g))) * (u + F32(1.0))).astype(F32)


def round_to(x, dtype):
    """Round f32 values to bf16 or fp16 (RNE), returned as f32."""
    if dtype == "fp16":
        return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)
    return codecs.round_bf16(x)


def stage1(a_deq, w1_deq, topk_ids, activation="silu", expert_list=None, topk_weights=None, dtype="bf16",
           bias=None):
    """a_deq: [M, D] f32, w1_deq: callable e -> [2I, D] f32 (or array [E,2I,D]).
    With `topk_weights` the GEMM output is multiplied by the token's top-k weight
    before the activation (doweight, aiter/fused_moe.py:1569-1570); `bias` [E, 2I] is
    then added (w1_bias, :1572-1573).  Returns f32 [M, k, I] rounded to `dtype` (bf16
    or fp16)."""
    M, k = topk_ids.shape
    get_w = w1_deq if callable(w1_deq) else (lambda e: w1_deq[e])
    E = int(topk_ids.max()) + 1 if expert_list is None else None
    experts = np.unique(topk_ids) if expert_list is None else expert_list
    out = None
    for e in experts:
        tok, slot = np.nonzero(topk_ids == e)
        if tok.size == 0:
            continue
        w = get_w(int(e))
        h = a_deq[tok] @ w.T
        if topk_weights is not None:
            h = (h * np.asarray(topk_weights, dtype=F32)[tok, slot][:, None]).astype(F32)
        if bias is not None:
            h = (h + np.asarray(bias, dtype=F32)[int(e)][None, :]).astype(F32)
        if out is None:
            out = np.zeros((M, k, w.shape[0]), dtype=F32)
        out[tok, slot] = h
    if out is None:
        raise ValueError("no routed tokens")
    inter = out.shape[-1] // 2
    gate, up = out[..., :inter], out[..., inter:]
    if activation == "swiglu":
        y = swiglu(gate, up)
    else:
        y = (silu(gate) if activation == "silu" else gelu(gate)) * up
    return round_to(np.asarray(y, dtype=F32), dtype)


def stage2(a2_deq, w2_deq, topk_weights, topk_ids, expert_list=None, doweight=True, dtype="bf16", bias=None):
    """a2_deq: [M, k, I] f32; w2_deq: callable e -> [D, I] or array [E, D, I].
    `bias` [E, D] is added to each expert's output before the top-k weight (w2_bias,
    aiter/fused_moe.py:1662-1665).  Returns f32 [M, D] rounded to `dtype`;
    `doweight=False` when stage 1 applied the top-k weights."""
    M, k = topk_ids.shape
    get_w = w2_deq if callable(w2_deq) else (lambda e: w2_deq[e])
    experts = np.unique(topk_ids) if expert_list is None else expert_list
    out = None
    for e in experts:
        tok, slot = np.nonzero(topk_ids == e)
        if tok.size == 0:
            continue
        w = get_w(int(e))
        y = a2_deq[tok, slot] @ w.T
        if bias is not None:
            y = (y + np.asarray(bias, dtype=F32)[int(e)][None, :]).astype(F32)
        if out is None:
            out = np.zeros((M, k, w.shape[0]), dtype=F32)
        out[tok, slot] = y
    if doweight:
        out = out * np.asarray(topk_weights, dtype=F32)[:, :, None]
    return round_to(out.sum(axis=1, dtype=F32), dtype)


def fused_moe_fp8_blockscale(hidden, w1_q, w1_s, w2_q, w2_s, topk_weights, topk_ids,
                             activation="silu", return_intermediate=False, doweight_stage1=False, dtype="bf16",
                             bias1=None, bias2=None):
    """QuantType.per_1x128 end to end. hidden: [M, D] bf16 (or fp16) values (f32 array);
    `dtype` is the activation / intermediate / output type; bias1 [E, 2I] / bias2
    [E, D] the experts' biases of the two GEMMs."""
    a1_q, a1_s = quant.per_1x128_quant(hidden)
    a1 = quant.dequant_1x128(a1_q, a1_s)
    w1 = lambda e: quant.dequant_128x128(w1_q[e:e + 1], w1_s[e:e + 1])[0]
    w2 = lambda e: quant.dequant_128x128(w2_q[e:e + 1], w2_s[e:e + 1])[0]
    out1 = stage1(a1, w1, topk_ids, activation, topk_weights=topk_weights if doweight_stage1 else None,
                  dtype=dtype, bias=bias1)
    a2_q, a2_s = quant.per_1x128_quant(out1)
    a2 = quant.dequant_1x128(a2_q, a2_s)
    out = stage2(a2, w2, topk_weights, topk_ids, doweight=not doweight_stage1, dtype=dtype, bias=bias2)
    if return_intermediate:
        return out, dict(a1_q=a1_q, a1_s=a1_s, out1=out1, a2_q=a2_q, a2_s=a2_s)
    return out


def fused_moe_a8w4(hidden, w1_p, w1_e, w2_p, w2_e, topk_weights, topk_ids,
                   activation="silu", return_intermediate=False, bias1=None, bias2=None):
    """A8W4 as BASELINE defines it: fp8 1x128 activations, MXFP4 weights; with
    Swiglu the reference's per_1x32 path also takes the experts' biases."""
    a1_q, a1_s = quant.per_1x128_quant(hidden)
    a1 = quant.dequant_1x128(a1_q, a1_s)
    w1 = lambda e: quant.dequant_mxfp4(w1_p[e], w1_e[e])
    w2 = lambda e: quant.dequant_mxfp4(w2_p[e], w2_e[e])
    out1 = stage1(a1, w1, topk_ids, activation, bias=bias1)
    a2_q, a2_s = quant.per_1x128_quant(out1)
    a2 = quant.dequant_1x128(a2_q, a2_s)
    out = stage2(a2, w2, topk_weights, topk_ids, bias=bias2)
    if return_intermediate:
        return out, dict(a1_q=a1_q, a1_s=a1_s, out1=out1, a2_q=a2_q, a2_s=a2_s)
    return out


def fused_moe_fp8_blockscale_threaded(hidden, w1_q, w1_s, w2_q, w2_s, topk_weights, topk_ids,
                                      threads=None, activation="silu", doweight=True, dtype="bf16"):
    """Same arithmetic as `fused_moe_fp8_blockscale`, experts processed by a thread
    pool (numpy releases the GIL in the decode and the matmuls).  Used as the timed
    CPU baseline; every call dequantises the weights of every routed expert, as the
    reference torch path does on each call (aiter/fused_moe.py:1502-1536)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    threads = threads or os.cpu_count() or 1
    M, k = topk_ids.shape
    a1_q, a1_s = quant.per_1x128_quant(hidden)
    a1 = quant.dequant_1x128(a1_q, a1_s)
    experts = [int(e) for e in np.unique(topk_ids)]
    inter = w2_q.shape[2]
    D = w2_q.shape[1]
    out1 = np.zeros((M, k, inter), dtype=F32)

    def s1(e):
        tok, slot = np.nonzero(topk_ids == e)
        w = quant.dequant_128x128(w1_q[e:e + 1], w1_s[e:e + 1])[0]
        h = a1[tok] @ w.T
        g, u = h[:, :inter], h[:, inter:]
        act = silu(g) if activation == "silu" else gelu(g)
        out1[tok, slot] = codecs.round_bf16((act * u).astype(F32))

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(s1, experts))
    a2_q, a2_s = quant.per_1x128_quant(out1)
    a2 = quant.dequant_1x128(a2_q, a2_s)
    out = np.zeros((M, k, D), dtype=F32)

    def s2(e):
        tok, slot = np.nonzero(topk_ids == e)
        w = quant.dequant_128x128(w2_q[e:e + 1], w2_s[e:e + 1])[0]
        out[tok, slot] = a2[tok, slot] @ w.T

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(s2, experts))
    if doweight:
        out = out * np.asarray(topk_weights, dtype=F32)[:, :, None]
    return round_to(out.sum(axis=1, dtype=F32), dtype)


def moe_sum(x, dtype="bf16"):
    """`moe_sum` (aiter/ops/moe_op.py:45-46, csrc/kernels/topk_softmax_kernels.cu:737-854):
    [M, k, D] -> [M, D].  For k = 2, 4, 5 the reference's kernel adds slot by slot in the
    element type (one rounding per add); other k go through at::sum_out (fp32
    accumulation, one rounding).  `dtype`: "fp32", "bf16" or "fp16"."""
    x = np.asarray(x, dtype=F32)
    k = x.shape[1]
    rnd = (lambda a: a.astype(F32)) if dtype == "fp32" else (lambda a: round_to(a, dtype))
    acc = np.zeros((x.shape[0], x.shape[2]), dtype=F32)
    for s in range(k):
        acc = (acc + x[:, s]).astype(F32)
        if k in (2, 4, 5):
            acc = rnd(acc)
    return rnd(acc)
