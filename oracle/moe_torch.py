"""The reference's torch CPU MoE path, restated with torch CPU ops (TEST
INFRASTRUCTURE ONLY: the timed CPU baseline of `bench.py` and its CPU test).

The reference checks its fused MoE against a pure-torch pipeline
(op_tests/test_moe_2stage.py:187-231): 1x128 `pertoken_quant` of the activations
(aiter/ops/quant.py:42-72), `torch_moe_stage1` (aiter/fused_moe.py:1483-1585),
1x128 requant of the bf16 intermediate, `torch_moe_stage2`
(aiter/fused_moe.py:1588-1666).  That pipeline is the "reference torch CPU MoE
path" the benchmark times beside the GPU.  The reference checkout cannot be
imported on the GPU box, so this module does the same work with the same torch
operations, in the same order and at the same sizes:

* activations quantised to fp8 e4m3 per 128-element group (scale amax/448,
  0 -> 1), then dequantised to fp32 and replicated over the top-k slots into an
  [M, k, D] fp32 tensor (the reference's `.repeat(1, topk, 1)`, :1556);
* per expert: the expert's fp8 weights dequantised with their 128x128 block
  scales (the reference dequantises every expert before its loop, :1523-1530;
  here each expert is dequantised inside the loop, the same total work), a
  boolean mask over [M, k], the masked rows times the expert's weights in fp32,
  written back through the mask;
* act(gate) * up, cast to bf16; requant 1x128; the same per-expert loop for the
  down projection; the top-k weights multiplied in and the k slots summed in
  fp32; cast to bf16.

`experts` limits the per-expert loops to a subset of expert ids so that a
bounded sample of a large configuration can be timed; `timer` (a dict) then
receives the seconds spent inside the per-expert sections ("experts") and in
the shared sections ("shared"), so that the caller can scale the per-expert part
to all experts.  With `experts=None` every expert is processed and the result is
the reference pipeline's output.
"""
import time

import torch

FP8_MAX = 448.0


def quant_1x128(x):
    """pertoken_quant over 128-wide groups: x [..., K] -> (fp8 [..., K], f32 [..., K/128])."""
    x = x.to(torch.float32)
    shp = x.shape
    g = x.reshape(-1, 128)
    scale = g.abs().amax(dim=-1, keepdim=True) / FP8_MAX
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = (g / scale).to(torch.float8_e4m3fn).reshape(shp)
    return q, scale.reshape(*shp[:-1], shp[-1] // 128)


def dequant_1x128(q, s):
    shp = q.shape
    v = q.to(torch.float32).reshape(-1, 128) * s.reshape(-1, 1)
    return v.reshape(shp)


def dequant_128x128(wq, ws):
    """wq fp8 [N, K], ws f32 [N/128, K/128] -> f32 [N, K]."""
    N, K = wq.shape
    v = wq.to(torch.float32).reshape(N // 128, 128, K // 128, 128) * ws.reshape(N // 128, 1, K // 128, 1)
    return v.reshape(N, K)


def _silu(x):
    return torch.nn.functional.silu(x)


def fused_moe_fp8_blockscale(hidden, w1q, w1s, w2q, w2s, topk_weights, topk_ids, experts=None,
                             weight_of=None, timer=None):
    """hidden [M, D] bf16; w1q fp8 [Ew, 2I, D] + w1s f32 [Ew, 2I/128, D/128]; w2q fp8
    [Ew, D, I] + w2s f32 [Ew, D/128, I/128]; topk_weights f32 [M, k]; topk_ids int [M, k].
    `weight_of(e)` maps an expert id to its index in the weight tensors (identity
    by default).  Returns bf16 [M, D]."""
    t_shared = t_exp = 0.0
    t0 = time.perf_counter()
    M, D = hidden.shape
    k = topk_ids.shape[1]
    inter = w2q.shape[2]
    n_experts = int(topk_ids.max().item()) + 1 if experts is None else None
    expert_ids = range(n_experts) if experts is None else experts
    widx = weight_of or (lambda e: e)
    ids = topk_ids.to(torch.int64)

    a1q, a1s = quant_1x128(hidden)
    x = dequant_1x128(a1q, a1s)
    x = x.view(M, 1, D).repeat(1, k, 1)
    h = torch.zeros(M, k, 2 * inter, dtype=torch.float32)
    t_shared += time.perf_counter() - t0

    t0 = time.perf_counter()
    for e in expert_ids:
        mask = ids == e
        if not bool(mask.any()):
            continue
        w = dequant_128x128(w1q[widx(e)], w1s[widx(e)])
        h[mask] = x[mask] @ w.t()
    t_exp += time.perf_counter() - t0

    t0 = time.perf_counter()
    out1 = (_silu(h[..., :inter]) * h[..., inter:]).to(torch.bfloat16)
    a2q, a2s = quant_1x128(out1.view(M, k, inter))
    y_in = dequant_1x128(a2q, a2s)
    y = torch.zeros(M, k, D, dtype=torch.float32)
    t_shared += time.perf_counter() - t0

    t0 = time.perf_counter()
    for e in expert_ids:
        mask = ids == e
        if not bool(mask.any()):
            continue
        w = dequant_128x128(w2q[widx(e)], w2s[widx(e)])
        y[mask] = y_in[mask] @ w.t()
    t_exp += time.perf_counter() - t0

    t0 = time.perf_counter()
    out = (y * topk_weights.to(torch.float32).view(M, k, 1)).sum(dim=1).to(torch.bfloat16)
    t_shared += time.perf_counter() - t0
    if timer is not None:
        timer["shared"] = timer.get("shared", 0.0) + t_shared
        timer["experts"] = timer.get("experts", 0.0) + t_exp
    return out


def route_softmax_topk(logits, k):
    """The reference's torch routing (op_tests/test_moeTopkSoftmax.py:21-41): softmax
    over the experts in fp32, top-k, renormalise."""
    p = torch.softmax(logits.to(torch.float32), dim=-1)
    w, i = torch.topk(p, k, dim=-1)
    return w / w.sum(dim=-1, keepdim=True), i.to(torch.int32)


def quant_weight_128x128(w):
    """128x128 block quantiser of op_tests/test_moe_2stage.py:84-110 (amax/448 per block):
    w f32 [E, N, K] -> (fp8 [E, N, K], f32 [E, N/128, K/128])."""
    E, N, K = w.shape
    blk = w.reshape(E, N // 128, 128, K // 128, 128)
    scale = blk.abs().amax(dim=(2, 4), keepdim=True) / FP8_MAX
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = (blk / scale).to(torch.float8_e4m3fn).reshape(E, N, K)
    return q, scale.reshape(E, N // 128, K // 128)
