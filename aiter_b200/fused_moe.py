"""Fused-MoE front door with the reference's Python surface (aiter/fused_moe.py).

* `fused_moe(...)`      aiter/fused_moe.py:118-169 (same signature and defaults)
* `moe_sorting(...)`    aiter/fused_moe.py:70-103
* `fused_topk(...)`     aiter/fused_moe.py:1853-1923
* `get_inter_dim`, `get_padded_M`  aiter/fused_moe.py:108-115,606-612

The per_1x128 (== per_128x128, aiter/fused_moe.py:597) path runs four kernels of
libaiter_b200.so on the current stream, with no host synchronisation:
moe_sorting_fwd (also zeroes the output) -> 1x128 fp8 activation quant ->
stage-1 grouped GEMM (gate/up, act, fp8 requant fused) -> stage-2 grouped GEMM
(top-k weighted scatter-add into the output).  Weights are taken unshuffled
([E, 2I, D] / [E, D, I], K contiguous); AMD pre-shuffled weights
(`is_shuffled=True`, aiter/ops/shuffle.py:7-27) are rejected.
"""
import functools
from dataclasses import dataclass
from typing import Optional

import torch

from . import dtypes, moe_op
from .enums import ActivationType, QuantType

BLOCK_SIZE_M = 128

quant_remap = {QuantType.per_128x128: QuantType.per_1x128}


@functools.lru_cache(maxsize=2048)
def get_inter_dim(w1_shape, w2_shape):
    """(E, model_dim, inter_dim); the fp4x2 packing of w1's K is undone
    (aiter/fused_moe.py:108-115)."""
    E, _, model_dim = w1_shape
    E, model_dim, inter_dim = w2_shape
    int4_war = model_dim // w1_shape[-1]
    inter_dim *= int4_war
    return E, model_dim, inter_dim


def nextPow2(n):
    if n <= 1:
        return 1
    return 1 << (n - 1).bit_length()


def get_padded_M(M):
    return nextPow2(M) if M < 32768 else 32768


@dataclass
class MOEMetadata:
    """Kernel choice for one problem shape (the role of MOEMetadata,
    aiter/fused_moe.py:615-624).  One tcgen05 kernel family serves every shape
    here, so only the sort unit varies."""
    block_m: int
    ksplit: int = 0
    run_1stage: bool = False


@functools.lru_cache(maxsize=2048)
def get_2stage_cfgs(padded_M, model_dim, inter_dim, expert, topk, dtype, q_dtype_a, q_dtype_w,
                    q_type, use_g1u1, activation, doweight_stage1):
    """Frozen heuristic table (replaces the tuned-CSV lookup of
    aiter/fused_moe.py:719-911): the grouped GEMM tiles 128 sorted rows."""
    return MOEMetadata(block_m=BLOCK_SIZE_M)


def moe_sorting(topk_ids, topk_weights, num_experts, model_dim, moebuf_dtype, block_size=BLOCK_SIZE_M,
                expert_mask=None, num_local_tokens=None, dispatch_policy=0):
    """Returns (sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf);
    moe_buf [M, model_dim] is zeroed."""
    device = topk_ids.device
    M, topk = topk_ids.shape
    max_num_tokens_padded = int(topk_ids.numel() + num_experts * block_size - topk)
    max_num_m_blocks = int((max_num_tokens_padded + block_size - 1) // block_size)
    sorted_ids = torch.empty(max_num_tokens_padded, dtype=dtypes.i32, device=device)
    sorted_weights = torch.empty(max_num_tokens_padded, dtype=dtypes.fp32, device=device)
    sorted_expert_ids = torch.empty(max_num_m_blocks, dtype=dtypes.i32, device=device)
    num_valid_ids = torch.empty(2, dtype=dtypes.i32, device=device)
    moe_buf = torch.empty((M, model_dim), dtype=moebuf_dtype, device=device)
    moe_op.moe_sorting_fwd(topk_ids, topk_weights, sorted_ids, sorted_weights, sorted_expert_ids,
                           num_valid_ids, moe_buf, num_experts, int(block_size), expert_mask,
                           num_local_tokens, dispatch_policy)
    return sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf


def fused_topk(hidden_states, gating_output, topk, renormalize, topk_ids=None, topk_weights=None):
    assert hidden_states.shape[0] == gating_output.shape[0], "Number of tokens mismatch"
    M = hidden_states.shape[0]
    dev = hidden_states.device
    token_expert_indicies = torch.empty(M, topk, dtype=dtypes.i32, device=dev)
    if topk_weights is None:
        topk_weights = torch.empty(M, topk, dtype=dtypes.fp32, device=dev)
    if topk_ids is None:
        topk_ids = torch.empty(M, topk, dtype=dtypes.i32, device=dev)
    moe_op.topk_softmax(topk_weights, topk_ids, token_expert_indicies, gating_output, renormalize)
    return topk_weights, topk_ids


def fused_moe(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask: Optional[torch.Tensor] = None,
              activation=ActivationType.Silu, quant_type=QuantType.No, doweight_stage1=False,
              w1_scale: Optional[torch.Tensor] = None, w2_scale: Optional[torch.Tensor] = None,
              a1_scale: Optional[torch.Tensor] = None, a2_scale: Optional[torch.Tensor] = None,
              block_size_M=None, num_local_tokens: Optional[torch.Tensor] = None,
              moe_sorting_dispatch_policy=0, dtype=None, hidden_pad=0, intermediate_pad=0,
              bias1=None, bias2=None, splitk=0):
    activation = ActivationType(int(activation))
    quant_type = quant_remap.get(QuantType(int(quant_type)), QuantType(int(quant_type)))
    M, topk = topk_ids.shape
    E, model_dim, inter_dim = get_inter_dim(tuple(w1.shape), tuple(w2.shape))
    assert w1.shape[1] in (inter_dim, inter_dim * 2), f"Invalid MoE weight: {w1.shape=} {w2.shape=}"
    is_g1u1 = w1.shape[1] == 2 * inter_dim
    if getattr(w1, "is_shuffled", False) or getattr(w2, "is_shuffled", False):
        raise ValueError("pre-shuffled (AMD MFMA layout) weights are not accepted; pass [E, N, K] weights")
    dtype = hidden_states.dtype if dtype is None else dtype
    if dtype == dtypes.fp8:          # pre-quantised input: output defaults to bf16
        dtype = dtypes.bf16
    assert dtype in (dtypes.bf16, dtypes.fp16), f"Fused_moe unsupported out dtype: {dtype}"
    if dtype != dtypes.bf16:
        raise NotImplementedError("the B200 path writes bf16 outputs")
    if not is_g1u1:
        raise NotImplementedError("only gate+up (g1u1) MoE weights are supported")
    if activation not in (ActivationType.Silu, ActivationType.Gelu):
        raise NotImplementedError(f"activation {activation} not supported")
    if bias1 is not None or bias2 is not None or hidden_pad or intermediate_pad:
        raise NotImplementedError("bias / padding variants are not supported")
    if doweight_stage1:
        raise NotImplementedError("doweight_stage1 is not supported")
    global_E = expert_mask.numel() if expert_mask is not None else E
    if quant_type == QuantType.per_1x128:
        if w1.dtype != dtypes.fp8 or w2.dtype != dtypes.fp8:
            raise TypeError("per_1x128 needs fp8 weights")
        meta = get_2stage_cfgs(get_padded_M(M), model_dim, inter_dim, E, topk, dtype, dtypes.fp8,
                               w1.dtype, quant_type, True, activation, doweight_stage1)
        block_m = meta.block_m if not block_size_M else int(block_size_M)
        if block_m != BLOCK_SIZE_M:
            raise NotImplementedError(f"block_size_M={block_m}: the grouped GEMM tiles {BLOCK_SIZE_M} rows")
        sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf = moe_sorting(
            topk_ids, topk_weight, global_E, model_dim, dtype, block_m, expert_mask, num_local_tokens,
            moe_sorting_dispatch_policy)
        if hidden_states.dtype == dtypes.fp8 and a1_scale is not None:
            a1 = hidden_states
        else:
            a1, a1_scale = moe_op.per_group_quant_hip(hidden_states, quant_dtype=dtypes.fp8, group_size=128,
                                                      num_rows=num_local_tokens)
        a2 = torch.empty((M, topk, inter_dim), dtype=dtypes.fp8, device=hidden_states.device)
        a2_scale = torch.empty((M * topk, inter_dim // 128), dtype=dtypes.fp32, device=hidden_states.device)
        moe_op.moe_stage1_fp8_blockscale(a1, w1, sorted_ids, sorted_expert_ids, num_valid_ids, a2, a2_scale,
                                         topk, w1_scale, a1_scale, block_m, activation)
        moe_op.moe_stage2_fp8_blockscale(a2, w2, sorted_ids, sorted_expert_ids, num_valid_ids, moe_buf, topk,
                                         w2_scale, a2_scale, sorted_weights, block_m)
        return moe_buf
    raise NotImplementedError(f"quant_type {quant_type} is not supported by the B200 path")
