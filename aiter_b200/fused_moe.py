"""Fused-MoE front door with the reference's Python surface (aiter/fused_moe.py).

* `fused_moe(...)`      aiter/fused_moe.py:118-169 (same signature and defaults)
* `moe_sorting(...)`    aiter/fused_moe.py:70-103
* `fused_topk(...)`     aiter/fused_moe.py:1853-1923
* `get_inter_dim`, `get_padded_M`  aiter/fused_moe.py:108-115,606-612

The per_1x128 (== per_128x128, aiter/fused_moe.py:597) path runs four kernels of
libaiter_b200.so on the current stream (five launches when sorting takes its
multi-CTA form), with no host synchronisation: moe_sorting_fwd (also zeroes the
output) -> gather + 1x128 fp8 activation quant into sorted-row order -> stage-1
grouped GEMM (gate/up, act, fp8 requant fused; sorted rows out) -> stage-2
grouped GEMM (top-k weighted scatter-add into the output).  Options: Silu / Gelu /
Swiglu, doweight_stage1, bf16 or fp16 activations and output.  Weights are taken unshuffled
([E, 2I, D] / [E, D, I], K contiguous); AMD pre-shuffled weights
(`is_shuffled=True`, aiter/ops/shuffle.py:7-27) are rejected.
"""
import functools
import os
from dataclasses import dataclass
from typing import Optional

import torch

from . import dtypes, moe_op
from .enums import ActivationType, QuantType

# The reference's module default sort unit (aiter/fused_moe.py:22): the default block_size
# of the public moe_sorting.  The tcgen05 grouped GEMMs tile GEMM_BLOCK_M sorted rows, so
# fused_moe sorts with that unit.
BLOCK_SIZE_M = 32
GEMM_BLOCK_M = 128

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


@functools.lru_cache(maxsize=2048)
def get_block_size_M(token, topk, expert, inter_dim):
    """Sort unit for a problem (aiter/fused_moe.py:514-529 balances 32/64/128-row tiles over
    the CUs).  The tcgen05 grouped GEMM tiles 128 sorted rows (64-row half tiles are
    chosen inside the kernel), so the unit is always 128."""
    return GEMM_BLOCK_M


@functools.lru_cache(maxsize=2048)
def use_nt(token, topk, e):
    """The reference's non-temporal-load switch (aiter/fused_moe.py:531-537), same rule and
    AITER_USE_NT override; the B200 kernels stream weights through TMA either way."""
    v = int(os.environ.get("AITER_USE_NT", "-1"))
    if v != -1:
        return bool(v)
    return (token * topk // e) < 64


@functools.lru_cache(maxsize=2048)
def get_ksplit(token, topk, expert, inter_dim, model_dim):
    """Split-K factor (aiter/fused_moe.py:539-567 splits decode-size stage 1 over idle
    CUs).  The B200 stage 1 does not split K: always 0."""
    return 0


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
    return MOEMetadata(block_m=GEMM_BLOCK_M)


def _moe_sorting_ext(topk_ids, topk_weights, num_experts, model_dim, moebuf_dtype, block_size,
                     expert_mask=None, num_local_tokens=None, dispatch_policy=0, with_pos=False, moe_buf=None):
    device = topk_ids.device
    M, topk = topk_ids.shape
    max_num_tokens_padded = int(topk_ids.numel() + num_experts * block_size - topk)
    max_num_m_blocks = int((max_num_tokens_padded + block_size - 1) // block_size)
    sorted_ids = torch.empty(max_num_tokens_padded, dtype=dtypes.i32, device=device)
    sorted_weights = torch.empty(max_num_tokens_padded, dtype=dtypes.fp32, device=device)
    sorted_expert_ids = torch.empty(max_num_m_blocks, dtype=dtypes.i32, device=device)
    num_valid_ids = torch.empty(2, dtype=dtypes.i32, device=device)
    if moe_buf is None:
        moe_buf = torch.empty((M, model_dim), dtype=moebuf_dtype, device=device)
    pos = torch.empty(M * topk, dtype=dtypes.i32, device=device) if with_pos else None
    moe_op.moe_sorting_fwd(topk_ids, topk_weights, sorted_ids, sorted_weights, sorted_expert_ids,
                           num_valid_ids, moe_buf, num_experts, int(block_size), expert_mask,
                           num_local_tokens, dispatch_policy, token_sorted_pos=pos)
    return sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf, pos


def moe_sorting(topk_ids, topk_weights, num_experts, model_dim, moebuf_dtype, block_size=BLOCK_SIZE_M,
                expert_mask=None, num_local_tokens=None, dispatch_policy=0):
    """Returns (sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf);
    moe_buf [M, model_dim] is zeroed."""
    return _moe_sorting_ext(topk_ids, topk_weights, num_experts, model_dim, moebuf_dtype, block_size,
                            expert_mask, num_local_tokens, dispatch_policy)[:5]


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
              bias1=None, bias2=None, splitk=0, moe_buf=None):
    """Reference signature (aiter/fused_moe.py:118-144) plus `moe_buf`: an optional
    [M, model_dim] bf16 output to write into (e.g. the staging buffer of the
    tensor-parallel allreduce); it is zeroed and filled like the returned buffer.

    While torch is compiling, the call goes through the custom op
    `torch.ops.aiter_b200.fused_moe_` (fake implementation in torch_ops.py), as
    the reference's `fused_moe` goes through `fused_moe_`."""
    plain = (block_size_M is None and dtype is None and not hidden_pad and not intermediate_pad and bias1 is None
             and bias2 is None and not splitk and moe_buf is None)
    if plain and torch.compiler.is_compiling():
        from . import torch_ops  # noqa: F401  (registers the ops)
        return torch.ops.aiter_b200.fused_moe_(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask,
                                               int(activation), int(quant_type), bool(doweight_stage1), w1_scale,
                                               w2_scale, a1_scale, a2_scale, num_local_tokens,
                                               int(moe_sorting_dispatch_policy))
    return _fused_moe_impl(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask, activation, quant_type,
                           doweight_stage1, w1_scale, w2_scale, a1_scale, a2_scale, block_size_M, num_local_tokens,
                           moe_sorting_dispatch_policy, dtype, hidden_pad, intermediate_pad, bias1, bias2, splitk,
                           moe_buf)


def _fused_moe_impl(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask=None, activation=ActivationType.Silu,
                    quant_type=QuantType.No, doweight_stage1=False, w1_scale=None, w2_scale=None, a1_scale=None,
                    a2_scale=None, block_size_M=None, num_local_tokens=None, moe_sorting_dispatch_policy=0,
                    dtype=None, hidden_pad=0, intermediate_pad=0, bias1=None, bias2=None, splitk=0, moe_buf=None):
    activation = ActivationType(int(activation))
    quant_type = quant_remap.get(QuantType(int(quant_type)), QuantType(int(quant_type)))
    M, topk = topk_ids.shape
    E, model_dim, inter_dim = get_inter_dim(tuple(w1.shape), tuple(w2.shape))
    assert w1.shape[1] in (inter_dim, inter_dim * 2), f"Invalid MoE weight: {w1.shape=} {w2.shape=}"
    is_g1u1 = w1.shape[1] == 2 * inter_dim
    if getattr(w1, "is_shuffled", False) or getattr(w2, "is_shuffled", False):
        raise ValueError("pre-shuffled (AMD MFMA layout) weights are not accepted; pass [E, N, K] weights "
                         "(aiter_b200.weights.unshuffle_weight undoes shuffle_weight once)")
    dtype = hidden_states.dtype if dtype is None else dtype
    if dtype == dtypes.fp8:          # pre-quantised input: output defaults to bf16
        dtype = dtypes.bf16
    assert dtype in (dtypes.bf16, dtypes.fp16), f"Fused_moe unsupported out dtype: {dtype}"
    if not is_g1u1:
        raise NotImplementedError("only gate+up (g1u1) MoE weights are supported")
    if activation not in (ActivationType.Silu, ActivationType.Gelu, ActivationType.Swiglu):
        raise NotImplementedError(f"activation {activation} not supported")
    # hidden_pad / intermediate_pad only tell the reference's cktile kernels which
    # trailing weight rows / columns are zero so that they can skip them
    # (aiter/fused_moe.py:985-1028); the weights are zero there, so the result is the
    # same without skipping.  The experts' biases are used, as in the reference, only by
    # the per_1x32 Swiglu path with bf16 / fp16 activations (aiter/fused_moe.py:985-1008,
    # 1228-1238); other configurations ignore them there and here.
    use_bias = (quant_type == QuantType.per_1x32 and activation == ActivationType.Swiglu
                and dtype in (dtypes.bf16, dtypes.fp16) and (bias1 is not None or bias2 is not None))
    b1 = b2 = None
    if use_bias:
        if bias1 is not None:
            b1 = bias1.to(device=hidden_states.device, dtype=dtypes.fp32).contiguous().view(E, -1)
            if b1.shape[1] != 2 * inter_dim:
                raise ValueError(f"bias1 must be [E, 2 * inter_dim], got {tuple(bias1.shape)}")
        if bias2 is not None:
            b2 = bias2.to(device=hidden_states.device, dtype=dtypes.fp32).contiguous().view(E, -1)
            if b2.shape[1] != model_dim:
                raise ValueError(f"bias2 must be [E, model_dim], got {tuple(bias2.shape)}")
    global_E = expert_mask.numel() if expert_mask is not None else E
    w4 = quant_type == QuantType.per_1x32
    if w4:
        # A8W4: fp8 1x128 activations x MXFP4 weights, which stay at 4 bits; their e8m0
        # scales are applied by the block-scaled MMA and are taken either as the
        # reference passes them, [E, N, K/32] (rearranged here by one small kernel),
        # or already as chunks (weights.prepare_a8w4_native, once).
        from . import weights as _w
        if w1.dtype not in (dtypes.fp4x2, torch.uint8) or w2.dtype not in (dtypes.fp4x2, torch.uint8):
            raise TypeError("per_1x32 needs MXFP4 (fp4x2) weights")
        if w1_scale is None or w2_scale is None:
            raise ValueError("per_1x32 needs the e8m0 scales w1_scale and w2_scale")
        if not _w.is_scale_chunks(w1_scale):
            w1_scale = _w.mxfp4_moe_weight_scale_chunks(w1_scale.view(E, w1.shape[1], -1))
        if not _w.is_scale_chunks(w2_scale):
            w2_scale = _w.mxfp4_moe_weight_scale_chunks(w2_scale.view(E, w2.shape[1], -1))
    if quant_type in (QuantType.per_1x128, QuantType.per_1x32):
        if not w4 and (w1.dtype != dtypes.fp8 or w2.dtype != dtypes.fp8):
            raise TypeError("per_1x128 needs fp8 weights")
        meta = get_2stage_cfgs(get_padded_M(M), model_dim, inter_dim, E, topk, dtype, dtypes.fp8,
                               w1.dtype, quant_type, True, activation, doweight_stage1)
        # block_size_M picks the tile height of the reference's kernels (16 / 32 / 64 / 128,
        # aiter/fused_moe.py:514-529); the result does not depend on it.  The tcgen05
        # grouped GEMM here always tiles 128 sorted rows (blocks whose rows 64.. are all
        # padding can run as M=64 tiles), so any of those values is accepted and mapped
        # to GEMM_BLOCK_M.
        if block_size_M and int(block_size_M) not in (16, 32, 64, 128):
            raise ValueError(f"block_size_M must be one of 16, 32, 64, 128, got {block_size_M}")
        block_m = GEMM_BLOCK_M
        sorted_ids, sorted_weights, sorted_expert_ids, num_valid_ids, moe_buf, pos = _moe_sorting_ext(
            topk_ids, topk_weight, global_E, model_dim, dtype, block_m, expert_mask, num_local_tokens,
            moe_sorting_dispatch_policy, with_pos=True, moe_buf=moe_buf)
        rows = sorted_ids.numel()
        dev = hidden_states.device
        if hidden_states.dtype == dtypes.fp8:
            if a1_scale is None:
                raise ValueError("a1_scale must be provided for quantized input for fused_moe")
            a1, a1s = moe_op.moe_gather_quant_1x128(hidden_states, pos, topk, rows, hidden_scale=a1_scale)
        else:
            a1, a1s = moe_op.moe_gather_quant_1x128(hidden_states, pos, topk, rows)
        a2 = torch.empty((rows, inter_dim), dtype=dtypes.fp8, device=dev)
        a2s = torch.empty((inter_dim // 128, rows), dtype=dtypes.fp32, device=dev)
        # doweight_stage1: the top-k weight scales the stage-1 GEMM output (before the
        # activation) and stage 2 adds unweighted rows (torch_moe_stage1/2 `doweight`)
        stage1 = moe_op.moe_stage1_a8w4 if w4 else moe_op.moe_stage1_fp8_blockscale
        stage2 = moe_op.moe_stage2_a8w4 if w4 else moe_op.moe_stage2_fp8_blockscale
        stage1(a1, a1s, w1, w1_scale, sorted_ids, sorted_expert_ids, num_valid_ids, a2, a2s, M, block_m, activation,
               sorted_weights=sorted_weights if doweight_stage1 else None, inter_dtype=dtype, bias=b1)
        stage2(a2, a2s, w2, w2_scale, sorted_ids, sorted_expert_ids, num_valid_ids,
               None if doweight_stage1 else sorted_weights, moe_buf, block_m, bias=b2)
        return moe_buf
    raise NotImplementedError(f"quant_type {quant_type} is not supported by the B200 path")
