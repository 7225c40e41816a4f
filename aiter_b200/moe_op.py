"""Operator stubs of the path, same names and argument meaning as the reference's
`@compile_ops` stubs, each calling one C-ABI entry point of libaiter_b200.so.

Reference stubs:
* topk_softmax              aiter/ops/moe_op.py:15-24
* grouped_topk              aiter/ops/topk.py:28-38
* biased_grouped_topk       aiter/ops/topk.py:75-113 (the HIP / moe_fused_gate
                            split of :87-113 is one kernel here)
* moe_sorting_fwd           aiter/ops/moe_sorting.py:11-24
* dynamic_per_token_scaled_quant  aiter/ops/quant.py:473-481
* per_group_quant_hip       aiter/ops/quant.py:261-292
* ck_moe_stage1_fwd / ck_moe_stage2_fwd  aiter/ops/moe_op.py:534-615 -> here
  moe_stage1_fp8_blockscale (with the fused fp8 requant) / moe_stage2_fp8_blockscale
"""
from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _lib, dtypes
from .enums import ActivationType


def topk_softmax(topk_weights: Tensor, topk_indices: Tensor, token_expert_indices: Tensor,
                 gating_output: Tensor, need_renorm: bool, num_shared_experts: int = 0,
                 shared_expert_scoring_func: str = "") -> None:
    _lib.call("topk_softmax", topk_weights, topk_indices, token_expert_indices, gating_output,
              need_renorm, num_shared_experts, shared_expert_scoring_func)


def grouped_topk(gating_output: Tensor, topk_weights: Tensor, topk_ids: Tensor, num_expert_group: int,
                 topk_group: int, need_renorm: bool, is_softmax: bool = True,
                 routed_scaling_factor: float = 1.0) -> None:
    _lib.call("grouped_topk", gating_output, topk_weights, topk_ids, num_expert_group, topk_group,
              need_renorm, is_softmax, routed_scaling_factor)


def biased_grouped_topk(gating_output: Tensor, correction_bias: Tensor, topk_weights: Tensor,
                        topk_ids: Tensor, num_expert_group: int, topk_group: int, need_renorm: bool,
                        routed_scaling_factor: float = 1.0) -> None:
    _lib.call("biased_grouped_topk", gating_output, correction_bias, topk_weights, topk_ids,
              num_expert_group, topk_group, need_renorm, routed_scaling_factor)


biased_grouped_topk_hip = biased_grouped_topk


def moe_sorting_get_workspace_size(num_tokens: int, num_experts: int, topk: int,
                                   dispatch_policy: int = 0) -> int:
    return int(_lib.lib().moe_sorting_get_workspace_size(num_tokens, num_experts, topk, dispatch_policy))


def moe_sorting_fwd(topk_ids: Tensor, topk_weights: Tensor, sorted_token_ids: Tensor,
                    sorted_weights: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                    moe_buf: Tensor, num_experts: int, unit_size: int,
                    local_expert_mask: Optional[Tensor] = None,
                    num_local_tokens: Optional[Tensor] = None, dispatch_policy: int = 0,
                    workspace: Optional[Tensor] = None, token_sorted_pos: Optional[Tensor] = None) -> None:
    """In place.  Allocates the workspace itself when none is given, as the
    reference binding does (csrc/py_itfs_ck/moe_sorting_kernels.cu:33-40)."""
    M, topk = topk_ids.shape
    if workspace is None:
        ws = moe_sorting_get_workspace_size(M, num_experts, topk, dispatch_policy)
        if ws > 0:
            workspace = torch.empty(ws, dtype=torch.uint8, device=topk_ids.device)
    _lib.call("moe_sorting_fwd", topk_ids, topk_weights, sorted_token_ids, sorted_weights,
              sorted_expert_ids, num_valid_ids, moe_buf, num_experts, unit_size,
              local_expert_mask, num_local_tokens, dispatch_policy, workspace, token_sorted_pos)


def moe_sorting_opus_fwd(topk_ids: Tensor, topk_weights: Tensor, sorted_token_ids: Tensor,
                         sorted_weights: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                         moe_buf: Tensor, num_experts: int, unit_size: int,
                         local_expert_mask: Optional[Tensor] = None, num_local_tokens: Optional[Tensor] = None,
                         dispatch_policy: int = 0) -> None:
    """aiter.moe_sorting_opus_fwd (aiter/ops/moe_sorting_opus.py:12-25): the opus sorting
    kernel has the same contract as moe_sorting_fwd (csrc/include/moe_sorting_opus.h:274-322),
    so both names run the same kernels here."""
    moe_sorting_fwd(topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids, num_valid_ids,
                    moe_buf, num_experts, unit_size, local_expert_mask, num_local_tokens, dispatch_policy)


def dynamic_per_token_scaled_quant(out: Tensor, input: Tensor, scales: Tensor,
                                   scale_ub: Optional[Tensor] = None, shuffle_scale: bool = False,
                                   num_rows: Optional[Tensor] = None, num_rows_factor: int = 1) -> None:
    _lib.call("dynamic_per_token_scaled_quant", out, input, scales, scale_ub, shuffle_scale,
              num_rows, num_rows_factor)


def per_group_quant_hip(x: Tensor, scale: Optional[Tensor] = None, quant_dtype=dtypes.i8,
                        group_size: int = 128, transpose_scale: bool = False,
                        num_rows: Optional[Tensor] = None, num_rows_factor: int = 1) -> Tuple[Tensor, Tensor]:
    """1 x group_size dynamic quantisation -> (fp8 or int8 [.., K], f32 scales [.., K/group]).
    The default output dtype is the reference's, int8 (aiter/ops/quant.py:261-264); the
    MoE path passes fp8."""
    if scale is not None:
        raise ValueError("unsupported: static per group quant")
    if quant_dtype not in (dtypes.fp8, dtypes.i8):
        raise ValueError(f"unsupported quant dtype {quant_dtype}")
    if group_size not in (32, 64, 128):
        raise ValueError(f"unsupported group size {group_size=}, only support [32, 64, 128]")
    shape = x.shape
    x = x.contiguous()
    scale = torch.empty((*shape[:-1], shape[-1] // group_size), dtype=dtypes.fp32, device=x.device)
    y = torch.empty(shape, dtype=quant_dtype, device=x.device)
    dynamic_per_token_scaled_quant(y, x.view(-1, group_size), scale, shuffle_scale=transpose_scale,
                                   num_rows=num_rows, num_rows_factor=num_rows_factor)
    return y, scale


def dynamic_per_group_scaled_quant_fp4(out: Tensor, input: Tensor, scales: Tensor, group_size: int = 32,
                                       shuffle_scale: bool = True, num_rows: Optional[Tensor] = None,
                                       num_rows_factor: int = 1) -> None:
    """MXFP4 quant of `input` rows (aiter/ops/quant.py:485-497): fp4x2 codes into `out`,
    one e8m0 scale per 32 elements into `scales` (row order, or the e8m0_shuffle layout
    when `shuffle_scale`).  Rows from num_rows[0] * num_rows_factor on are skipped."""
    _lib.call("dynamic_per_group_scaled_quant_fp4", out, input, scales, group_size, shuffle_scale, num_rows,
              num_rows_factor)


def per_1x32_f4_quant_hip(x: Tensor, scale: Optional[Tensor] = None, quant_dtype=dtypes.fp4x2, shuffle: bool = False,
                          num_rows: Optional[Tensor] = None, num_rows_factor: int = 1) -> Tuple[Tensor, Tensor]:
    """(fp4x2 [m, n/2], e8m0 scales) of x [m, n] (aiter/ops/quant.py:295-343)."""
    m, n = x.shape
    assert quant_dtype == dtypes.fp4x2
    assert n % 2 == 0
    if scale is not None:
        raise ValueError("unsupported: static per token quant")
    if shuffle:
        scale = torch.empty(((m + 255) // 256 * 256, ((n + 31) // 32 + 7) // 8 * 8), dtype=torch.uint8,
                            device=x.device).view(dtypes.fp8_e8m0)
    else:
        scale = torch.empty((m, (n + 31) // 32), dtype=torch.uint8, device=x.device).view(dtypes.fp8_e8m0)
    y = torch.empty(m, n // 2, dtype=quant_dtype, device=x.device)
    dynamic_per_group_scaled_quant_fp4(y, x, scale, 32, shuffle_scale=shuffle, num_rows=num_rows,
                                       num_rows_factor=num_rows_factor)
    return y, scale


def mxfp4_moe_sort_hip(out_scale: Tensor, scale: Tensor, sorted_ids: Tensor, num_valid_ids: Tensor, token_num: int,
                       cols: int) -> None:
    """e8m0 scales gathered into moe_sorting order and shuffled (aiter/ops/quant.py:552-563)."""
    _lib.call("mxfp4_moe_sort_hip", out_scale, scale, sorted_ids, num_valid_ids, token_num, cols)


def mxfp4_moe_sort_fwd(scale: Tensor, sorted_ids: Tensor, num_valid_ids: Tensor, token_num: int,
                       cols: int) -> Tensor:
    """aiter/ops/quant.py:566-580."""
    out_scale = torch.empty(((sorted_ids.shape[0] + 31) // 32 * 32, (cols + 31) // 32), dtype=dtypes.fp8_e8m0,
                            device=scale.device)
    mxfp4_moe_sort_hip(out_scale, scale, sorted_ids, num_valid_ids, token_num, cols)
    return out_scale


def fused_dynamic_mxfp4_quant_moe_sort_hip(out: Tensor, scales: Tensor, input: Tensor, sorted_ids: Tensor,
                                           num_valid_ids: Tensor, token_num: int, block_m: int,
                                           group_size: int = 32) -> None:
    """MXFP4 quant of every input row and its scales in sorted, shuffled order, one
    launch (aiter/ops/quant.py:584-597)."""
    _lib.call("fused_dynamic_mxfp4_quant_moe_sort_hip", out, scales, input, sorted_ids, num_valid_ids, token_num,
              block_m, group_size)


def fused_dynamic_mxfp4_quant_moe_sort(input: Tensor, sorted_ids: Tensor, num_valid_ids: Tensor, token_num: int,
                                       topk: int, block_size: int, num_rows: Optional[Tensor] = None,
                                       group_size: int = 32) -> Tuple[Tensor, Tensor]:
    """(fp4x2 [M, N/2] in row order, sorted shuffled e8m0 scales), with the reference's
    choice between the one-launch kernel (few tokens) and quant then sort
    (aiter/ops/quant.py:600-652); both give the same bytes."""
    switch = [8 * 384 / topk, 8 * 1024 / topk]
    M, N = input.view(-1, input.shape[-1]).shape
    is_stage1 = M == token_num
    topk = 1 if is_stage1 else topk
    scale = torch.empty(((sorted_ids.shape[0] + 31) // 32 * 32, (N + 31) // 32), dtype=dtypes.fp8_e8m0,
                        device=input.device)
    if (is_stage1 and M <= switch[0]) or (not is_stage1 and M <= switch[1] * topk) or group_size != 32:
        out = torch.empty(M, N // 2, dtype=dtypes.fp4x2, device=input.device)
        fused_dynamic_mxfp4_quant_moe_sort_hip(out, scale, input, sorted_ids, num_valid_ids, token_num, block_size,
                                               group_size)
    else:
        out, scale_ = per_1x32_f4_quant_hip(input, None, dtypes.fp4x2, num_rows=num_rows, num_rows_factor=topk)
        mxfp4_moe_sort_hip(scale, scale_, sorted_ids, num_valid_ids, token_num, N)
    return out, scale


def moe_gather_quant_1x128(hidden_states: Tensor, token_sorted_pos: Tensor, topk: int, rows: int,
                           hidden_scale: Optional[Tensor] = None, out: Optional[Tensor] = None,
                           out_scale: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """Sorted-row fp8 activations for stage 1: ([rows, D] fp8, [D/128, rows] f32)."""
    D = hidden_states.shape[-1]
    dev = hidden_states.device
    if out is None:
        out = torch.empty((rows, D), dtype=dtypes.fp8, device=dev)
    if out_scale is None:
        out_scale = torch.empty((D // 128, rows), dtype=dtypes.fp32, device=dev)
    _lib.call("moe_gather_quant_1x128", hidden_states, hidden_scale, token_sorted_pos, topk, out, out_scale)
    return out, out_scale


def topk_sigmoid(topk_weights: Tensor, topk_indices: Tensor, gating_output: Tensor) -> None:
    """aiter.topk_sigmoid (aiter/ops/moe_op.py:40-42): the topk largest logits per token
    (descending) into topk_indices, sigmoid of each (fp32 math) into topk_weights."""
    _lib.call("topk_sigmoid", topk_weights, topk_indices, gating_output)


def moe_sum(input: Tensor, output: Tensor) -> None:
    """aiter.moe_sum (aiter/ops/moe_op.py:45-46): output [M, D] = input [M, topk, D]
    summed over the slots."""
    _lib.call("moe_sum", input, output)


def moe_stage1_fp8_blockscale(a1: Tensor, a1_scale: Tensor, w1: Tensor, w1_scale: Tensor,
                              sorted_token_ids: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                              out: Tensor, out_scale: Tensor, num_tokens: int, block_m: int = 128,
                              activation=ActivationType.Silu, sorted_weights: Optional[Tensor] = None,
                              inter_dtype=dtypes.bf16, bias: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """Gate/up grouped GEMM with fused act and 1x128 fp8 requant; sorted-row in and out.
    `sorted_weights` given: doweight_stage1 (gate/up scaled by the top-k weight before
    the activation); `inter_dtype`: bf16 or fp16 rounding of the intermediate; `bias`:
    the experts' f32 [E, 2 * inter_dim] bias, added before the activation."""
    if bias is not None:
        _lib.call("moe_stage1_fp8_blockscale_bias", a1, a1_scale, w1, w1_scale, sorted_token_ids,
                  sorted_expert_ids, num_valid_ids, out, out_scale, num_tokens, block_m, int(activation),
                  sorted_weights, _lib.dtype_code(inter_dtype), bias)
    elif sorted_weights is None and inter_dtype == dtypes.bf16:
        _lib.call("moe_stage1_fp8_blockscale", a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids,
                  num_valid_ids, out, out_scale, num_tokens, block_m, int(activation))
    else:
        _lib.call("moe_stage1_fp8_blockscale_ex", a1, a1_scale, w1, w1_scale, sorted_token_ids,
                  sorted_expert_ids, num_valid_ids, out, out_scale, num_tokens, block_m, int(activation),
                  sorted_weights, _lib.dtype_code(inter_dtype))
    return out, out_scale


def moe_stage2_fp8_blockscale(a2: Tensor, a2_scale: Tensor, w2: Tensor, w2_scale: Tensor,
                              sorted_token_ids: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                              sorted_weights: Optional[Tensor], out: Tensor, block_m: int = 128,
                              bias: Optional[Tensor] = None) -> Tensor:
    """Down grouped GEMM; adds the top-k weighted rows into out [M, D] (bf16 or fp16);
    `sorted_weights` None: unweighted (the weights were applied in stage 1); `bias`: the
    experts' f32 [E, D] bias, added before the top-k weight."""
    if bias is not None:
        _lib.call("moe_stage2_fp8_blockscale_bias", a2, a2_scale, w2, w2_scale, sorted_token_ids,
                  sorted_expert_ids, num_valid_ids, sorted_weights, out, block_m, bias)
    else:
        _lib.call("moe_stage2_fp8_blockscale", a2, a2_scale, w2, w2_scale, sorted_token_ids, sorted_expert_ids,
                  num_valid_ids, sorted_weights, out, block_m)
    return out


def moe_stage1_a8w4(a1: Tensor, a1_scale: Tensor, w1: Tensor, w1_scale_chunks: Tensor,
                    sorted_token_ids: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                    out: Tensor, out_scale: Tensor, num_tokens: int, block_m: int = 128,
                    activation=ActivationType.Silu, sorted_weights: Optional[Tensor] = None,
                    inter_dtype=dtypes.bf16, bias: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """moe_stage1_fp8_blockscale with MXFP4 weights (the A8W4 path of
    moe_cktile2stages_gemm1, aiter/ops/moe_op.py:343-403): w1 [E, 2I, D/2] fp4x2 kept at
    4 bits, its e8m0 scales as chunks (weights.mxfp4_moe_weight_scale_chunks)."""
    _lib.call("moe_stage1_a8w4", a1, a1_scale, w1, w1_scale_chunks, sorted_token_ids, sorted_expert_ids,
              num_valid_ids, out, out_scale, num_tokens, block_m, int(activation), sorted_weights,
              _lib.dtype_code(inter_dtype), bias)
    return out, out_scale


def moe_stage2_a8w4(a2: Tensor, a2_scale: Tensor, w2: Tensor, w2_scale_chunks: Tensor,
                    sorted_token_ids: Tensor, sorted_expert_ids: Tensor, num_valid_ids: Tensor,
                    sorted_weights: Optional[Tensor], out: Tensor, block_m: int = 128,
                    bias: Optional[Tensor] = None) -> Tensor:
    """moe_stage2_fp8_blockscale with MXFP4 weights (the A8W4 path of
    moe_cktile2stages_gemm2, aiter/ops/moe_op.py:406-465): w2 [E, D, I/2] fp4x2."""
    _lib.call("moe_stage2_a8w4", a2, a2_scale, w2, w2_scale_chunks, sorted_token_ids, sorted_expert_ids,
              num_valid_ids, sorted_weights, out, block_m, bias)
    return out
