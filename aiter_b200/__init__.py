"""aiter_b200: the quantised fused-MoE hot path of AITER, written from scratch for
NVIDIA B200 (sm_100a), behind AITER's Python operator surface.

    import aiter_b200 as aiter
    w, ids = aiter.fused_topk(x, logits, topk=8, renormalize=True)
    y = aiter.fused_moe(x, w1, w2, w, ids, quant_type=aiter.QuantType.per_1x128,
                        w1_scale=s1, w2_scale=s2)

All compute runs in hand-written CUDA kernels of libaiter_b200.so (C ABI,
include/aiter_b200.h), called through ctypes; there is no CPU fallback.
"""
from . import dtypes
from .enums import ActivationType, QuantType
from .moe_op import (biased_grouped_topk, biased_grouped_topk_hip, dynamic_per_group_scaled_quant_fp4,
                     dynamic_per_token_scaled_quant, fused_dynamic_mxfp4_quant_moe_sort,
                     fused_dynamic_mxfp4_quant_moe_sort_hip, grouped_topk, moe_gather_quant_1x128,
                     moe_sorting_fwd, moe_sorting_get_workspace_size, moe_stage1_fp8_blockscale,
                     moe_stage2_fp8_blockscale, mxfp4_moe_sort_fwd, mxfp4_moe_sort_hip, per_1x32_f4_quant_hip,
                     per_group_quant_hip, topk_softmax, topk_sigmoid, moe_sum, moe_sorting_opus_fwd)
from .activation import gelu_and_mul, gelu_tanh_and_mul, scaled_silu_and_mul, silu_and_mul
from .fused_moe import fused_moe, fused_topk, moe_sorting, get_inter_dim
from ._lib import device_error
from .quick_all_reduce import (init_custom_qr, qr_all_reduce, qr_destroy, qr_device_error, qr_get_handle,
                               qr_max_size, qr_open_handles)
from . import torch_ops  # registers torch.ops.aiter_b200.* (fake impls for torch.compile)

__all__ = [
    "dtypes", "ActivationType", "QuantType", "topk_softmax", "grouped_topk", "biased_grouped_topk",
    "biased_grouped_topk_hip", "moe_gather_quant_1x128", "moe_sorting_fwd", "moe_sorting_get_workspace_size",
    "dynamic_per_token_scaled_quant", "per_group_quant_hip", "moe_stage1_fp8_blockscale",
    "moe_stage2_fp8_blockscale", "fused_moe", "fused_topk", "moe_sorting", "get_inter_dim",
    "device_error", "dynamic_per_group_scaled_quant_fp4", "per_1x32_f4_quant_hip", "mxfp4_moe_sort_hip",
    "mxfp4_moe_sort_fwd", "fused_dynamic_mxfp4_quant_moe_sort_hip", "fused_dynamic_mxfp4_quant_moe_sort",
    "init_custom_qr", "qr_get_handle", "qr_open_handles", "qr_all_reduce", "qr_destroy", "qr_max_size",
    "qr_device_error", "topk_sigmoid", "moe_sum", "silu_and_mul", "gelu_and_mul", "gelu_tanh_and_mul",
    "scaled_silu_and_mul", "moe_sorting_opus_fwd",
]
