"""torch.library registration of the path's operators, the role of the reference's
`torch_compile_guard` (aiter/jit/utils/torch_guard.py:192) and `fused_moe_fake`
(aiter/fused_moe.py:172-202): every operator is a torch custom op with a fake
(shape-only) implementation, so torch.compile / dynamo trace through it without
running a kernel.  The in-place operators declare what they mutate.

Eager calls of the public functions do not go through the dispatcher;
`aiter_b200.fused_moe` routes to `torch.ops.aiter_b200.fused_moe_` only while
torch is compiling.
"""
from typing import Optional

import torch
from torch import Tensor

from . import moe_op

NS = "aiter_b200"


@torch.library.custom_op(f"{NS}::fused_moe_", mutates_args=())
def fused_moe_(hidden_states: Tensor, w1: Tensor, w2: Tensor, topk_weight: Tensor, topk_ids: Tensor,
               expert_mask: Optional[Tensor] = None, activation: int = 0, quant_type: int = 0,
               doweight_stage1: bool = False, w1_scale: Optional[Tensor] = None,
               w2_scale: Optional[Tensor] = None, a1_scale: Optional[Tensor] = None,
               a2_scale: Optional[Tensor] = None, num_local_tokens: Optional[Tensor] = None,
               moe_sorting_dispatch_policy: int = 0) -> Tensor:
    from .fused_moe import _fused_moe_impl
    return _fused_moe_impl(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask, activation, quant_type,
                           doweight_stage1, w1_scale, w2_scale, a1_scale, a2_scale, None, num_local_tokens,
                           moe_sorting_dispatch_policy)


@fused_moe_.register_fake
def _fused_moe_fake(hidden_states, w1, w2, topk_weight, topk_ids, expert_mask=None, activation=0, quant_type=0,
                    doweight_stage1=False, w1_scale=None, w2_scale=None, a1_scale=None, a2_scale=None,
                    num_local_tokens=None, moe_sorting_dispatch_policy=0):
    # output [M, model_dim] in the activation dtype: fp16 for fp16 inputs, else bf16
    # (w2 is [E, model_dim, inter_dim] or its fp4x2 packing)
    out_dtype = torch.float16 if hidden_states.dtype == torch.float16 else torch.bfloat16
    return hidden_states.new_empty((topk_ids.shape[0], w2.shape[1]), dtype=out_dtype)


@torch.library.custom_op(f"{NS}::topk_softmax",
                         mutates_args=("topk_weights", "topk_indices", "token_expert_indices"))
def topk_softmax(topk_weights: Tensor, topk_indices: Tensor, token_expert_indices: Tensor,
                 gating_output: Tensor, need_renorm: bool, num_shared_experts: int = 0,
                 shared_expert_scoring_func: str = "") -> None:
    moe_op.topk_softmax(topk_weights, topk_indices, token_expert_indices, gating_output, need_renorm,
                        num_shared_experts, shared_expert_scoring_func)


@topk_softmax.register_fake
def _topk_softmax_fake(topk_weights, topk_indices, token_expert_indices, gating_output, need_renorm,
                       num_shared_experts=0, shared_expert_scoring_func=""):
    return None


@torch.library.custom_op(f"{NS}::grouped_topk", mutates_args=("topk_weights", "topk_ids"))
def grouped_topk(gating_output: Tensor, topk_weights: Tensor, topk_ids: Tensor, num_expert_group: int,
                 topk_group: int, need_renorm: bool, is_softmax: bool = True,
                 routed_scaling_factor: float = 1.0) -> None:
    moe_op.grouped_topk(gating_output, topk_weights, topk_ids, num_expert_group, topk_group, need_renorm,
                        is_softmax, routed_scaling_factor)


@grouped_topk.register_fake
def _grouped_topk_fake(gating_output, topk_weights, topk_ids, num_expert_group, topk_group, need_renorm,
                       is_softmax=True, routed_scaling_factor=1.0):
    return None


@torch.library.custom_op(f"{NS}::biased_grouped_topk", mutates_args=("topk_weights", "topk_ids"))
def biased_grouped_topk(gating_output: Tensor, correction_bias: Tensor, topk_weights: Tensor, topk_ids: Tensor,
                        num_expert_group: int, topk_group: int, need_renorm: bool,
                        routed_scaling_factor: float = 1.0) -> None:
    moe_op.biased_grouped_topk(gating_output, correction_bias, topk_weights, topk_ids, num_expert_group,
                               topk_group, need_renorm, routed_scaling_factor)


@biased_grouped_topk.register_fake
def _biased_grouped_topk_fake(gating_output, correction_bias, topk_weights, topk_ids, num_expert_group,
                              topk_group, need_renorm, routed_scaling_factor=1.0):
    return None


@torch.library.custom_op(f"{NS}::moe_sorting_fwd",
                         mutates_args=("sorted_token_ids", "sorted_weights", "sorted_expert_ids", "num_valid_ids",
                                       "moe_buf"))
def moe_sorting_fwd(topk_ids: Tensor, topk_weights: Tensor, sorted_token_ids: Tensor, sorted_weights: Tensor,
                    sorted_expert_ids: Tensor, num_valid_ids: Tensor, moe_buf: Tensor, num_experts: int,
                    unit_size: int, local_expert_mask: Optional[Tensor] = None,
                    num_local_tokens: Optional[Tensor] = None, dispatch_policy: int = 0) -> None:
    moe_op.moe_sorting_fwd(topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids,
                           num_valid_ids, moe_buf, num_experts, unit_size, local_expert_mask, num_local_tokens,
                           dispatch_policy)


@moe_sorting_fwd.register_fake
def _moe_sorting_fwd_fake(topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids,
                          num_valid_ids, moe_buf, num_experts, unit_size, local_expert_mask=None,
                          num_local_tokens=None, dispatch_policy=0):
    return None


@torch.library.custom_op(f"{NS}::gemm_a16w16", mutates_args=())
def gemm_a16w16(a: Tensor, w: Tensor) -> Tensor:
    from .gemm import gemm_a16w16 as _g
    return _g(a, w)


@gemm_a16w16.register_fake
def _gemm_a16w16_fake(a, w):
    return a.new_empty((a.shape[0], w.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{NS}::topk_sigmoid", mutates_args=("topk_weights", "topk_indices"))
def topk_sigmoid(topk_weights: Tensor, topk_indices: Tensor, gating_output: Tensor) -> None:
    moe_op.topk_sigmoid(topk_weights, topk_indices, gating_output)


@topk_sigmoid.register_fake
def _topk_sigmoid_fake(topk_weights, topk_indices, gating_output):
    return None


@torch.library.custom_op(f"{NS}::moe_sum", mutates_args=("output",))
def moe_sum(input: Tensor, output: Tensor) -> None:
    moe_op.moe_sum(input, output)


@moe_sum.register_fake
def _moe_sum_fake(input, output):
    return None


def _register_act(name):
    from . import activation

    @torch.library.custom_op(f"{NS}::{name}", mutates_args=("out",))
    def op(out: Tensor, input: Tensor) -> None:
        getattr(activation, name)(out, input)

    @op.register_fake
    def _fake(out, input):
        return None

    return op


silu_and_mul = _register_act("silu_and_mul")
gelu_and_mul = _register_act("gelu_and_mul")
gelu_tanh_and_mul = _register_act("gelu_tanh_and_mul")


@torch.library.custom_op(f"{NS}::scaled_silu_and_mul", mutates_args=("out",))
def scaled_silu_and_mul(out: Tensor, input: Tensor, scale: Tensor) -> None:
    from . import activation
    activation.scaled_silu_and_mul(out, input, scale)


@scaled_silu_and_mul.register_fake
def _scaled_silu_and_mul_fake(out, input, scale):
    return None
