"""Collective front-ends (aiter/dist/communication_op.py:30-37)."""
import torch

from .parallel_state import get_tp_group


def tensor_model_parallel_all_reduce(input_: torch.Tensor, use_new: bool = True, open_fp8_quant: bool = False,
                                     prefill_support: bool = False) -> torch.Tensor:
    """All-reduce the input tensor across the tensor-parallel group."""
    return get_tp_group().all_reduce(input_, use_new, open_fp8_quant, prefill_support)


def tensor_model_parallel_gemm_all_reduce(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """allreduce(a @ w^T) over the TP group, GEMM and allreduce sharing the IPC
    staging buffer.  Equals tensor_model_parallel_all_reduce(tgemm.mm(a, w)); the
    reference has no fused entry, this one is new."""
    return get_tp_group().gemm_all_reduce(a, w)


def shard_moe_weights_for_tp(w1, w1_scale, w2, w2_scale, rank, tp):
    """Rank `rank`'s share of FP8 block-scale MoE weights under tensor parallelism:
    inter_dim/tp columns of the gate and of the up half of w1 and the matching rows of
    w2's K, for every expert (the MoE TP layout of the reference's callers).  Needs
    inter_dim/tp to be a multiple of the 128-wide scale blocks."""
    E, two_i, D = w1.shape
    I = two_i // 2
    assert I % tp == 0 and (I // tp) % 128 == 0, "inter_dim / tp must be a multiple of 128"
    il = I // tp
    b0, b1 = rank * il // 128, (rank + 1) * il // 128
    w1l = torch.cat([w1[:, rank * il:(rank + 1) * il], w1[:, I + rank * il:I + (rank + 1) * il]], dim=1)
    s1l = torch.cat([w1_scale[:, b0:b1], w1_scale[:, I // 128 + b0:I // 128 + b1]], dim=1)
    w2l = w2[:, :, rank * il:(rank + 1) * il]
    s2l = w2_scale[:, :, b0:b1]
    return w1l.contiguous(), s1l.contiguous(), w2l.contiguous(), s2l.contiguous()


def tensor_model_parallel_fused_moe(hidden_states, w1, w2, topk_weight, topk_ids, **kwargs):
    """Tensor-parallel fused MoE: each rank holds inter_dim/tp of every expert
    (`shard_moe_weights_for_tp`), runs the fused MoE on its shard with the stage-2
    scatter-add landing in the allreduce's staging buffer, and the IPC allreduce sums
    the partial outputs in place.  Equals
    tensor_model_parallel_all_reduce(fused_moe(...)) on the shards."""
    from ..fused_moe import fused_moe
    tp = get_tp_group()
    if tp.world_size == 1:
        return fused_moe(hidden_states, w1, w2, topk_weight, topk_ids, **kwargs)
    ca = tp.ca_comm
    M, D = hidden_states.shape[0], w2.shape[1]
    if ca is None or ca.disabled or M * D * 2 > ca.max_size:
        return tp.all_reduce(fused_moe(hidden_states, w1, w2, topk_weight, topk_ids, **kwargs))
    stage = ca.next_buffer_tensor((M, D), torch.bfloat16)
    fused_moe(hidden_states, w1, w2, topk_weight, topk_ids, moe_buf=stage, **kwargs)
    return ca.all_reduce(stage)
