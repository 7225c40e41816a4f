"""Collective front-ends of the TP and EP groups (aiter/dist/communication_op.py:30-244)."""
import torch

from .parallel_state import get_ep_group, get_tp_group


def tensor_model_parallel_all_reduce(input_: torch.Tensor, use_new: bool = True, open_fp8_quant: bool = False,
                                     prefill_support: bool = False) -> torch.Tensor:
    """All-reduce the input tensor across the tensor-parallel group."""
    return get_tp_group().all_reduce(input_, use_new, open_fp8_quant, prefill_support)


def tensor_model_parallel_custom_all_gather(input_: torch.Tensor) -> torch.Tensor:
    """(communication_op.py:68-69 in the reference)"""
    return get_tp_group().custom_all_gather(input_)


def tensor_model_parallel_reduce_scatter(input_: torch.Tensor, use_custom: bool = True,
                                         dim: int = 0) -> torch.Tensor:
    """(communication_op.py:72-77)"""
    return get_tp_group().reduce_scatter_tensor(input_, use_custom, dim)


def tensor_model_parallel_all_gather(input_: torch.Tensor, use_custom: bool = False, dim: int = -1) -> torch.Tensor:
    """(communication_op.py:80-86)"""
    return get_tp_group().all_gather(input_, use_custom, dim)


def tensor_model_parallel_gather(input_: torch.Tensor, dst: int = 0, dim: int = -1):
    """(communication_op.py:89-93)"""
    return get_tp_group().gather(input_, dst, dim)


def tensor_model_parallel_gemm_all_reduce(a: torch.Tensor, w: torch.Tensor, fused: bool = None) -> torch.Tensor:
    """allreduce(a @ w^T) over the TP group, GEMM and allreduce sharing the IPC
    staging buffer (`fused=True`: one kernel, the GEMM pushing its tiles to the
    peers; None: the one-kernel form for small M, the two-kernel form above).  Equals tensor_model_parallel_all_reduce(tgemm.mm(a, w)); the reference
    has no fused entry, this one is new."""
    return get_tp_group().gemm_all_reduce(a, w, fused=fused)


def shard_moe_weights_for_tp(w1, w1_scale, w2, w2_scale, rank, tp, chunk=8):
    """Rank `rank`'s share of FP8 block-scale MoE weights under tensor parallelism:
    inter_dim/tp columns of the gate and of the up half of w1 and the matching rows of
    w2's K, for every expert (the MoE TP layout of the reference's callers).

    When inter_dim/tp is a multiple of the 128-wide scale blocks the shard is a plain
    slice (bit-exact).  Otherwise (e.g. 1536/8 = 192) the shard cuts through scale
    blocks, so it is dequantised, zero-padded to the next multiple of 128 and
    re-quantised into shard-local 128x128 blocks.  The padded gate/up rows give
    act(0) * 0 = 0 in the intermediate and meet zero columns of w2, so they add
    nothing; the re-quantisation rounds the shard's weights once more to fp8."""
    E, two_i, D = w1.shape
    I = two_i // 2
    assert I % tp == 0, "inter_dim must divide by tp"
    il = I // tp
    if il % 128 == 0:
        b0, b1 = rank * il // 128, (rank + 1) * il // 128
        w1l = torch.cat([w1[:, rank * il:(rank + 1) * il], w1[:, I + rank * il:I + (rank + 1) * il]], dim=1)
        s1l = torch.cat([w1_scale[:, b0:b1], w1_scale[:, I // 128 + b0:I // 128 + b1]], dim=1)
        w2l = w2[:, :, rank * il:(rank + 1) * il]
        s2l = w2_scale[:, :, b0:b1]
        return w1l.contiguous(), s1l.contiguous(), w2l.contiguous(), s2l.contiguous()
    from ..weights import dequant_128x128, quant_weight_128x128
    ilp = (il + 127) // 128 * 128
    lo, hi = rank * il, (rank + 1) * il
    q1, q1s, q2, q2s = [], [], [], []
    for e0 in range(0, E, chunk):
        e1 = min(E, e0 + chunk)
        f1 = dequant_128x128(w1[e0:e1], w1_scale[e0:e1])
        pad1 = torch.zeros((e1 - e0, ilp - il, D), dtype=f1.dtype, device=f1.device)
        q, sc = quant_weight_128x128(torch.cat([f1[:, lo:hi], pad1, f1[:, I + lo:I + hi], pad1], dim=1))
        q1.append(q)
        q1s.append(sc)
        del f1
        f2 = dequant_128x128(w2[e0:e1], w2_scale[e0:e1])
        pad2 = torch.zeros((e1 - e0, D, ilp - il), dtype=f2.dtype, device=f2.device)
        q, sc = quant_weight_128x128(torch.cat([f2[:, :, lo:hi], pad2], dim=2))
        q2.append(q)
        q2s.append(sc)
        del f2
    return torch.cat(q1), torch.cat(q1s), torch.cat(q2), torch.cat(q2s)


def tensor_model_parallel_fused_allreduce_rmsnorm(input_, residual_inp_, weight_, eps, prefill_support=False):
    """(RMSNorm(allreduce(x) + residual) * w, allreduce(x) + residual)
    (aiter/dist/communication_op.py:40-49)."""
    return get_tp_group().fused_allreduce_rmsnorm(input_, residual_inp_, weight_, eps, prefill_support)


def tensor_model_parallel_fused_allreduce_rmsnorm_quant(input_, residual_inp_, weight_, eps,
                                                        prefill_support=False):
    """fp8 per-row-quantised variant: (out_fp8, residual_out, scale)
    (aiter/dist/communication_op.py:52-65)."""
    return get_tp_group().fused_allreduce_rmsnorm_quant(input_, residual_inp_, weight_, eps, prefill_support)


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


# ---------------------------------------------------------------- EP group
# (communication_op.py:105-136 in the reference)

def expert_parallel_all_reduce(input_, use_new=True, open_fp8_quant=False):
    return get_ep_group().all_reduce(input_, use_new, open_fp8_quant)


def expert_parallel_all_gather(input_, use_custom=False, dim=-1):
    return get_ep_group().all_gather(input_, use_custom, dim)


def expert_parallel_reduce_scatter(input_, use_custom=True, dim=0):
    return get_ep_group().reduce_scatter_tensor(input_, use_custom, dim)


def expert_parallel_gather(input_, dst=0, dim=-1):
    return get_ep_group().gather(input_, dst, dim)


def expert_parallel_broadcast(input_, src=0):
    return get_ep_group().broadcast(input_, src)
