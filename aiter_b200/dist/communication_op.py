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
