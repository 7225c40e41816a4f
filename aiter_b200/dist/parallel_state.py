"""Process groups for tensor parallelism (the role of aiter/dist/parallel_state.py).

One process per GPU.  `init_distributed_environment` starts torch.distributed
(nccl) (parallel_state.py:1087-1145); `initialize_model_parallel` builds the TP
GroupCoordinator (parallel_state.py:1147, get_tp_group :1022).  Like the reference,
a GroupCoordinator holds an NCCL device group plus a gloo CPU group
(parallel_state.py:262-270), and attaches the custom allreduce to the CPU group.
"""
import contextlib
import dataclasses
import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist

from .custom_all_reduce import CustomAllreduce
from .quick_all_reduce import QuickAllReduce

_TP: Optional["GroupCoordinator"] = None


def _rmsnorm_after(ar: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float, quant: bool):
    """The math of the fused kernel on an already reduced tensor (used when the IPC
    allreduce does not take the tensor): x = ar + res in fp32, res_out = bf16(x),
    y = x * w * rsqrt(mean(x^2) + eps)."""
    x = ar.float() + res.float()
    res_out = x.to(ar.dtype)
    y = x * w.float() * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    if not quant:
        return y.to(ar.dtype), res_out
    amax = y.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax == 0, torch.ones_like(amax), amax / 448.0)
    return (y / scale).to(torch.float8_e4m3fn), res_out, scale


@dataclasses.dataclass
class GraphCaptureContext:
    stream: torch.cuda.Stream


class GroupCoordinator:
    def __init__(self, ranks, local_rank, backend="nccl", use_custom_allreduce=True,
                 ca_max_size=128 * 1024 * 1024, timeout_s=120):
        self.ranks = list(ranks)
        self.world_size = len(self.ranks)
        self.rank = dist.get_rank()
        self.rank_in_group = self.ranks.index(self.rank)
        self.local_rank = local_rank
        to = datetime.timedelta(seconds=timeout_s)
        self.device_group = dist.new_group(self.ranks, backend=backend, timeout=to)
        self.cpu_group = dist.new_group(self.ranks, backend="gloo", timeout=to)
        self.device = torch.device(f"cuda:{local_rank}") if torch.cuda.is_available() and backend == "nccl" \
            else torch.device("cpu")
        self.ca_comm = None
        self.qr_comm = None
        if use_custom_allreduce and self.world_size > 1 and self.device.type == "cuda":
            self.ca_comm = CustomAllreduce(self.cpu_group, self.device, ca_max_size)
        if self.world_size > 1 and self.device.type == "cuda":
            # disabled unless AITER_QUICK_REDUCE_QUANTIZATION names a regime
            # (communicator_cuda.py:92-102 in the reference)
            self.qr_comm = QuickAllReduce(self.cpu_group, self.device)

    def all_reduce(self, input_: torch.Tensor, use_new: bool = True, open_fp8_quant: bool = False,
                   prefill_support: bool = False) -> torch.Tensor:
        """Out-of-place allreduce (parallel_state.py:376-407, communicator_cuda.py:
        157-204): the quick allreduce when enabled and the tensor is eligible, else
        the IPC allreduce for eligible tensors, the NCCL group otherwise."""
        if self.world_size == 1:
            return input_
        qr = self.qr_comm
        if qr is not None and not qr.disabled and qr.should_quick_allreduce(input_):
            return qr.quick_all_reduce(input_)
        if self.ca_comm is not None and not self.ca_comm.disabled:
            out = self.ca_comm.custom_all_reduce(input_, use_new, open_fp8_quant)
            if out is not None:
                return out
        out = input_.clone()
        dist.all_reduce(out, group=self.device_group)
        return out

    def fused_allreduce_rmsnorm(self, input_: torch.Tensor, residual_inp_: torch.Tensor, weight_: torch.Tensor,
                                eps: float, prefill_support: bool = False):
        """(out, residual_out) = (RMSNorm(allreduce(input_) + residual_inp_) * weight_,
        allreduce(input_) + residual_inp_) -- the fused kernel when the IPC allreduce
        takes the tensor, else the allreduce followed by the same math in torch
        (communicator_cuda.py:207-255 in the reference)."""
        if self.world_size > 1 and self.ca_comm is not None:
            r = self.ca_comm.custom_fused_ar_rms(input_, residual_inp_, weight_, eps)
            if r is not None:
                return r
        return _rmsnorm_after(self.all_reduce(input_), residual_inp_, weight_, eps, quant=False)

    def fused_allreduce_rmsnorm_quant(self, input_: torch.Tensor, residual_inp_: torch.Tensor,
                                      weight_: torch.Tensor, eps: float, prefill_support: bool = False):
        """As fused_allreduce_rmsnorm with the normalised rows quantised to fp8 e4m3,
        one scale per row: (out_fp8, residual_out, scale [.., 1])."""
        if self.world_size > 1 and self.ca_comm is not None:
            r = self.ca_comm.custom_fused_ar_rms_quant(input_, residual_inp_, weight_, eps)
            if r is not None:
                return r
        return _rmsnorm_after(self.all_reduce(input_), residual_inp_, weight_, eps, quant=True)

    def gemm_all_reduce(self, a: torch.Tensor, w: torch.Tensor, fused: bool = False) -> torch.Tensor:
        if self.world_size == 1:
            from ..gemm import gemm_a16w16
            return gemm_a16w16(a, w)
        if self.ca_comm is None or self.ca_comm.disabled:
            raise RuntimeError("GEMM + allreduce needs the custom allreduce (world sizes 2, 4, 6, 8)")
        return self.ca_comm.gemm_all_reduce(a, w, fused=fused)

    @contextlib.contextmanager
    def graph_capture(self, graph_capture_context: Optional["GraphCaptureContext"] = None):
        """Run the body on a side stream inside the allreduce's capture context
        (parallel_state.py:345-374 in the reference)."""
        if graph_capture_context is None:
            graph_capture_context = GraphCaptureContext(torch.cuda.Stream(device=self.device))
        stream = graph_capture_context.stream
        curr = torch.cuda.current_stream(self.device)
        if curr != stream:
            stream.wait_stream(curr)
        ca = self.ca_comm.capture() if self.ca_comm is not None and not self.ca_comm.disabled \
            else contextlib.nullcontext()
        with torch.cuda.stream(stream), ca:
            yield graph_capture_context

    def destroy(self):
        if self.ca_comm is not None:
            self.ca_comm.close()
            self.ca_comm = None
        if self.qr_comm is not None:
            self.qr_comm.close()
            self.qr_comm = None


def init_distributed_environment(world_size=-1, rank=-1, distributed_init_method="env://", local_rank=-1,
                                 backend="nccl", timeout_s=120):
    if not dist.is_initialized():
        if world_size == -1:
            world_size = int(os.environ.get("WORLD_SIZE", "1"))
        if rank == -1:
            rank = int(os.environ.get("RANK", "0"))
        dist.init_process_group(backend=backend, init_method=distributed_init_method, world_size=world_size,
                                rank=rank, timeout=datetime.timedelta(seconds=timeout_s))
    if local_rank == -1:
        local_rank = int(os.environ.get("LOCAL_RANK", str(dist.get_rank())))
    if backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    return local_rank


def initialize_model_parallel(tensor_model_parallel_size=1, local_rank=None, backend="nccl",
                              use_custom_allreduce=True, ca_max_size=128 * 1024 * 1024):
    global _TP
    world = dist.get_world_size()
    assert world % tensor_model_parallel_size == 0
    if local_rank is None:
        local_rank = int(os.environ.get("LOCAL_RANK", str(dist.get_rank())))
    me = dist.get_rank()
    for g in range(world // tensor_model_parallel_size):
        ranks = list(range(g * tensor_model_parallel_size, (g + 1) * tensor_model_parallel_size))
        if me in ranks:
            # every rank creates every group (torch.distributed requirement): only ours is kept
            _TP = GroupCoordinator(ranks, local_rank, backend, use_custom_allreduce, ca_max_size)
        else:
            dist.new_group(ranks, backend=backend)
            dist.new_group(ranks, backend="gloo")
    return _TP


def get_tp_group() -> GroupCoordinator:
    assert _TP is not None, "tensor model parallel group is not initialized"
    return _TP


@contextlib.contextmanager
def graph_capture():
    """Context around CUDA-graph capture of tensor-parallel code
    (parallel_state.py:1058-1074 in the reference): yields a GraphCaptureContext
    whose stream the graph should be captured on."""
    with get_tp_group().graph_capture() as ctx:
        yield ctx


def destroy_model_parallel():
    global _TP
    if _TP is not None:
        _TP.destroy()
    _TP = None


def destroy_distributed_environment():
    destroy_model_parallel()
    if dist.is_initialized():
        dist.destroy_process_group()
