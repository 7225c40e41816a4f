"""Process groups of the tensor- and expert-parallel MoE path (the role of
aiter/dist/parallel_state.py for this path).

One process per GPU.  `init_distributed_environment` starts torch.distributed
(nccl) and the world group (parallel_state.py:1087-1145); `initialize_model_parallel`
builds the TP group, which carries the IPC allreduces, and the EP group of the
expert-parallel dispatch / combine (parallel_state.py:1147-1275, get_tp_group :1022).
A GroupCoordinator holds an NCCL device group and a gloo CPU group for the IPC
handle exchange (parallel_state.py:262-270).

Pipeline and data parallelism are not part of this library's path: the MoE layer
and its TP / EP collectives.  `initialize_model_parallel` keeps the reference's
pipeline / data-parallel size arguments so that callers bind unchanged, and rejects
sizes above 1.
"""
import contextlib
import dataclasses
import datetime
import os
from typing import Any, List, Optional

import torch
import torch.distributed as dist

from .custom_all_reduce import CustomAllreduce
from .quick_all_reduce import QuickAllReduce

_TP: Optional["GroupCoordinator"] = None
_EP: Optional["GroupCoordinator"] = None
_WORLD: Optional["GroupCoordinator"] = None
_ENABLE_CUSTOM_ALL_REDUCE = True
_TP_STATE_PATCHED = False


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
                 ca_max_size=128 * 1024 * 1024, timeout_s=120, use_quick_allreduce=True, group_name=""):
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
        if use_quick_allreduce and self.world_size > 1 and self.device.type == "cuda":
            # disabled unless AITER_QUICK_REDUCE_QUANTIZATION names a regime
            # (communicator_cuda.py:92-102 in the reference)
            self.qr_comm = QuickAllReduce(self.cpu_group, self.device)
        self.unique_name = group_name
        self._all2all_manager = None

    @property
    def all2all_manager(self):
        """The EP group's dispatch / combine manager, created on first use
        (communicator_cuda.py:104-146 in the reference, whose EP groups build MoRI's)."""
        if self._all2all_manager is None and self.world_size > 1:
            from .ep import EpAll2AllManager
            self._all2all_manager = EpAll2AllManager(self.cpu_group)
        return self._all2all_manager

    # ---- the group's end ranks (parallel_state.py:310-327), global rank numbers
    @property
    def first_rank(self):
        return self.ranks[0]

    @property
    def last_rank(self):
        return self.ranks[-1]

    @property
    def is_first_rank(self):
        return self.rank == self.ranks[0]

    @property
    def is_last_rank(self):
        return self.rank == self.ranks[-1]

    def all_reduce(self, input_: torch.Tensor, ca_use_new: bool = True, ca_fp8_quant: bool = False,
                   prefill_support: bool = False) -> torch.Tensor:
        """Out-of-place allreduce (parallel_state.py:376-407, communicator_cuda.py:
        157-204): the quick allreduce when enabled and the tensor is eligible, else
        the IPC allreduce for eligible tensors (ca_fp8_quant: its fp8-quantised form),
        the NCCL group otherwise."""
        if self.world_size == 1:
            return input_
        qr = self.qr_comm
        if qr is not None and not qr.disabled and qr.should_quick_allreduce(input_):
            return qr.quick_all_reduce(input_)
        if self.ca_comm is not None and not self.ca_comm.disabled:
            out = self.ca_comm.custom_all_reduce(input_, ca_use_new, ca_fp8_quant)
            if out is not None:
                return out
        out = input_.clone()
        dist.all_reduce(out, group=self.device_group)
        return out

    def custom_all_gather(self, input_: torch.Tensor) -> torch.Tensor:
        """All-gather along dim 0 over peer memory (parallel_state.py:500-501 in the
        reference), NCCL when the IPC path does not take the tensor."""
        return self.all_gather(input_, use_custom=True, dim=0)

    def all_gather(self, input_: torch.Tensor, use_custom: bool = False, dim: int = -1) -> torch.Tensor:
        """Concatenate every rank's tensor along `dim` (parallel_state.py:540-577).
        use_custom: the IPC all-gather for dim 0 or the last dim when eligible."""
        world = self.world_size
        if world == 1:
            return input_
        assert -input_.dim() <= dim < input_.dim(), f"Invalid dim ({dim}) for input tensor with shape {input_.size()}"
        if dim < 0:
            dim += input_.dim()
        if use_custom and self.ca_comm is not None and not self.ca_comm.disabled:
            out = self.ca_comm.custom_all_gather(input_, dim)
            if out is not None:
                return out
        size = input_.size()
        # [world * n0, ...] is the output layout every backend accepts; viewed as [world, ...]
        flat = torch.empty((world * size[0],) + tuple(size[1:]), dtype=input_.dtype, device=input_.device)
        dist.all_gather_into_tensor(flat, input_.contiguous(), group=self.device_group)
        out = flat.view((world,) + tuple(size)).movedim(0, dim)
        return out.reshape(size[:dim] + (world * size[dim],) + size[dim + 1:])

    def reduce_scatter_tensor(self, input_: torch.Tensor, use_custom: bool = True, dim: int = 0) -> torch.Tensor:
        """This rank's 1/world share of the sum along dim 0 (parallel_state.py:511-538):
        [n0 / world, ...] when dim 0 divides, else the flat share.  use_custom: the IPC
        reduce-scatter (rank-ordered fp32 sums, the allreduce's bits) when eligible."""
        world = self.world_size
        assert world > 1, "error! world_size = 1"
        assert input_.numel() % world == 0, "input shape error, input.numel() % world_size should equals to 0"
        if input_.shape[0] % world == 0:
            out_shape = (input_.shape[0] // world,) + tuple(input_.shape[1:])
        else:
            out_shape = (input_.numel() // world,)
        out = torch.empty(out_shape, dtype=input_.dtype, device=input_.device)
        if use_custom and self.ca_comm is not None and not self.ca_comm.disabled:
            if self.ca_comm.custom_reduce_scatter(input_, out):
                return out
        src = input_.contiguous()
        if out.dim() == 1 and input_.dim() != 1:
            src = src.reshape(-1)  # flat shares: [n] in, [n / world] out
        dist.reduce_scatter_tensor(out, src, group=self.device_group)
        return out

    def gather(self, input_: torch.Tensor, dst: int = 0, dim: int = -1) -> Optional[torch.Tensor]:
        """Concatenation along `dim` on rank `dst` of the group, None elsewhere
        (parallel_state.py:579-610)."""
        world = self.world_size
        if world == 1:
            return input_
        assert -input_.dim() <= dim < input_.dim(), f"Invalid dim ({dim}) for input tensor with shape {input_.size()}"
        if dim < 0:
            dim += input_.dim()
        gather_list = [torch.empty_like(input_) for _ in range(world)] if self.rank_in_group == dst else None
        dist.gather(input_, gather_list, dst=self.ranks[dst], group=self.device_group)
        return torch.cat(gather_list, dim=dim) if self.rank_in_group == dst else None

    def broadcast(self, input_: torch.Tensor, src: int = 0) -> torch.Tensor:
        assert src < self.world_size, f"Invalid src rank ({src})"
        if self.world_size == 1:
            return input_
        dist.broadcast(input_, src=self.ranks[src], group=self.device_group)
        return input_

    def broadcast_object(self, obj: Optional[Any] = None, src: int = 0):
        assert src < self.world_size, f"Invalid src rank ({src})"
        if self.world_size == 1:
            return obj
        holder = [obj if self.rank_in_group == src else None]
        dist.broadcast_object_list(holder, src=self.ranks[src], group=self.cpu_group)
        return holder[0]

    def barrier(self):
        """Barrier over the CPU group (parallel_state.py:928-935: an NCCL barrier would
        allocate device tensors behind the caller's back)."""
        dist.barrier(group=self.cpu_group)

    def prepare_communication_buffer_for_model(self, model: torch.nn.Module):
        """Hook for communicators that register model buffers (parallel_state.py:965-967).
        The IPC allreduce stages through its own buffers, so there is nothing to do."""
        return None

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

    def gemm_all_reduce(self, a: torch.Tensor, w: torch.Tensor, fused: bool = None) -> torch.Tensor:
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
        if self._all2all_manager is not None:
            self._all2all_manager.destroy()
            self._all2all_manager = None


def set_custom_all_reduce(enable: bool):
    """Whether groups built afterwards attach the IPC allreduce (parallel_state.py:1082-1084)."""
    global _ENABLE_CUSTOM_ALL_REDUCE
    _ENABLE_CUSTOM_ALL_REDUCE = enable


def init_world_group(ranks: List[int], local_rank: int, backend: str) -> GroupCoordinator:
    """The group of every rank, without device communicators (parallel_state.py:990-999)."""
    return GroupCoordinator(ranks, local_rank, backend, use_custom_allreduce=False, use_quick_allreduce=False,
                            group_name="world")


def get_world_group() -> GroupCoordinator:
    assert _WORLD is not None, "world group is not initialized"
    return _WORLD


def init_model_parallel_group(group_ranks: List[List[int]], local_rank: int, backend: str,
                              use_message_queue_broadcaster: bool = False,
                              group_name: Optional[str] = None) -> GroupCoordinator:
    """A group per rank list of `group_ranks`; returns the one holding this rank
    (parallel_state.py:1002-1017).  The IPC allreduce is attached unless disabled by
    set_custom_all_reduce; no message-queue broadcaster exists here (objects go over
    the group's CPU group)."""
    return _init_groups(group_ranks, local_rank, backend, group_name or "", _ENABLE_CUSTOM_ALL_REDUCE,
                        128 * 1024 * 1024)


def init_distributed_environment(world_size=-1, rank=-1, distributed_init_method="env://", local_rank=-1,
                                 backend="nccl", data_parallel_size=1, data_parallel_rank=0, timeout_s=120):
    """Start torch.distributed and the world group (parallel_state.py:1087-1145).
    `data_parallel_size` / `data_parallel_rank` keep the reference's signature; sizes
    above 1 are rejected (data parallelism is outside this library's path)."""
    global _WORLD
    _check_single("data_parallel", data_parallel_size)
    if world_size == -1:
        world_size = int(os.environ.get("WORLD_SIZE", "1"))
    if rank == -1:
        rank = int(os.environ.get("RANK", "0"))
    if not dist.is_initialized():
        dist.init_process_group(backend=backend, init_method=distributed_init_method, world_size=world_size,
                                rank=rank, timeout=datetime.timedelta(seconds=timeout_s))
    if local_rank == -1:
        local_rank = int(os.environ.get("LOCAL_RANK", str(dist.get_rank())))
    if backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    if _WORLD is None:
        _WORLD = init_world_group(list(range(dist.get_world_size())), local_rank, backend)
    else:
        assert _WORLD.world_size == dist.get_world_size(), "world group already initialized with a different world size"
    return local_rank


def _init_groups(group_ranks, local_rank, backend, name, use_custom_allreduce=False, ca_max_size=0,
                 use_quick_allreduce=False):
    """Every rank creates every group (a torch.distributed requirement); the rank keeps
    a GroupCoordinator for the group that contains it."""
    me = dist.get_rank()
    mine = None
    for ranks in group_ranks:
        if me in ranks:
            mine = GroupCoordinator(ranks, local_rank, backend, use_custom_allreduce, ca_max_size,
                                    use_quick_allreduce=use_quick_allreduce, group_name=name)
        else:
            dist.new_group(ranks, backend=backend)
            dist.new_group(ranks, backend="gloo")
    return mine


def _check_single(what: str, size: int):
    if size != 1:
        raise NotImplementedError(f"{what} size {size}: pipeline and data parallelism are outside this library's "
                                  f"path (the MoE layer and its tensor- / expert-parallel collectives)")


def initialize_model_parallel(tensor_model_parallel_size=1, pipeline_model_parallel_size=1, backend=None,
                              data_parallel_size=1, local_rank=None, use_custom_allreduce=True,
                              ca_max_size=128 * 1024 * 1024):
    """TP and EP groups (parallel_state.py:1147-1275).  Consecutive ranks form a TP group
    (TP is the fastest-varying dimension of the reference's layout); with no data
    parallelism the EP group of a rank is its TP group.  The TP group carries the IPC
    allreduce and, when AITER_QUICK_REDUCE_QUANTIZATION names a regime, the quick
    allreduce.  Returns the TP group."""
    global _TP, _EP
    assert _TP is None, "tensor model parallel group is already initialized"
    _check_single("pipeline_model_parallel", pipeline_model_parallel_size)
    _check_single("data_parallel", data_parallel_size)
    world = dist.get_world_size()
    tp = tensor_model_parallel_size
    assert world % tp == 0, f"world size {world} is not a multiple of tensor_model_parallel_size {tp}"
    backend = backend or dist.get_backend()
    if local_rank is None:
        local_rank = int(os.environ.get("LOCAL_RANK", str(dist.get_rank())))
    groups = [list(range(g * tp, (g + 1) * tp)) for g in range(world // tp)]
    _TP = _init_groups(groups, local_rank, backend, "tp", use_custom_allreduce and _ENABLE_CUSTOM_ALL_REDUCE,
                       ca_max_size, use_quick_allreduce=True)
    _EP = _init_groups(groups, local_rank, backend, "ep")
    return _TP


def ensure_model_parallel_initialized(tensor_model_parallel_size, pipeline_model_parallel_size=1, backend=None,
                                      data_parallel_size=1):
    """(parallel_state.py:1278-1308)"""
    if not model_parallel_is_initialized():
        initialize_model_parallel(tensor_model_parallel_size, pipeline_model_parallel_size, backend,
                                  data_parallel_size)
        return
    assert get_tp_group().world_size == tensor_model_parallel_size, "tensor parallel group already initialized"


def model_parallel_is_initialized() -> bool:
    return _TP is not None and _EP is not None


def get_tp_group() -> GroupCoordinator:
    assert _TP is not None, "tensor model parallel group is not initialized"
    return _TP


def get_ep_group() -> GroupCoordinator:
    assert _EP is not None, "expert parallel group is not initialized"
    return _EP


def get_tensor_model_parallel_world_size() -> int:
    return get_tp_group().world_size


def get_tensor_model_parallel_rank() -> int:
    return get_tp_group().rank_in_group


@contextlib.contextmanager
def graph_capture():
    """Context around CUDA-graph capture of tensor-parallel code
    (parallel_state.py:1058-1074 in the reference): yields a GraphCaptureContext
    whose stream the graph should be captured on."""
    with get_tp_group().graph_capture() as ctx:
        yield ctx


def destroy_model_parallel():
    global _TP, _EP
    for g in (_TP, _EP):
        if g is not None:
            g.destroy()
    _TP = _EP = None


@contextlib.contextmanager
def patch_tensor_parallel_group(tp_group: GroupCoordinator):
    """Use `tp_group` as the TP group inside the context (a draft model with another TP
    degree; parallel_state.py:1320-1341)."""
    global _TP, _TP_STATE_PATCHED
    assert not _TP_STATE_PATCHED, "Should not call when it's already patched"
    _TP_STATE_PATCHED = True
    old = get_tp_group()
    _TP = tp_group
    try:
        yield
    finally:
        _TP_STATE_PATCHED = False
        _TP = old


def in_the_same_node_as(pg, source_rank: int = 0) -> List[bool]:
    """For each rank of `pg` (a CPU / gloo group), whether it runs on the same host as
    group rank `source_rank` (parallel_state.py:1386-1452); compared by host name."""
    import socket
    names = [None] * dist.get_world_size(group=pg)
    dist.all_gather_object(names, socket.gethostname(), group=pg)
    return [n == names[source_rank] for n in names]


def is_global_first_rank() -> bool:
    """Global rank 0 across every parallel dimension, True without torch.distributed
    (parallel_state.py:1455-1483)."""
    if _WORLD is not None:
        return _WORLD.is_first_rank
    return not dist.is_initialized() or dist.get_rank() == 0


def prepare_communication_buffer_for_model(model: torch.nn.Module):
    """Let every group's communicators size buffers for `model` (parallel_state.py:1526-1544)."""
    for g in (_TP, _EP):
        if g is not None:
            g.prepare_communication_buffer_for_model(model)


def destroy_distributed_environment():
    global _WORLD
    destroy_model_parallel()
    if _WORLD is not None:
        _WORLD.destroy()
    _WORLD = None
    if dist.is_initialized():
        dist.destroy_process_group()
