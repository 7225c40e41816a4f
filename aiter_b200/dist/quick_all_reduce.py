"""QuickAllReduce: the quantised two-shot allreduce of libaiter_b200.so behind the
reference's interface (aiter/dist/device_communicators/quick_all_reduce.py:20-268).

Enabled, as in the reference, only when AITER_QUICK_REDUCE_QUANTIZATION names a
regime (FP, FP8, INT6, INT4; NONE or unset disables it).  bf16 inputs run the fp16
kernels unless AITER_QUICK_REDUCE_CAST_BF16_TO_FP16=0, and
AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB sets the registered size (default
qr_max_size(), 2 GiB).  The communicator lives on sm_100 GPUs (the reference's
MI300 check, `qr_rocm_arch_available`, :37-46) in a single node; its IPC
handles travel over the CPU (gloo) group.

The minimum message sizes per (dtype, world size, regime) are the reference's
table (:62-69), measured on MI300; below them the caller falls through to the
custom allreduce.
"""
import logging
import os
from enum import Enum
from typing import Union

import torch
import torch.distributed as dist

from .. import quick_all_reduce as ops

logger = logging.getLogger("aiter_b200")

MB = 1024 * 1024


class QuickReduceRegime(Enum):
    FP = 0
    FP8 = 1
    INT6 = 2
    INT4 = 3
    NONE = 4


def qr_arch_available() -> bool:
    """sm_100 (B200) devices only."""
    try:
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception as e:  # noqa: BLE001 - mirrors the reference's broad check
        logger.warning("Failed to determine the GPU architecture for quick allreduce: %s", e)
        return False


def quick_ar_requested() -> bool:
    """The reference's module-level `quick_ar` (:29-37): a regime is named and the
    library answers qr_max_size()."""
    if os.environ.get("AITER_QUICK_REDUCE_QUANTIZATION") not in QuickReduceRegime.__members__:
        return False
    try:
        ops.qr_max_size()
        return True
    except Exception:  # noqa: BLE001 - library missing: quick allreduce stays off
        return False


def is_weak_contiguous(inp: torch.Tensor) -> bool:
    return inp.is_contiguous() or (inp.untyped_storage().nbytes() - inp.storage_offset() * inp.element_size()
                                   == inp.numel() * inp.element_size())


class QuickAllReduce:
    _SUPPORTED_WORLD_SIZES = [2, 4, 8]
    _SUPPORTED_DTYPES = [torch.float16, torch.bfloat16]
    # [FP, FP8, INT6, INT4] minimum sizes (the reference's MI300 table, :62-69)
    _QR_MIN_SIZE = {
        (torch.float16, 2): [1 * MB, 2 * MB, 2 * MB, 1 * MB],
        (torch.float16, 4): [1 * MB, 16 * MB, 4 * MB, 2 * MB],
        (torch.float16, 8): [16 * MB, 4 * MB, 4 * MB, 8 * MB],
        (torch.bfloat16, 2): [2 * MB, 8 * MB, 8 * MB, 8 * MB],
        (torch.bfloat16, 4): [8 * MB, 64 * MB, 64 * MB, 16 * MB],
        (torch.bfloat16, 8): [16 * MB, 2048 * MB, 2048 * MB, 2048 * MB],
    }

    def __init__(self, group, device: Union[int, str, torch.device]) -> None:
        self.disabled = True
        self._ptr = 0
        if not qr_arch_available():
            logger.debug("quick allreduce is only supported on sm_100 GPUs")
            return
        if not quick_ar_requested():
            return
        self.group = group
        assert dist.get_backend(group) != dist.Backend.NCCL, \
            "Custom quick allreduce should be attached to a non-NCCL group."
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        if self.world_size == 1:
            return
        if self.world_size not in QuickAllReduce._SUPPORTED_WORLD_SIZES:
            logger.warning("quick allreduce disabled: unsupported world size %d (supported: %s)",
                           self.world_size, QuickAllReduce._SUPPORTED_WORLD_SIZES)
            return
        if isinstance(device, int):
            device = torch.device(f"cuda:{device}")
        elif isinstance(device, str):
            device = torch.device(device)
        self.device = device
        self.init_quick_all_reduce()

    def init_quick_all_reduce(self):
        self.use_fp16_kernels = int(os.environ.get("AITER_QUICK_REDUCE_CAST_BF16_TO_FP16", 1))
        regime_str = os.environ.get("AITER_QUICK_REDUCE_QUANTIZATION", "NONE")
        if regime_str not in QuickReduceRegime.__members__:
            logger.warning("quick allreduce: invalid quantization level %s; supported: %s", regime_str,
                           list(QuickReduceRegime.__members__.keys()))
            return
        if regime_str == "NONE":
            return
        self.qr_quant_level = QuickReduceRegime[regime_str]
        qr_max_size = int(os.environ.get("AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB", 0))
        if qr_max_size > 0:
            qr_max_size = qr_max_size * MB
        with torch.cuda.device(self.device):
            self._ptr = ops.init_custom_qr(self.rank, self.world_size, qr_max_size if qr_max_size > 0 else None)
        self.qr_max_size = qr_max_size if qr_max_size > 0 else ops.qr_max_size()
        try:
            self.create_shared_buffer()
        except Exception:
            ops.qr_destroy(self._ptr)
            self._ptr = 0
            raise
        self.disabled = False

    def create_shared_buffer(self):
        """Exchange the IPC handles over the CPU group and open the peers' regions."""
        handle = ops.qr_get_handle(self._ptr)
        handles = [None] * self.world_size
        dist.all_gather_object(handles, handle, group=self.group)
        ops.qr_open_handles(self._ptr, handles)

    def should_quick_allreduce(self, inp: torch.Tensor) -> bool:
        if self.disabled:
            return False
        if inp.dtype not in self._SUPPORTED_DTYPES:
            return False
        inp_size = inp.numel() * inp.element_size()
        if inp_size % 16 != 0:
            return False
        if not is_weak_contiguous(inp):
            return False
        dtype = torch.float16 if self.use_fp16_kernels else inp.dtype
        return (inp_size <= self.qr_max_size
                and inp_size >= self._QR_MIN_SIZE[(dtype, self.world_size)][self.qr_quant_level.value])

    def quick_all_reduce(self, inp: torch.Tensor, *, out: torch.Tensor = None) -> torch.Tensor:
        """Out-of-place quick allreduce.  Graph capture needs no registration: the
        regions are IPC-shared at construction and tile epochs live on the device."""
        if out is None:
            out = torch.empty_like(inp)
        ops.qr_all_reduce(self._ptr, inp, out, self.qr_quant_level.value, bool(self.use_fp16_kernels))
        return out

    def close(self):
        if not self.disabled and getattr(self, "_ptr", 0):
            ops.qr_destroy(self._ptr)
            self._ptr = 0
            self.disabled = True

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
