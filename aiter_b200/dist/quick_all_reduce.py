"""Quick allreduce communicator: the quantised two-shot allreduce of libaiter_b200.so
(csrc/quick_reduce.cu) behind the interface of the reference's QuickAllReduce
(aiter/dist/device_communicators/quick_all_reduce.py:20-268) -- constructed with a
CPU (gloo) process group and a device, with `disabled`, `should_quick_allreduce(inp)`,
`quick_all_reduce(inp, out=None)` and `close()`.

Settings come from the reference's environment variables, with their meanings:
AITER_QUICK_REDUCE_QUANTIZATION names the level of the NVLink traffic (FP, FP8, INT6,
INT4; unset or NONE leaves the communicator disabled), AITER_QUICK_REDUCE_CAST_BF16_TO_FP16
(default 1) runs bf16 messages on the fp16 kernels, AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB
sets the registered size (default: the library's qr_max_size()).

Which messages take the quick allreduce rather than the custom IPC allreduce is a
property of the interconnect: `B200_WINDOWS` holds, per world size and level, the
range of message sizes in which the quick allreduce was faster than the custom
allreduce on B200 GPUs (NVLink 5 through NVSwitch), from `bench.py --mode
allreduce`; a level that never won at a world size is absent, and such messages
stay on the custom allreduce.
"""
import dataclasses
import logging
import os
from enum import Enum
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist

from .. import quick_all_reduce as ops

logger = logging.getLogger("aiter_b200")

MB = 1 << 20


class QuickReduceRegime(Enum):
    """Levels of the quick allreduce, numbered as the kernels take them."""
    FP = 0
    FP8 = 1
    INT6 = 2
    INT4 = 3
    NONE = 4


# (world size, level) -> (smallest, largest) message in bytes for which the quick
# allreduce beat the custom IPC allreduce on B200, measured with bench.py --mode
# allreduce (fp16 kernels, sizes 64 KB .. 256 MB in powers of two):
# * world size 2: no level won at any size (the one-shot custom allreduce ran at
#   0.46-0.53 of the 770 GB/s peer bandwidth; quantising and decoding cost more than the
#   NVLink bytes they save), so no entry;
# * world size 8: every level won from 2 MB (where the two-shot's second barrier and
#   peer reads dominate) up to 4 MB (FP) or 8 MB (FP8, INT6, INT4); from 16 MB on the
#   custom allreduce was faster again;
# * world size 4: not measured, no entry.
B200_WINDOWS = {
    (8, "FP"): (2 * MB, 4 * MB),
    (8, "FP8"): (2 * MB, 8 * MB),
    (8, "INT6"): (2 * MB, 8 * MB),
    (8, "INT4"): (2 * MB, 8 * MB),
}


@dataclasses.dataclass(frozen=True)
class QuickReduceSettings:
    level: QuickReduceRegime
    fp16_kernels: bool
    max_bytes: Optional[int]  # None: the library's qr_max_size()

    @staticmethod
    def from_env() -> Optional["QuickReduceSettings"]:
        name = os.environ.get("AITER_QUICK_REDUCE_QUANTIZATION", "NONE")
        if name not in QuickReduceRegime.__members__:
            logger.warning("AITER_QUICK_REDUCE_QUANTIZATION=%s is not one of %s; quick allreduce disabled",
                           name, ", ".join(QuickReduceRegime.__members__))
            return None
        level = QuickReduceRegime[name]
        if level is QuickReduceRegime.NONE:
            return None
        mb = int(os.environ.get("AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB", "0"))
        return QuickReduceSettings(level=level,
                                   fp16_kernels=os.environ.get("AITER_QUICK_REDUCE_CAST_BF16_TO_FP16", "1") != "0",
                                   max_bytes=mb * MB if mb > 0 else None)


def _on_sm100() -> bool:
    try:
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except RuntimeError:
        return False


def _dense(t: torch.Tensor) -> bool:
    """Contiguous, or a view whose storage holds exactly its elements from its offset."""
    if t.is_contiguous():
        return True
    tail = t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()
    return tail == t.numel() * t.element_size()


class QuickAllReduce:
    WORLD_SIZES = (2, 4, 8)
    DTYPES = (torch.float16, torch.bfloat16)

    def __init__(self, group, device: Union[int, str, torch.device]) -> None:
        self.disabled = True
        self._ptr = 0
        self.settings = QuickReduceSettings.from_env()
        if self.settings is None or not _on_sm100():
            return
        if dist.get_backend(group) == dist.Backend.NCCL:
            raise ValueError("the quick allreduce exchanges its IPC handles over a CPU (gloo) group, not NCCL")
        self.group = group
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        if self.world_size not in self.WORLD_SIZES:
            if self.world_size > 1:
                logger.warning("quick allreduce disabled: world size %d is not one of %s", self.world_size,
                               self.WORLD_SIZES)
            return
        self.device = torch.device(f"cuda:{device}") if isinstance(device, int) else torch.device(device)
        self.init_quick_all_reduce()

    def init_quick_all_reduce(self):
        """Allocate this rank's IPC regions and open the peers' (the handles travel over
        the CPU group)."""
        with torch.cuda.device(self.device):
            self._ptr = ops.init_custom_qr(self.rank, self.world_size, self.settings.max_bytes)
        self.max_bytes = self.settings.max_bytes or ops.qr_max_size()
        try:
            self.create_shared_buffer()
        except Exception:
            ops.qr_destroy(self._ptr)
            self._ptr = 0
            raise
        self.disabled = False

    def create_shared_buffer(self):
        handles = [None] * self.world_size
        dist.all_gather_object(handles, ops.qr_get_handle(self._ptr), group=self.group)
        ops.qr_open_handles(self._ptr, handles)

    # the names the reference's callers read
    @property
    def qr_quant_level(self) -> QuickReduceRegime:
        return self.settings.level

    @property
    def use_fp16_kernels(self) -> bool:
        return self.settings.fp16_kernels

    def window(self) -> Optional[Tuple[int, int]]:
        """(smallest, largest) message that goes to the quick allreduce at this world
        size and level, None when the level never beat the custom allreduce on B200."""
        return B200_WINDOWS.get((self.world_size, self.settings.level.name))

    def should_quick_allreduce(self, inp: torch.Tensor) -> bool:
        if self.disabled or inp.dtype not in self.DTYPES or not _dense(inp):
            return False
        nbytes = inp.numel() * inp.element_size()
        w = self.window()
        return nbytes % 16 == 0 and w is not None and w[0] <= nbytes <= min(w[1], self.max_bytes)

    def quick_all_reduce(self, inp: torch.Tensor, *, out: torch.Tensor = None) -> torch.Tensor:
        """Out-of-place quick allreduce.  Graph capture needs no registration: the
        regions are IPC-shared at construction and tile epochs live on the device."""
        if out is None:
            out = torch.empty_like(inp)
        ops.qr_all_reduce(self._ptr, inp, out, self.settings.level.value, self.settings.fp16_kernels)
        return out

    def close(self):
        if self._ptr:
            ops.qr_destroy(self._ptr)
            self._ptr = 0
        self.disabled = True

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
