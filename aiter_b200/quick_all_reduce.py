"""Quick allreduce operators, the reference's `aiter.ops.quick_all_reduce`
(aiter/ops/quick_all_reduce.py:13-38): init_custom_qr, qr_get_handle,
qr_open_handles, qr_all_reduce, qr_destroy, qr_max_size.

The communicator is created on the current CUDA device, as the reference's
`DeviceComms::init` allocates on the current HIP device
(csrc/include/quick_all_reduce.cuh:884-915).  Handles are 64-byte uint8 CPU
tensors.
"""
import ctypes
from typing import List, Optional

import torch

from . import _lib

IPC_HANDLE_BYTES = 64
_handles = {}  # communicator -> its own IPC handle (bytes)


def init_custom_qr(rank: int, world_size: int, qr_max_size: Optional[int] = None) -> int:
    L = _lib.lib()
    ctx = ctypes.c_int64(0)
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    dev = torch.cuda.current_device()
    size = -1 if qr_max_size is None else int(qr_max_size)
    _lib.check_status("init_custom_qr", L.init_custom_qr(int(rank), int(world_size), size, dev, ctypes.byref(ctx),
                                                         handle))
    _handles[ctx.value] = handle.raw
    return ctx.value


def qr_get_handle(fa: int) -> torch.Tensor:
    try:
        raw = _handles[fa]
    except KeyError:
        raise RuntimeError("unknown quick allreduce communicator") from None
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone()


def qr_open_handles(fa: int, handles: List[torch.Tensor]) -> None:
    blobs = []
    for h in handles:
        b = bytes(h.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
        if len(b) != IPC_HANDLE_BYTES:
            raise RuntimeError("malformed IPC handle")
        blobs.append(b)
    _lib.check_status("qr_open_handles", _lib.lib().qr_open_handles(int(fa), b"".join(blobs)))


def qr_all_reduce(fa: int, inp: torch.Tensor, out: torch.Tensor, quant_level: int, cast_bf2half: bool = False) -> None:
    a, b = _lib.to_aiter(inp), _lib.to_aiter(out)
    st = _lib.current_stream_ptr(inp.get_device())
    ret = _lib.lib().qr_all_reduce(int(fa), ctypes.byref(a), ctypes.byref(b), int(quant_level),
                                   1 if cast_bf2half else 0, st)
    if ret:
        _lib.check_status("qr_all_reduce", ret)


def qr_all_reduce_emulated(inp: torch.Tensor, quant_level: int, cast_bf2half: bool = False) -> torch.Tensor:
    """Test hook: the quick allreduce of inp.shape[0] ranks (2, 4 or 8) emulated on
    one GPU in one launch; row r of the result is rank r's output."""
    out = torch.empty_like(inp)
    a, b = _lib.to_aiter(inp), _lib.to_aiter(out)
    st = _lib.current_stream_ptr(inp.get_device())
    ret = _lib.lib().qr_all_reduce_emulated(int(inp.shape[0]), ctypes.byref(a), ctypes.byref(b), int(quant_level),
                                            1 if cast_bf2half else 0, st)
    if ret:
        _lib.check_status("qr_all_reduce_emulated", ret)
    return out


def qr_destroy(fa: int) -> None:
    if fa:
        _handles.pop(fa, None)
        _lib.check_status("qr_destroy", _lib.lib().qr_destroy(int(fa)))


def qr_max_size() -> int:
    return int(_lib.lib().qr_max_size())


def qr_device_error(clear: bool = True) -> int:
    """Error word of the quick allreduce's bounded peer waits (0 = none)."""
    return _lib.lib().qr_device_error(1 if clear else 0)
