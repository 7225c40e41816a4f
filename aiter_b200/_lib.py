"""ctypes binding of the in-tree C-ABI library (libaiter_b200.so).

Mirrors the reference's torch-free ctypes call path (aiter/jit/core.py:1105-1363):
tensors travel as `aiter_tensor_t*` (NULL for None), Optional[int] as -1, bools as
int, floats as float, strings as bytes, and the current CUDA stream of the first
tensor's device is appended.  A non-zero status raises
`RuntimeError("<fn> failed: <message>")` with the thread-local message of
`aiter_get_last_error()`.

There is no fallback: if the library is missing, every op raises.
"""
import ctypes
import os
import struct
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libaiter_b200.so")

# AiterDtype values (csrc/include/aiter_enum.h:26-41)
_DTYPE_CODES = {
    torch.float8_e4m3fn: 0,
    torch.float8_e8m0fnu: 1,
    torch.float16: 2,
    torch.bfloat16: 3,
    torch.float32: 4,
    torch.float4_e2m1fn_x2: 6,
    torch.uint32: 7,
    torch.int32: 8,
    torch.int16: 9,
    torch.int8: 10,
    torch.uint8: 11,
    torch.int64: 12,
    torch.uint64: 13,
}


class aiter_tensor_t(ctypes.Structure):
    """Byte-compatible with aiter_tensor_t (csrc/include/aiter_tensor.h:8-18)."""
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("numel_", ctypes.c_size_t),
        ("ndim", ctypes.c_int),
        ("shape", ctypes.c_int64 * 8),
        ("strides", ctypes.c_int64 * 8),
        ("dtype_", ctypes.c_int),
        ("device_id", ctypes.c_int),
    ]


assert ctypes.sizeof(aiter_tensor_t) == 160


def dtype_code(dt):
    try:
        return _DTYPE_CODES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


_PACK = struct.Struct("<QQi4x8q8qii")  # the 160-byte aiter_tensor_t layout
_ZEROS = (0,) * 8
# one format per rank: the unused shape / stride slots are pad bytes (zeros), so the
# tensor's own shape and stride tuples go in without concatenation
_PACKS = [struct.Struct(f"<QQi4x{nd}q{(8 - nd) * 8}x{nd}q{(8 - nd) * 8}xii") for nd in range(9)]
assert all(p.size == 160 for p in _PACKS)


def to_aiter(t: torch.Tensor) -> aiter_tensor_t:
    nd = t.dim()
    if nd > 8:
        raise ValueError("at most 8 dims")
    n = t.numel()
    try:
        code = _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None
    return aiter_tensor_t.from_buffer_copy(_PACKS[nd].pack(t.data_ptr() if n > 0 else 0, n, nd, *t.shape,
                                                           *t.stride(), code, t.get_device()))


def current_stream_ptr(device_index: int) -> int:
    """Raw cudaStream_t of the current torch stream of a device."""
    return torch._C._cuda_getCurrentRawStream(device_index)


_lock = threading.Lock()
_lib = None

T = "tensor"
OT = "opt_tensor"
I64 = "int"
OI64 = "opt_int"
B = "bool"
F = "float"
S = "str"

# name -> argument kinds (stream appended) ; ret int status
SIGNATURES = {
    "topk_softmax": [T, T, OT, T, B, I64, S],
    "grouped_topk": [T, T, T, I64, I64, B, B, F],
    "biased_grouped_topk": [T, T, T, T, I64, I64, B, F],
    "moe_sorting_fwd": [T, T, T, T, T, T, OT, I64, I64, OT, OT, I64, OT, OT],
    "moe_sorting_fwd_static_scratch": [T, T, T, T, T, T, OT, I64, I64, OT, OT, I64, OT],
    "dynamic_per_token_scaled_quant": [T, T, T, OT, B, OT, I64],
    "moe_gather_quant_1x128": [T, OT, T, I64, T, T],
    "mxfp4_to_fp8_blockscale": [T, T, T, T, OT],
    "gemm_a16w16": [T, T, T],
    "dynamic_per_group_scaled_quant_fp4": [T, T, T, I64, B, OT, I64],
    "mxfp4_moe_sort_hip": [T, T, T, T, I64, I64],
    "fused_dynamic_mxfp4_quant_moe_sort_hip": [T, T, T, T, T, I64, I64, I64],
    "moe_stage1_fp8_blockscale": [T, T, T, T, T, T, T, T, T, I64, I64, I64],
    "moe_stage1_fp8_blockscale_ex": [T, T, T, T, T, T, T, T, T, I64, I64, I64, OT, I64],
    "moe_stage2_fp8_blockscale": [T, T, T, T, T, T, T, OT, T, I64],
    "topk_sigmoid": [T, T, T],
    "moe_sum": [T, T],
    "silu_and_mul": [T, T],
    "gelu_and_mul": [T, T],
    "gelu_tanh_and_mul": [T, T],
    "scaled_silu_and_mul": [T, T, T],
    "moe_stage1_fp8_blockscale_bias": [T, T, T, T, T, T, T, T, T, I64, I64, I64, OT, I64, T],
    "moe_stage2_fp8_blockscale_bias": [T, T, T, T, T, T, T, OT, T, I64, T],
    "moe_stage1_a8w4": [T, T, T, T, T, T, T, T, T, I64, I64, I64, OT, I64, OT],
    "moe_stage2_a8w4": [T, T, T, T, T, T, T, OT, T, I64, OT],
    "mxfp4_moe_weight_scale_chunks": [T, T],
}

_CT = {T: ctypes.POINTER(aiter_tensor_t), OT: ctypes.POINTER(aiter_tensor_t), I64: ctypes.c_int64,
       OI64: ctypes.c_int64, B: ctypes.c_int, F: ctypes.c_float, S: ctypes.c_char_p}


def lib():
    """Load libaiter_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m aiter_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        L.aiter_ctypes_abi_version.restype = ctypes.c_int
        L.aiter_get_last_error.restype = ctypes.c_char_p
        L.aiter_clear_last_error.restype = None
        L.moe_sorting_get_workspace_size.restype = ctypes.c_int64
        L.moe_sorting_get_workspace_size.argtypes = [ctypes.c_int64] * 4
        L.aiter_device_error.restype = ctypes.c_int
        L.aiter_device_error.argtypes = [ctypes.c_int]
        L.qr_max_size.restype = ctypes.c_int64
        L.qr_max_size.argtypes = []
        c64, vp, p64 = ctypes.c_int64, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)
        for name, args in (("custom_ar_init", [c64, c64, c64, c64, p64, vp]),
                           ("custom_ar_open_peers", [c64, vp]), ("custom_ar_open_loopback", [c64]),
                           ("custom_ar_next_buffer", [c64, p64, p64]),
                           ("custom_ar_next_buffer_ex", [c64, c64, p64, p64]),
                           ("custom_ar_all_reduce", [c64, ctypes.POINTER(aiter_tensor_t),
                                                     ctypes.POINTER(aiter_tensor_t), c64, vp]),
                           ("custom_ar_all_reduce_fp8", [c64, ctypes.POINTER(aiter_tensor_t),
                                                         ctypes.POINTER(aiter_tensor_t), vp]),
                           ("custom_ar_gemm_all_reduce", [c64, ctypes.POINTER(aiter_tensor_t),
                                                          ctypes.POINTER(aiter_tensor_t),
                                                          ctypes.POINTER(aiter_tensor_t), c64, vp]),
                           ("custom_ar_gemm_all_reduce_fused", [c64, ctypes.POINTER(aiter_tensor_t),
                                                                ctypes.POINTER(aiter_tensor_t),
                                                                ctypes.POINTER(aiter_tensor_t), c64, vp]),
                           ("custom_ar_allreduce_rmsnorm", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 5 +
                            [ctypes.c_float, ctypes.POINTER(aiter_tensor_t), vp]),
                           ("custom_ar_allreduce_rmsnorm_ex", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 5 +
                            [ctypes.c_float, ctypes.POINTER(aiter_tensor_t), c64, vp]),
                           ("custom_ar_all_gather", [c64, ctypes.POINTER(aiter_tensor_t),
                                                     ctypes.POINTER(aiter_tensor_t), c64, vp]),
                           ("custom_ar_reduce_scatter", [c64, ctypes.POINTER(aiter_tensor_t),
                                                         ctypes.POINTER(aiter_tensor_t), vp]),
                           ("custom_ar_dispose", [c64]), ("custom_ar_device_error", [ctypes.c_int]),
                           ("init_custom_qr", [c64, c64, c64, c64, p64, vp]), ("qr_open_handles", [c64, vp]),
                           ("qr_all_reduce", [c64, ctypes.POINTER(aiter_tensor_t), ctypes.POINTER(aiter_tensor_t),
                                              c64, c64, vp]),
                           ("qr_all_reduce_emulated", [c64, ctypes.POINTER(aiter_tensor_t),
                                                       ctypes.POINTER(aiter_tensor_t), c64, c64, vp]),
                           ("qr_destroy", [c64]), ("qr_device_error", [ctypes.c_int]),
                           ("ep_init", [c64] * 10 + [p64, vp]), ("ep_open_handles", [c64, vp]),
                           ("ep_buffers", [c64, p64, p64]),
                           ("ep_dispatch", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 4 + [vp]),
                           ("ep_combine", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 2 + [vp]),
                           ("ep_emu_init", [c64] * 9 + [p64]), ("ep_emu_buffers", [c64, c64, p64, p64]),
                           ("ep_emu_dispatch", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 4 + [vp]),
                           ("ep_emu_combine", [c64] + [ctypes.POINTER(aiter_tensor_t)] * 2 + [vp]),
                           ("ep_destroy", [c64]), ("ep_device_error", [ctypes.c_int])):
            fn = getattr(L, name)
            fn.restype = ctypes.c_int
            fn.argtypes = args
        for name, kinds in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [_CT[k] for k in kinds] + [ctypes.c_void_p]
        if L.aiter_ctypes_abi_version() != 2:
            raise RuntimeError("unexpected C ABI version")
        _lib = L
    return _lib


def call(name, *args, stream=None):
    """Call entry `name` with Python values converted per SIGNATURES[name]."""
    L = lib()
    kinds = SIGNATURES[name]
    if len(args) != len(kinds):
        raise TypeError(f"{name}: expected {len(kinds)} arguments, got {len(args)}")
    cargs = []
    keep = []
    device = None
    for k, v in zip(kinds, args):
        if k in (T, OT):
            if v is None:
                if k == T:
                    raise TypeError(f"{name}: a required tensor is None")
                cargs.append(ctypes.POINTER(aiter_tensor_t)())
            else:
                if not isinstance(v, torch.Tensor):
                    raise TypeError(f"{name}: expected a tensor, got {type(v).__name__}")
                if device is None and v.is_cuda:
                    device = v.get_device()
                a = to_aiter(v)
                keep.append(a)
                cargs.append(ctypes.byref(a))
        elif k == OI64:
            cargs.append(-1 if v is None else int(v))
        elif k == I64:
            cargs.append(int(v))
        elif k == B:
            cargs.append(1 if v else 0)
        elif k == F:
            cargs.append(float(v))
        elif k == S:
            cargs.append(None if v is None else v.encode())
    if stream is None:
        stream = current_stream_ptr(device) if device is not None else 0
    # every entry point clears the thread's last error on entry
    ret = getattr(L, name)(*cargs, ctypes.c_void_p(stream))
    if ret != 0:
        raw = L.aiter_get_last_error()
        msg = raw.decode(errors="replace") if raw else f"status={ret}"
        L.aiter_clear_last_error()
        raise RuntimeError(f"{name} failed: {msg}")
    return None


def check_status(name, ret):
    """Raise RuntimeError for a non-zero status of a directly called entry point."""
    if ret != 0:
        L = lib()
        raw = L.aiter_get_last_error()
        msg = raw.decode(errors="replace") if raw else f"status={ret}"
        L.aiter_clear_last_error()
        raise RuntimeError(f"{name} failed: {msg}")


def device_view(ptr, shape, dtype, device):
    """A tensor over library-owned device memory at `ptr` (no copy; the memory
    stays owned by the library object that returned the pointer)."""
    esz = torch.empty((), dtype=dtype).element_size()
    typestr = {1: "|u1", 2: "<i2", 4: "<i4", 8: "<i8"}[esz]

    class _View:
        pass

    v = _View()
    v.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": typestr,
                                  "data": (int(ptr), False), "version": 3, "strides": None}
    return torch.as_tensor(v, device=device).view(dtype)


def device_error(clear=True):
    """Error word of the device-side bounded waits (0 = none, 1 = a wait timed out)."""
    return lib().aiter_device_error(1 if clear else 0)


def exported_symbols():
    """Entry points declared in include/aiter_b200.h."""
    import re
    hdr = os.path.join(os.path.dirname(_PKG), "include", "aiter_b200.h")
    src = open(hdr).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:int|int64_t|void|const char\*)\s+\**(\w+)\s*\(", src, flags=re.M)
    return names
