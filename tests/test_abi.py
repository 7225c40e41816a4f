"""C-ABI boundary checks that need no GPU: the library loads, exports every entry
point include/aiter_b200.h declares, and reports argument errors through the
status + thread-local message bridge (csrc/include/aiter_ctypes_error.h:56-130)."""
import ctypes
import os

import pytest
import torch

from aiter_b200 import _lib


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = _lib.exported_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/aiter_b200.h but not exported"


def test_abi_version_and_struct_size():
    assert _lib.lib().aiter_ctypes_abi_version() == 2
    assert ctypes.sizeof(_lib.aiter_tensor_t) == 160


def test_error_bridge_reports_bad_arguments():
    w = torch.empty(4, 2, dtype=torch.float32)
    g = torch.empty(4, 8, dtype=torch.float32)
    ids = torch.empty(4, 2, dtype=torch.int64)          # wrong dtype
    with pytest.raises(RuntimeError, match="topk_indices must be i32"):
        _lib.call("topk_softmax", w, ids, None, g, True, 0, "")
    # the message is cleared after it was raised
    assert _lib.lib().aiter_get_last_error() is None


def test_required_tensor_none_rejected_before_the_call():
    with pytest.raises(TypeError):
        _lib.call("moe_sorting_fwd", None, None, None, None, None, None, None, 8, 32, None, None, 0, None)


def test_sorting_workspace_size_policy():
    L = _lib.lib()
    assert L.moe_sorting_get_workspace_size(32, 8, 2, 0) == 0            # one-shot
    assert L.moe_sorting_get_workspace_size(4096, 128, 8, 1) == 0        # forced single CTA
    n = L.moe_sorting_get_workspace_size(4096, 128, 8, 0)
    assert n == ((4096 + 127) // 128) * 128 * 4
    assert L.moe_sorting_get_workspace_size(0, 128, 8, 0) == 0


def test_stage_gemm_rejects_unsupported_block_m():
    t = lambda *s, dt=torch.int32: torch.empty(*s, dtype=dt)
    f8 = torch.float8_e4m3fn
    args = (t(640, 128, dt=f8), t(1, 640, dt=torch.float32), t(2, 256, 128, dt=f8), t(2, 2, 1, dt=torch.float32),
            t(640), t(5), t(2), t(640, 128, dt=f8), t(1, 640, dt=torch.float32), 16, 32, 0)
    with pytest.raises(RuntimeError, match="block_m must be 128"):
        _lib.call("moe_stage1_fp8_blockscale", *args)


def test_gather_quant_rejects_fp8_without_scale():
    f8 = torch.float8_e4m3fn
    with pytest.raises(RuntimeError, match="hidden_scale must not be None"):
        _lib.call("moe_gather_quant_1x128", torch.empty(4, 128, dtype=f8), None, torch.empty(8, dtype=torch.int32),
                  2, torch.empty(8, 128, dtype=f8), torch.empty(1, 8))


def test_tensor_descriptor_packing():
    """to_aiter packs the 160-byte aiter_tensor_t (aiter_tensor.h:8-18) field by field."""
    x = torch.empty(3, 5, 7, dtype=torch.bfloat16)[:, 1:4]          # strided view
    a = _lib.to_aiter(x)
    assert a.ptr == x.data_ptr() and a.numel_ == x.numel() and a.ndim == 3
    assert list(a.shape)[:3] == [3, 3, 7] and list(a.strides)[:3] == list(x.stride())
    assert list(a.shape)[3:] == [0] * 5 and a.dtype_ == 3 and a.device_id == -1
    e = _lib.to_aiter(torch.empty(0, 4, dtype=torch.int32))
    assert e.ptr is None and e.numel_ == 0 and e.dtype_ == 8
    with pytest.raises(ValueError):
        _lib.to_aiter(torch.empty([1] * 9))


def test_gemm_rejects_bad_shapes():
    a = torch.empty(4, 96, dtype=torch.bfloat16)                   # K not a multiple of 64
    w = torch.empty(256, 96, dtype=torch.bfloat16)
    o = torch.empty(4, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="K % 64"):
        _lib.call("gemm_a16w16", a, w, o)
    with pytest.raises(RuntimeError, match="W must be"):
        _lib.call("gemm_a16w16", torch.empty(4, 128, dtype=torch.bfloat16), w, o)


def test_allreduce_entries_reject_bad_context_and_world():
    L = _lib.lib()
    ctx = ctypes.c_int64(0)
    handle = ctypes.create_string_buffer(64)
    assert L.custom_ar_init(0, 9, 1 << 20, 0, ctypes.byref(ctx), handle) != 0
    assert b"world size" in L.aiter_get_last_error()
    x = _lib.to_aiter(torch.empty(8, dtype=torch.bfloat16))
    assert L.custom_ar_all_reduce(0, ctypes.byref(x), ctypes.byref(x), -1, None) != 0
    assert b"null allreduce context" in L.aiter_get_last_error()
    assert L.custom_ar_allreduce_rmsnorm(0, *([ctypes.byref(x)] * 5), 1e-6, None, None) != 0
    assert b"null allreduce context" in L.aiter_get_last_error()
