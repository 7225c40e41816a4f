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
