"""The torch custom-op registration (the reference's torch_compile_guard /
fused_moe_fake): every operator is reachable as torch.ops.aiter_b200.* and its fake
implementation gives the right output metadata without running a kernel (CPU)."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import aiter_b200  # noqa: F401
from aiter_b200 import dtypes


def test_ops_are_registered():
    for name in ("fused_moe_", "topk_softmax", "grouped_topk", "biased_grouped_topk", "moe_sorting_fwd",
                 "gemm_a16w16"):
        assert hasattr(torch.ops.aiter_b200, name), name


def test_fused_moe_fake_shape():
    M, D, I, E, k = 7, 1024, 512, 8, 2
    with FakeTensorMode():
        x = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")
        w1 = torch.empty(E, 2 * I, D, dtype=dtypes.fp8, device="cuda")
        w2 = torch.empty(E, D, I, dtype=dtypes.fp8, device="cuda")
        s1 = torch.empty(E, 2 * I // 128, D // 128, device="cuda")
        s2 = torch.empty(E, D // 128, I // 128, device="cuda")
        tw = torch.empty(M, k, device="cuda")
        ti = torch.empty(M, k, dtype=torch.int32, device="cuda")
        y = torch.ops.aiter_b200.fused_moe_(x, w1, w2, tw, ti, None, 0, 4, False, s1, s2)
        assert y.shape == (M, D) and y.dtype == torch.bfloat16 and y.device.type == "cuda"


def test_gemm_fake_shape_and_mutating_ops_trace():
    with FakeTensorMode():
        a = torch.empty(5, 256, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(384, 256, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.aiter_b200.gemm_a16w16(a, w)
        assert y.shape == (5, 384) and y.dtype == torch.bfloat16
        g = torch.empty(5, 64, device="cuda")
        tw = torch.empty(5, 4, device="cuda")
        ti = torch.empty(5, 4, dtype=torch.int32, device="cuda")
        tei = torch.empty(5, 4, dtype=torch.int32, device="cuda")
        assert torch.ops.aiter_b200.topk_softmax(tw, ti, tei, g, True) is None
