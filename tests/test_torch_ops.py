"""The torch custom-op registration (the reference's torch_compile_guard /
fused_moe_fake): every operator is reachable as torch.ops.aiter_b200.* and its fake
implementation gives the right output metadata without running a kernel (CPU)."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import aiter_b200  # noqa: F401
from aiter_b200 import dtypes


def test_ops_are_registered():
    for name in ("fused_moe_", "topk_softmax", "grouped_topk", "biased_grouped_topk", "moe_sorting_fwd",
                 "gemm_a16w16", "topk_sigmoid", "moe_sum", "silu_and_mul", "gelu_and_mul", "gelu_tanh_and_mul",
                 "scaled_silu_and_mul"):
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


def test_fused_moe_fake_dtype_follows_fp16_activations():
    M, D, I, E, k = 3, 512, 256, 4, 2
    with FakeTensorMode():
        x = torch.empty(M, D, dtype=torch.float16, device="cuda")
        w1 = torch.empty(E, 2 * I, D, dtype=dtypes.fp8, device="cuda")
        w2 = torch.empty(E, D, I, dtype=dtypes.fp8, device="cuda")
        tw = torch.empty(M, k, device="cuda")
        ti = torch.empty(M, k, dtype=torch.int32, device="cuda")
        y = torch.ops.aiter_b200.fused_moe_(x, w1, w2, tw, ti, None, 2, 4, True)
        assert y.dtype == torch.float16 and y.shape == (M, D)


def test_fused_moe_rejects_what_the_b200_path_does_not_run():
    """Unsupported combinations raise before any kernel launch, as the reference
    raises for combinations it has no kernel for (aiter/fused_moe.py:251-254)."""
    import pytest
    from aiter_b200 import ActivationType, QuantType
    from aiter_b200.fused_moe import fused_moe
    M, D, I, E, k = 2, 256, 128, 4, 2
    x = torch.zeros(M, D, dtype=torch.bfloat16)
    w1 = torch.zeros(E, 2 * I, D, dtype=dtypes.fp8)
    w2 = torch.zeros(E, D, I, dtype=dtypes.fp8)
    tw = torch.zeros(M, k)
    ti = torch.zeros(M, k, dtype=torch.int32)
    sh = w1.clone()
    sh.is_shuffled = True
    with pytest.raises(ValueError, match="pre-shuffled"):
        fused_moe(x, sh, w2, tw, ti, quant_type=QuantType.per_1x128)
    # the experts' biases are used only on the per_1x32 Swiglu path (the reference
    # ignores them elsewhere); there a wrong shape raises before any launch
    w1p = torch.zeros(E, 2 * I, D // 2, dtype=torch.uint8)
    w2p = torch.zeros(E, D, I // 2, dtype=torch.uint8)
    with pytest.raises(ValueError, match="bias1 must be"):
        fused_moe(x, w1p, w2p, tw, ti, quant_type=QuantType.per_1x32, activation=ActivationType.Swiglu,
                  bias1=torch.zeros(E, I))
    with pytest.raises(ValueError, match="bias2 must be"):
        fused_moe(x, w1p, w2p, tw, ti, quant_type=QuantType.per_1x32, activation=ActivationType.Swiglu,
                  bias2=torch.zeros(E, D + 1))
    with pytest.raises(NotImplementedError, match="g1u1"):
        fused_moe(x, w1[:, :I], w2, tw, ti, quant_type=QuantType.per_1x128)
    with pytest.raises(NotImplementedError, match="quant_type"):
        fused_moe(x, w1, w2, tw, ti, quant_type=QuantType.per_Token)
    with pytest.raises(NotImplementedError, match="activation"):
        fused_moe(x, w1, w2, tw, ti, quant_type=QuantType.per_1x128, activation=ActivationType.No)
    # block_size_M takes the reference's tile heights (16 / 32 / 64 / 128, mapped to the
    # 128-row tcgen05 tile); other values raise before any launch
    with pytest.raises(ValueError, match="block_size_M must be"):
        fused_moe(x, w1, w2, tw, ti, quant_type=QuantType.per_1x128, block_size_M=48)



def test_new_mutating_ops_trace_with_fake_tensors():
    """topk_sigmoid, moe_sum and the gated activations trace under FakeTensorMode
    (torch.compile's first step) without running a kernel."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        w = torch.empty(4, 2)
        ids = torch.empty(4, 2, dtype=torch.int32)
        torch.ops.aiter_b200.topk_sigmoid(w, ids, torch.empty(4, 16))
        torch.ops.aiter_b200.moe_sum(torch.empty(4, 2, 64, dtype=torch.bfloat16), torch.empty(4, 64, dtype=torch.bfloat16))
        torch.ops.aiter_b200.silu_and_mul(torch.empty(4, 32, dtype=torch.bfloat16), torch.empty(4, 64, dtype=torch.bfloat16))
        torch.ops.aiter_b200.scaled_silu_and_mul(torch.empty(4, 32, dtype=torch.float8_e4m3fn),
                                                 torch.empty(4, 64), torch.empty(1))
