"""Host logic of QuickAllReduce (aiter_b200/dist/quick_all_reduce.py) on CPU: the
enable conditions and the eligibility rule of the reference
(aiter/dist/device_communicators/quick_all_reduce.py:29-37, 97-130, 210-233)."""
import pytest
import torch

from aiter_b200.dist import quick_all_reduce as qmod
from aiter_b200.dist.quick_all_reduce import MB, QuickAllReduce, QuickReduceRegime


def _enabled(world, regime, fp16_kernels=1, max_size=2048 * MB):
    q = object.__new__(QuickAllReduce)
    q.disabled = False
    q.world_size = world
    q.qr_quant_level = QuickReduceRegime[regime]
    q.use_fp16_kernels = fp16_kernels
    q.qr_max_size = max_size
    return q


def test_disabled_without_an_sm100_gpu(monkeypatch):
    monkeypatch.setenv("AITER_QUICK_REDUCE_QUANTIZATION", "INT4")
    q = QuickAllReduce(group=None, device="cpu")
    assert q.disabled


def test_not_requested_without_a_regime(monkeypatch):
    monkeypatch.delenv("AITER_QUICK_REDUCE_QUANTIZATION", raising=False)
    assert not qmod.quick_ar_requested()
    monkeypatch.setenv("AITER_QUICK_REDUCE_QUANTIZATION", "INT5")
    assert not qmod.quick_ar_requested()


@pytest.mark.parametrize("world,regime,mb_ok,mb_small", [
    (2, "INT4", 1, 0.5), (4, "FP8", 16, 8), (8, "FP", 16, 8), (8, "INT6", 4, 2)])
def test_min_sizes_fp16_kernels(world, regime, mb_ok, mb_small):
    q = _enabled(world, regime)
    for dtype in (torch.float16, torch.bfloat16):  # bf16 runs the fp16 kernels: fp16 thresholds
        ok = torch.empty(int(mb_ok * MB) // 2, dtype=dtype)
        small = torch.empty(int(mb_small * MB) // 2, dtype=dtype)
        assert q.should_quick_allreduce(ok)
        assert not q.should_quick_allreduce(small)


def test_min_sizes_native_bf16():
    q = _enabled(8, "INT4", fp16_kernels=0)
    assert not q.should_quick_allreduce(torch.empty(64 * MB // 2, dtype=torch.bfloat16))
    q = _enabled(2, "FP", fp16_kernels=0)
    assert q.should_quick_allreduce(torch.empty(2 * MB // 2, dtype=torch.bfloat16))


def test_eligibility_rules():
    q = _enabled(2, "INT4", max_size=4 * MB)
    assert not q.should_quick_allreduce(torch.empty(2 * MB // 4, dtype=torch.float32))  # dtype
    assert not q.should_quick_allreduce(torch.empty(2 * MB // 2 + 3, dtype=torch.float16))  # 16-byte multiple
    assert not q.should_quick_allreduce(torch.empty(8 * MB // 2, dtype=torch.float16))  # above max_size
    x = torch.empty(1024, 2048, dtype=torch.float16)
    assert not q.should_quick_allreduce(x[:, ::2])  # strided
    assert q.should_quick_allreduce(x)
    q.disabled = True
    assert not q.should_quick_allreduce(x)


def test_regime_values_match_kernel_levels():
    assert [QuickReduceRegime[n].value for n in ("FP", "FP8", "INT6", "INT4")] == [0, 1, 2, 3]
