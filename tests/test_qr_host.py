"""Host logic of QuickAllReduce (aiter_b200/dist/quick_all_reduce.py) on CPU: the
settings read from the reference's environment variables
(aiter/dist/device_communicators/quick_all_reduce.py:29-37, 210-233) and the
eligibility rule (dtype, 16-byte multiple, dense storage, the window of the B200
crossover table, the registered size)."""
import pytest
import torch

from aiter_b200.dist import quick_all_reduce as qmod
from aiter_b200.dist.quick_all_reduce import MB, QuickAllReduce, QuickReduceRegime, QuickReduceSettings


def _enabled(world, level, max_bytes=2048 * MB, fp16=True):
    q = object.__new__(QuickAllReduce)
    q.disabled = False
    q._ptr = 0
    q.world_size = world
    q.settings = QuickReduceSettings(QuickReduceRegime[level], fp16, max_bytes)
    q.max_bytes = max_bytes
    return q


def test_disabled_without_an_sm100_gpu(monkeypatch):
    monkeypatch.setenv("AITER_QUICK_REDUCE_QUANTIZATION", "INT4")
    q = QuickAllReduce(group=None, device="cpu")
    assert q.disabled


def test_settings_from_environment(monkeypatch):
    monkeypatch.delenv("AITER_QUICK_REDUCE_QUANTIZATION", raising=False)
    assert QuickReduceSettings.from_env() is None
    for bad in ("INT5", "NONE"):
        monkeypatch.setenv("AITER_QUICK_REDUCE_QUANTIZATION", bad)
        assert QuickReduceSettings.from_env() is None
    monkeypatch.setenv("AITER_QUICK_REDUCE_QUANTIZATION", "FP8")
    monkeypatch.setenv("AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB", "64")
    monkeypatch.setenv("AITER_QUICK_REDUCE_CAST_BF16_TO_FP16", "0")
    s = QuickReduceSettings.from_env()
    assert s.level is QuickReduceRegime.FP8 and s.max_bytes == 64 * MB and not s.fp16_kernels
    monkeypatch.delenv("AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB")
    monkeypatch.delenv("AITER_QUICK_REDUCE_CAST_BF16_TO_FP16")
    s = QuickReduceSettings.from_env()
    assert s.max_bytes is None and s.fp16_kernels


def test_crossover_table_decides(monkeypatch):
    monkeypatch.setattr(qmod, "B200_WINDOWS", {(2, "INT4"): (1 * MB, 4 * MB), (8, "FP8"): (16 * MB, 64 * MB)})
    q = _enabled(2, "INT4")
    for dtype in (torch.float16, torch.bfloat16):
        assert q.should_quick_allreduce(torch.empty(MB // 2, dtype=dtype))
        assert q.should_quick_allreduce(torch.empty(4 * MB // 2, dtype=dtype))
        assert not q.should_quick_allreduce(torch.empty(MB // 4, dtype=dtype))
        assert not q.should_quick_allreduce(torch.empty(8 * MB // 2, dtype=dtype))  # above the window
    q = _enabled(8, "FP8")
    assert q.should_quick_allreduce(torch.empty(16 * MB // 2, dtype=torch.float16))
    assert not q.should_quick_allreduce(torch.empty(8 * MB // 2, dtype=torch.float16))
    # a level that never won at this world size keeps every message on the custom allreduce
    assert not _enabled(4, "INT6").should_quick_allreduce(torch.empty(256 * MB // 2, dtype=torch.float16))


def test_measured_windows_are_well_formed():
    for (world, level), (lo, hi) in qmod.B200_WINDOWS.items():
        assert world in QuickAllReduce.WORLD_SIZES and level in QuickReduceRegime.__members__
        assert 0 < lo <= hi and lo % 16 == 0


def test_eligibility_rules(monkeypatch):
    monkeypatch.setattr(qmod, "B200_WINDOWS", {(2, "INT4"): (1 * MB, 64 * MB)})
    q = _enabled(2, "INT4", max_bytes=4 * MB)
    assert not q.should_quick_allreduce(torch.empty(2 * MB // 4, dtype=torch.float32))  # dtype
    assert not q.should_quick_allreduce(torch.empty(2 * MB // 2 + 3, dtype=torch.float16))  # 16-byte multiple
    assert not q.should_quick_allreduce(torch.empty(8 * MB // 2, dtype=torch.float16))  # above the registered size
    x = torch.empty(1024, 2048, dtype=torch.float16)
    assert not q.should_quick_allreduce(x[:, ::2])  # strided
    assert q.should_quick_allreduce(x)
    q.disabled = True
    assert not q.should_quick_allreduce(x)


def test_regime_values_match_kernel_levels():
    assert [QuickReduceRegime[n].value for n in ("FP", "FP8", "INT6", "INT4")] == [0, 1, 2, 3]
    q = _enabled(2, "INT6", fp16=False)
    assert q.qr_quant_level is QuickReduceRegime.INT6 and q.use_fp16_kernels is False
