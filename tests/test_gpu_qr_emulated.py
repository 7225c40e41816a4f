"""Single-GPU parity of the quick allreduce kernel: all W ranks emulated in one
cooperative launch (qr_all_reduce_emulated; CTA row y plays rank y), every rank's
output bit-exact against the restatement of the reference's QuickReduce
(oracle/quick_reduce.py) and identical across ranks.
"""
import numpy as np
import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU"),
]

MODES = [(torch.float16, False), (torch.bfloat16, False), (torch.bfloat16, True)]


def _inputs(world, n, seed, dtype, scale):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(world, n, generator=g) * scale
    if n >= 256:  # an all-zero group, a tiny group and a tied group on every rank
        x[:, 64:128] = 0
        x[:, 128:192] = 1e-6
        x[:, 192:256:2] = 3.0
        x[:, 193:256:2] = -3.0
    return x.to(dtype)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("level", [0, 1, 2, 3])
@pytest.mark.parametrize("dtype,cast", MODES)
def test_quick_allreduce_emulated_ranks(world, level, dtype, cast):
    from aiter_b200 import quick_all_reduce as qops
    from oracle.quick_reduce import quick_allreduce
    name = "fp16" if dtype == torch.float16 else "bf16"
    for i, (n, scale) in enumerate([(8, 1.0), (16384 + 8 * 9, 1e-3), (3 * 16384, 300.0), (16384 * 61 + 64, 1.0)]):
        x = _inputs(world, n, 1000 * world + 10 * level + i, dtype, scale)
        y = qops.qr_all_reduce_emulated(x.cuda(), level, cast)
        torch.cuda.synchronize()
        assert qops.qr_device_error() == 0
        y = y.cpu()
        for r in range(1, world):
            assert torch.equal(y[r].view(torch.int16), y[0].view(torch.int16)), (n, r)
        want = quick_allreduce([x[r].float().numpy() for r in range(world)], level, name, cast)
        got = y[0].float().numpy()
        assert np.array_equal(got, want), (n, int((got != want).sum()))
