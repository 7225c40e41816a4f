"""1 x group fp8 quantisation vs the oracle (`pertoken_quant` over 128 groups,
aiter/ops/quant.py:42-72): codes and scales bit-exact.  The int8 output (the default
dtype of the reference's per_group_quant_hip) is bit-exact as well."""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from gpu_util import codes, dev, requires_cuda, to_dev
from oracle import codecs, quant

pytestmark = [pytest.mark.gpu, requires_cuda]


@pytest.mark.parametrize("M,K", [(1, 128), (33, 1024), (4096, 4096), (7, 7168)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_group_quant_bit_exact(M, K, dtype):
    rng = np.random.default_rng(M * 7 + K)
    x = rng.standard_normal((M, K), dtype=np.float32) * 3
    x[0, :128] = 0.0            # zero group -> scale 1
    if M > 2:
        x[2, 5] = 900.0         # outlier
    xt = to_dev(x, dtype)
    q, s = aiter.per_group_quant_hip(xt, quant_dtype=torch.float8_e4m3fn, group_size=128)
    torch.cuda.synchronize()
    q0, s0 = quant.per_1x128_quant(xt.float().cpu().numpy())
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s0.view(np.uint32))
    assert np.array_equal(codes(q), q0)


@pytest.mark.parametrize("group", [32, 64])
def test_group_quant_small_groups(group):
    rng = np.random.default_rng(group)
    x = rng.standard_normal((64, 512), dtype=np.float32)
    xt = to_dev(x, torch.bfloat16)
    q, s = aiter.per_group_quant_hip(xt, quant_dtype=torch.float8_e4m3fn, group_size=group)
    q0, s0 = quant.per_1x128_quant(xt.float().cpu().numpy(), group=group)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s0.view(np.uint32))
    assert np.array_equal(codes(q), q0)


def test_group_quant_transposed_scale_and_num_rows():
    rng = np.random.default_rng(1)
    M, K = 50, 512
    x = to_dev(rng.standard_normal((M, K), dtype=np.float32), torch.bfloat16)
    nr = torch.tensor([30], dtype=torch.int32, device=dev())
    q = torch.full((M, K), 0.5, dtype=torch.float8_e4m3fn, device=dev())
    s = torch.full((M, K // 128), -1.0, device=dev())
    aiter.dynamic_per_token_scaled_quant(q, x.view(-1, 128), s, shuffle_scale=True, num_rows=nr)
    q0, s0 = quant.per_1x128_quant(x.float().cpu().numpy())
    st = s.cpu().numpy().reshape(-1)
    # transposed layout [K/128, M]: group (row r, col c) at c * M + r
    for r in range(30):
        for c in range(K // 128):
            assert st[c * M + r] == s0[r, c]
    assert np.array_equal(codes(q)[:30], q0[:30])
    assert np.all(codes(q)[30:] == codecs.fp8_e4m3_encode(np.float32(0.5)))


@pytest.mark.parametrize("group", [32, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_group_quant_int8_bit_exact(group, dtype):
    rng = np.random.default_rng(group + 11)
    x = rng.standard_normal((40, 1024), dtype=np.float32) * 3
    x[0, :group] = 0.0          # zero group -> scale 1
    x[2, 5] = -900.0            # outlier
    xt = to_dev(x, dtype)
    q, s = aiter.per_group_quant_hip(xt, group_size=group)   # default dtype: int8
    torch.cuda.synchronize()
    assert q.dtype == torch.int8
    q0, s0 = quant.per_group_quant_i8(xt.float().cpu().numpy(), group=group)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s0.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q0)
