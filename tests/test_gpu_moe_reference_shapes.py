"""fused_moe at the shapes the reference's own MoE tests default to, against the oracle:

* op_tests/test_moe_blockscale.py:303-345 -- D=7168, I=256, E=256, top-8, M in {1, 2, 5, 16,
  32} (and 1024 here, for fuller expert blocks);
* op_tests/test_moe_2stage.py:303-389 -- D=7168, I=256, E=257 (not a power of two), top-9.

DeepSeek-like: 56 K blocks in stage 1, 2 in stage 2, two 128-wide inter tiles.  Weights are
drawn and quantised on the GPU (N(0,1)/sqrt(K), 128x128 blocks) and the oracle dequantises
only the experts the tokens are routed to.  Tolerance as the other MoE parity tests
(rtol = atol = 2e-2, at most 1 % of elements beyond 1e-2).
"""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from gpu_util import check_no_device_error, requires_cuda
from oracle import moe

pytestmark = [pytest.mark.gpu, requires_cuda]

_CACHE = {}


def _weights(D, I, E):
    key = (D, I, E)
    if key not in _CACHE:
        from aiter_b200 import weights as W
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(D + I + E)
        w1q, w1s = W.quant_weight_128x128(torch.randn(E, 2 * I, D, device=dev, generator=g) / D ** 0.5)
        w2q, w2s = W.quant_weight_128x128(torch.randn(E, D, I, device=dev, generator=g) / I ** 0.5)
        torch.cuda.empty_cache()
        _CACHE.clear()
        _CACHE[key] = (w1q, w1s, w2q, w2s, w1q.view(torch.uint8).cpu().numpy(), w1s.cpu().numpy(),
                       w2q.view(torch.uint8).cpu().numpy(), w2s.cpu().numpy())
    return _CACHE[key]


def _run(M, D, I, E, k, seed):
    w1q, w1s, w2q, w2s, w1n, w1sn, w2n, w2sn = _weights(D, I, E)
    dev = w1q.device
    g = torch.Generator(device=dev).manual_seed(seed)
    hidden = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
    tw, tid = aiter.fused_topk(hidden, torch.randn(M, E, device=dev, generator=g), k, True)
    out = aiter.fused_moe(hidden, w1q, w2q, tw, tid, quant_type=aiter.QuantType.per_1x128,
                          activation=aiter.ActivationType.Silu, w1_scale=w1s, w2_scale=w2s)
    torch.cuda.synchronize()
    check_no_device_error()
    ref = moe.fused_moe_fp8_blockscale(hidden.float().cpu().numpy(), w1n, w1sn, w2n, w2sn, tw.cpu().numpy(),
                                       tid.cpu().numpy())
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=2e-2, atol=2e-2)
    assert (np.abs(got - ref) > 1e-2 + 1e-2 * np.abs(ref)).mean() <= 0.01


@pytest.mark.parametrize("M", [1, 2, 5, 16, 32, 1024])
def test_blockscale_reference_test_shapes(M):
    _run(M, 7168, 256, 256, 8, seed=M)


@pytest.mark.parametrize("M", [1, 32, 300])
def test_two_stage_reference_test_shapes(M):
    _run(M, 7168, 256, 257, 9, seed=1000 + M)
