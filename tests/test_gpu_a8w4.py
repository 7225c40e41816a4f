"""A8W4 (fp8 1x128 activations x MXFP4 weights, the BASELINE config-2 contract).

* weight preparation: the e4m3 x power-of-two block scale values equal the MXFP4
  dequantisation (mxfp4_to_f32 * e8m0_to_f32, aiter/utility/fp4_utils.py:19-69)
  bit for bit, including all-zero groups; blocks that cannot be exact are reported;
* fused_moe(quant_type=per_1x32) against the reference-composed golden output
  (tests/golden, moe_a8w4/cfg0) and against the oracle on sweeps, rtol = atol = 2e-2."""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from aiter_b200 import weights as W
from conftest import golden_group
from gpu_util import check_no_device_error, dev, requires_cuda, to_dev
from oracle import codecs, inputs, moe, quant
from test_gpu_moe import assert_moe_close

pytestmark = [pytest.mark.gpu, requires_cuda]


def _prep(c):
    return (to_dev(c["w1_q"]), to_dev(c["w1_s"]), to_dev(c["w2_q"]), to_dev(c["w2_s"]))


@pytest.mark.parametrize("E,N,K", [(2, 256, 384), (3, 128, 1024)])
def test_mxfp4_expansion_is_exact(E, N, K):
    rng = np.random.default_rng(E * N + K)
    w = (rng.standard_normal((E, N, K), dtype=np.float32) * rng.choice([0.1, 1.0, 10.0], size=(E, N, 1))).astype(np.float32)
    w[0, :5, :64] = 0.0            # all-zero groups get e8m0 code 0
    p, s = quant.per_1x32_f4_quant(w)
    q, qs = W.mxfp4_to_fp8_blockscale(to_dev(p), to_dev(s))
    got = (q.float().view(E, N // 128, 128, K // 128, 128) * qs[:, :, None, :, None]).view(E, N, K).cpu().numpy()
    ref = quant.dequant_mxfp4(p, s)
    assert np.array_equal(got, ref)


def test_mxfp4_expansion_reports_wide_blocks():
    E, N, K = 1, 128, 128
    p = np.full((E, N, K // 2), 0x22, dtype=np.uint8)       # all values 1.0
    s = np.full((E, N, K // 32), 127, dtype=np.uint8)
    s[0, 0, 0] = 127 + 20                                    # one group 2^20 larger
    with pytest.raises(ValueError, match="not exactly representable"):
        W.mxfp4_to_fp8_blockscale(to_dev(p), to_dev(s))


def _run_a8w4(c):
    w1p, w1s, w2p, w2s = _prep(c)
    out = aiter.fused_moe(to_dev(c["hidden"], torch.bfloat16), w1p.view(torch.float4_e2m1fn_x2),
                          w2p.view(torch.float4_e2m1fn_x2), to_dev(c["topk_weights"]), to_dev(c["topk_ids"]),
                          quant_type=aiter.QuantType.per_1x32, activation=aiter.ActivationType.Silu,
                          w1_scale=w1s.view(torch.float8_e8m0fnu), w2_scale=w2s.view(torch.float8_e8m0fnu))
    torch.cuda.synchronize()
    check_no_device_error()
    return out.float().cpu().numpy()


def test_fused_moe_a8w4_matches_reference_golden(golden):
    g = golden_group(golden, "moe_a8w4")["cfg0"]
    c = inputs.make_moe_case(11, 32, 1024, 512, 8, 2, wfmt="mxfp4")
    assert_moe_close(_run_a8w4(c), g["out"])


@pytest.mark.parametrize("M,D,I,E,k", [(1, 1024, 512, 8, 2), (64, 2048, 512, 16, 8), (200, 1024, 768, 32, 4)])
def test_fused_moe_a8w4_vs_oracle(M, D, I, E, k):
    c = inputs.make_moe_case(M + 3 * E, M, D, I, E, k, wfmt="mxfp4", zipf_s=1.1)
    ref = moe.fused_moe_a8w4(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"], c["topk_weights"],
                             c["topk_ids"])
    assert_moe_close(_run_a8w4(c), ref)


def test_prepared_a8w4_weights_match_per_call_conversion():
    c = inputs.make_moe_case(5, 48, 1024, 512, 8, 2, wfmt="mxfp4")
    w1p, w1s, w2p, w2s = _prep(c)
    w1, s1, w2, s2 = W.prepare_a8w4(w1p, w1s, w2p, w2s)
    o1 = aiter.fused_moe(to_dev(c["hidden"], torch.bfloat16), w1, w2, to_dev(c["topk_weights"]),
                         to_dev(c["topk_ids"]), quant_type=aiter.QuantType.per_1x128, w1_scale=s1, w2_scale=s2)
    o2 = _run_a8w4(c)
    assert np.array_equal(o1.float().cpu().numpy(), o2)
