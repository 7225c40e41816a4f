"""GPU parity of topk_sigmoid, moe_sum and the gated activations (moe_misc.cu)
against the reference's torch functions (golden vectors) and the oracle.

* topk_sigmoid: ids bit-exact, weights within 1e-6 (fp32 sigmoid), every experts /
  topk / dtype of the reference's test grid (op_tests/test_moe_topk_sigmoid.py:113-116);
* moe_sum: bit-exact against the oracle for topk 1..8 (stepwise rounding for 2, 4, 5),
  fp32 / bf16 / fp16, vector and scalar paths;
* silu / gelu / gelu_tanh_and_mul: within one unit in the last place of bf16 / fp16
  outputs (16 of fp32 outputs: the fp32 transcendentals differ in their last bits) of
  the oracle, every input /
  output dtype pair the reference accepts; scaled_silu_and_mul: fp8 codes within one
  step; unsupported dtype pairs raise.
"""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from conftest import golden_group
from gpu_util import requires_cuda
from oracle import activation as oact
from oracle.moe import moe_sum as moe_sum_ref
from oracle.routing import topk_sigmoid as topk_sigmoid_ref

pytestmark = [pytest.mark.gpu, requires_cuda]

DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _unique_logits(M, E, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    base = torch.arange(-1, 1, 2.0 / E).repeat((M, 1)).to(dtype)
    return torch.gather(base, -1, torch.argsort(torch.rand(base.shape, generator=g), dim=-1))


@pytest.mark.parametrize("tag", ["e64_k4_bf16", "e128_k8_fp16", "e128_k1_fp32"])
def test_topk_sigmoid_golden(golden, tag):
    g = golden_group(golden, "topk_sigmoid")[tag]
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[tag.split("_")[-1]]
    logits = torch.from_numpy(g["logits"]).to(dt).cuda()
    M, k = g["ids"].shape
    w = torch.empty(M, k, device="cuda")
    ids = torch.empty(M, k, dtype=torch.int32, device="cuda")
    aiter.topk_sigmoid(w, ids, logits)
    assert np.array_equal(ids.cpu().numpy(), g["ids"])
    np.testing.assert_allclose(w.cpu().numpy(), g["weights"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("E", [64, 128, 256, 1000])
@pytest.mark.parametrize("k", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_topk_sigmoid_vs_oracle(E, k, dtype):
    logits = _unique_logits(300, E, dtype, E + k)
    w = torch.empty(300, k, device="cuda")
    ids = torch.empty(300, k, dtype=torch.int32, device="cuda")
    aiter.topk_sigmoid(w, ids, logits.cuda())
    rw, rid = topk_sigmoid_ref(logits.float().numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("dt", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("D", [4096, 100])
def test_moe_sum_vs_oracle(k, dt, D):
    g = torch.Generator().manual_seed(k * 7 + D)
    x = (torch.randn(37, k, D, generator=g) * 3).to(DT[dt])
    out = torch.empty(37, D, dtype=DT[dt], device="cuda")
    aiter.moe_sum(x.cuda(), out)
    assert np.array_equal(out.float().cpu().numpy(), moe_sum_ref(x.float().numpy(), dt))


def _ulp_close(got, want, dtype):
    """One unit in the last place of bf16 / fp16 outputs, 16 of fp32 outputs (the device's
    fp32 exp / erf / tanh carry a few ulps), plus 1e-5 absolute: 1 + erf(x) cancels for
    very negative x, where the values themselves are below 1e-5."""
    eps = {"fp32": 16 * 2.0 ** -23, "bf16": 2.0 ** -7, "fp16": 2.0 ** -10}[dtype]
    assert np.all(np.abs(got - want) <= eps * np.abs(want) + 1e-5)


@pytest.mark.parametrize("kind,fn", [("silu", "silu_and_mul"), ("gelu", "gelu_and_mul"),
                                     ("gelu_tanh", "gelu_tanh_and_mul")])
@pytest.mark.parametrize("din,dout", [("fp32", "fp32"), ("fp32", "bf16"), ("fp32", "fp16"), ("bf16", "bf16"),
                                      ("fp16", "fp16")])
@pytest.mark.parametrize("N", [8192, 200])
def test_act_and_mul_vs_oracle(kind, fn, din, dout, N):
    g = torch.Generator().manual_seed(N)
    inp = (torch.randn(33, N, generator=g) * 2).to(DT[din])
    out = torch.empty(33, N // 2, dtype=DT[dout], device="cuda")
    getattr(aiter, fn)(out, inp.cuda())
    want = oact.act_and_mul(inp.float().numpy(), kind, dout)
    _ulp_close(out.float().cpu().numpy(), want, dout)


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
def test_silu_and_mul_golden(golden, tag):
    g = golden_group(golden, "silu_and_mul")[tag]
    inp = torch.from_numpy(g["input"]).to(DT[tag]).cuda()
    out = torch.empty(inp.shape[0], inp.shape[1] // 2, dtype=DT[tag], device="cuda")
    aiter.silu_and_mul(out, inp)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["out"], rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("din", ["fp32", "bf16", "fp16"])
def test_scaled_silu_and_mul_vs_oracle(din):
    g = torch.Generator().manual_seed(5)
    inp = torch.randn(17, 1024, generator=g).to(DT[din])
    scale = inp.float().max().reshape(1)
    out = torch.empty(17, 512, dtype=torch.float8_e4m3fn, device="cuda")
    aiter.scaled_silu_and_mul(out, inp.cuda(), scale.cuda())
    got = out.view(torch.uint8).cpu().numpy().astype(np.int32)
    want = oact.scaled_silu_and_mul(inp.float().numpy(), scale.item()).astype(np.int32)
    # one fp8 step at most (the fp32 silu may differ in its last bits near a rounding tie)
    same_sign = (got & 0x80) == (want & 0x80)
    assert np.all(same_sign | (np.minimum(got & 0x7F, want & 0x7F) == 0))
    assert np.all(np.abs((got & 0x7F) - (want & 0x7F)) <= 1)


def test_act_and_mul_rejects_mismatched_dtypes():
    inp = torch.randn(4, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="must match"):
        aiter.silu_and_mul(torch.empty(4, 32, dtype=torch.float16, device="cuda"), inp)
    with pytest.raises(RuntimeError, match="fp8"):
        aiter.scaled_silu_and_mul(torch.empty(4, 32, dtype=torch.bfloat16, device="cuda"), inp,
                                  torch.ones(1, device="cuda"))
