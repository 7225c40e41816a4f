"""fused_moe options of the reference's FP8 block-scale path on the tcgen05 kernels:
Swiglu (aiter/fused_moe.py:1473-1480), doweight_stage1 (top-k weight on the stage-1
GEMM output, none in stage 2), fp16 activations / output and the experts' biases
(w1_bias / w2_bias), each against the reference's own torch pipeline (golden vectors,
config-0 shape) and against the oracle at a larger shape; fused_moe passes the biases
only on the per_1x32 Swiglu path, as the reference's dispatch does."""
import os

import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from conftest import golden_group
from gpu_util import check_no_device_error, fp8_from_codes, requires_cuda, to_dev
from oracle import inputs, moe

pytestmark = [pytest.mark.gpu, requires_cuda]

OPTS = {"swiglu": (21, dict(activation="swiglu")), "doweight": (22, dict(doweight_stage1=True)),
        "fp16": (23, dict(dtype="fp16"))}


def _run(c, activation="silu", doweight_stage1=False, dtype="bf16"):
    tdt = torch.float16 if dtype == "fp16" else torch.bfloat16
    act = {"silu": aiter.ActivationType.Silu, "swiglu": aiter.ActivationType.Swiglu}[activation]
    out = aiter.fused_moe(to_dev(c["hidden"], tdt), fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"]),
                          to_dev(c["topk_weights"]), to_dev(c["topk_ids"]), quant_type=aiter.QuantType.per_1x128,
                          activation=act, doweight_stage1=doweight_stage1, w1_scale=to_dev(c["w1_s"]),
                          w2_scale=to_dev(c["w2_s"]))
    torch.cuda.synchronize()
    check_no_device_error()
    assert out.dtype == tdt
    return out.float().cpu().numpy()


def _close(out, ref):
    np.testing.assert_allclose(out, ref, rtol=2e-2, atol=2e-2)
    assert (np.abs(out - ref) > 1e-2 + 1e-2 * np.abs(ref)).mean() <= 0.01


@pytest.mark.parametrize("tag", list(OPTS))
def test_option_matches_reference_golden(golden, tag):
    seed, opts = OPTS[tag]
    g = golden_group(golden, "moe_fp8_opts")[tag]
    c = inputs.make_moe_case(seed, 32, 1024, 512, 8, 2)
    _close(_run(c, **opts), g["out"])


@pytest.mark.parametrize("tag", list(OPTS))
def test_option_vs_oracle(tag):
    _, opts = OPTS[tag]
    c = inputs.make_moe_case(90, 200, 2048, 768, 32, 8)
    hidden = c["hidden"].astype(np.float16).astype(np.float32) if opts.get("dtype") == "fp16" else c["hidden"]
    ref = moe.fused_moe_fp8_blockscale(hidden, c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"], c["topk_weights"],
                                       c["topk_ids"], **opts)
    _close(_run(c, **opts), ref)


def _stage_pipeline(c, bias1, bias2, activation=aiter.ActivationType.Swiglu):
    """The two stage entries with the experts' biases (per_1x128 weights): sorting ->
    gather-quant -> stage 1 (+ bias1) -> stage 2 (+ bias2)."""
    from aiter_b200 import moe_op
    from aiter_b200.fused_moe import _moe_sorting_ext
    hidden = to_dev(c["hidden"], torch.bfloat16)
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])
    w1, w2 = fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"])
    w1s, w2s = to_dev(c["w1_s"]), to_dev(c["w2_s"])
    M, k = tid.shape
    E, I, D = w1.shape[0], w2.shape[2], w2.shape[1]
    sids, sw, seids, nv, buf, pos = _moe_sorting_ext(tid, tw, E, D, torch.bfloat16, 128, None, None, 0,
                                                     with_pos=True)
    rows = sids.numel()
    a1, a1s = moe_op.moe_gather_quant_1x128(hidden, pos, k, rows)
    a2 = torch.empty((rows, I), dtype=torch.float8_e4m3fn, device=hidden.device)
    a2s = torch.empty((I // 128, rows), dtype=torch.float32, device=hidden.device)
    moe_op.moe_stage1_fp8_blockscale(a1, a1s, w1, w1s, sids, seids, nv, a2, a2s, M, 128, activation,
                                     bias=to_dev(bias1))
    moe_op.moe_stage2_fp8_blockscale(a2, a2s, w2, w2s, sids, seids, nv, sw, buf, 128, bias=to_dev(bias2))
    torch.cuda.synchronize()
    check_no_device_error()
    return buf.float().cpu().numpy()


def test_bias_stages_match_reference_golden(golden):
    """The bias entries against the reference's torch_moe_stage1/2 with w1_bias / w2_bias."""
    g = golden_group(golden, "moe_fp8_opts")["bias_swiglu"]
    c = inputs.make_moe_case(24, 32, 1024, 512, 8, 2)
    _close(_stage_pipeline(c, g["bias1"], g["bias2"]), g["out"])


def test_bias_stages_vs_oracle():
    c = inputs.make_moe_case(91, 200, 2048, 768, 32, 8)
    rng = np.random.default_rng(5)
    b1 = np.clip(rng.standard_normal((32, 2 * 768)), -1, 1).astype(np.float32)
    b2 = np.clip(rng.standard_normal((32, 2048)), -1, 1).astype(np.float32)
    ref = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"], c["topk_weights"],
                                       c["topk_ids"], activation="swiglu", bias1=b1, bias2=b2)
    _close(_stage_pipeline(c, b1, b2), ref)


def test_fused_moe_bias_only_on_the_per_1x32_swiglu_path():
    """As the reference's dispatch (aiter/fused_moe.py:985-1008, 1228-1238): the biases
    reach the kernels for per_1x32 + Swiglu and are ignored otherwise."""
    M, D, I, E, k = 64, 1024, 512, 8, 2
    c = inputs.make_moe_case(31, M, D, I, E, k, wfmt="mxfp4")
    rng = np.random.default_rng(6)
    b1 = np.clip(rng.standard_normal((E, 2 * I)), -1, 1).astype(np.float32)
    b2 = np.clip(rng.standard_normal((E, D)), -1, 1).astype(np.float32)
    w1 = to_dev(c["w1_q"]).view(torch.float4_e2m1fn_x2)
    w2 = to_dev(c["w2_q"]).view(torch.float4_e2m1fn_x2)
    w1e = to_dev(c["w1_s"]).view(torch.float8_e8m0fnu)
    w2e = to_dev(c["w2_s"]).view(torch.float8_e8m0fnu)
    hidden = to_dev(c["hidden"], torch.bfloat16)
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])
    kw = dict(quant_type=aiter.QuantType.per_1x32, w1_scale=w1e, w2_scale=w2e)
    out = aiter.fused_moe(hidden, w1, w2, tw, tid, activation=aiter.ActivationType.Swiglu,
                          bias1=to_dev(b1), bias2=to_dev(b2), **kw).float().cpu().numpy()
    ref = moe.fused_moe_a8w4(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"], c["topk_weights"],
                             c["topk_ids"], activation="swiglu", bias1=b1, bias2=b2)
    _close(out, ref)
    silu_b = aiter.fused_moe(hidden, w1, w2, tw, tid, activation=aiter.ActivationType.Silu,
                             bias1=to_dev(b1), bias2=to_dev(b2), **kw)
    silu = aiter.fused_moe(hidden, w1, w2, tw, tid, activation=aiter.ActivationType.Silu, **kw)
    torch.cuda.synchronize()
    check_no_device_error()
    assert torch.allclose(silu_b.float(), silu.float(), rtol=1e-2, atol=1e-2)
