"""fused_moe options of the reference's FP8 block-scale path on the tcgen05 kernels:
Swiglu (aiter/fused_moe.py:1473-1480), doweight_stage1 (top-k weight on the stage-1
GEMM output, none in stage 2) and fp16 activations / output, each against the
reference's own torch pipeline (golden vectors, config-0 shape) and against the oracle
at a larger shape.  Runs only with AITER_B200_TEST_UNRUN=1 until these variants have
been run on a B200."""
import os

import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from conftest import golden_group
from gpu_util import check_no_device_error, fp8_from_codes, requires_cuda, to_dev
from oracle import inputs, moe

pytestmark = [pytest.mark.gpu, requires_cuda,
              pytest.mark.skipif(os.environ.get("AITER_B200_TEST_UNRUN") != "1",
                                 reason="Swiglu / doweight_stage1 / fp16 variants not yet run on a B200")]

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
