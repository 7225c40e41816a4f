"""A8W4 (fp8 1x128 activations x MXFP4 weights, the BASELINE config-2 contract).

fused_moe(quant_type=per_1x32) runs the native grouped GEMMs (moe_stage1/2_a8w4:
weights read at 4 bits, e8m0 scales applied by the block-scaled MMA):
* against the reference-composed golden output (tests/golden, moe_a8w4/cfg0) and
  against the oracle on sweeps, rtol = atol = 2e-2 (assert_moe_close);
* config 2 at full size (D=4096, I=2048, E=256, top-8, Zipf routing), M = 64 and
  2048, on a sample of tokens against a plain fp32 torch reference (1x128 quant with
  IEEE division as the reference's pertoken_quant, MXFP4 decode, per-expert GEMMs):
  the stage-1 fp8 codes and the outputs;
* the scale chunks (mxfp4_moe_weight_scale_chunks) against a numpy restatement of
  their layout; scales passed as chunks give the same bits as scales rearranged per
  call; two stage-1 runs give the same bits;
* the FP8 expansion of the weights (mxfp4_to_fp8_blockscale): its e4m3 x power-of-two
  block values equal the MXFP4 dequantisation (mxfp4_to_f32 * e8m0_to_f32,
  aiter/utility/fp4_utils.py:19-69) bit for bit, blocks that cannot be exact are
  reported, and the FP8 kernels on expanded weights agree with the native path."""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from aiter_b200 import weights as W
from conftest import golden_group
from gpu_util import check_no_device_error, dev, requires_cuda, to_dev
from oracle import codecs, inputs, moe, quant
from aiter_b200.fused_moe import _moe_sorting_ext
from test_gpu_moe import assert_moe_close, torch_quant_1x128

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


def test_expanded_fp8_weights_agree_with_native_path():
    c = inputs.make_moe_case(5, 48, 1024, 512, 8, 2, wfmt="mxfp4")
    w1p, w1s, w2p, w2s = _prep(c)
    w1, s1, w2, s2 = W.prepare_a8w4(w1p, w1s, w2p, w2s)
    o1 = aiter.fused_moe(to_dev(c["hidden"], torch.bfloat16), w1, w2, to_dev(c["topk_weights"]),
                         to_dev(c["topk_ids"]), quant_type=aiter.QuantType.per_1x128, w1_scale=s1, w2_scale=s2)
    assert_moe_close(o1.float().cpu().numpy(), _run_a8w4(c))


def _chunks_numpy(s):
    E, N, G = s.shape
    K = G * 32
    out = np.zeros((E, N // 128, K // 128, 512), dtype=np.uint8)
    for r in range(32):
        for w in range(4):
            for b in range(4):
                out[:, :, :, r * 16 + w * 4 + b] = s[:, 32 * w + r::128, b::4]
    return out


def test_scale_chunk_layout():
    rng = np.random.default_rng(3)
    s = rng.integers(100, 140, size=(3, 256, 384 // 32), dtype=np.uint8)
    got = W.mxfp4_moe_weight_scale_chunks(to_dev(s)).cpu().numpy()
    assert np.array_equal(got, _chunks_numpy(s))


def test_prepared_scale_chunks_match_per_call_rearrangement():
    c = inputs.make_moe_case(5, 48, 1024, 512, 8, 2, wfmt="mxfp4")
    w1p, w1s, w2p, w2s = _prep(c)
    _, k1, _, k2 = W.prepare_a8w4_native(w1p, w1s, w2p, w2s)
    o1 = aiter.fused_moe(to_dev(c["hidden"], torch.bfloat16), w1p.view(torch.float4_e2m1fn_x2),
                         w2p.view(torch.float4_e2m1fn_x2), to_dev(c["topk_weights"]), to_dev(c["topk_ids"]),
                         quant_type=aiter.QuantType.per_1x32, w1_scale=k1, w2_scale=k2)
    torch.cuda.synchronize()
    check_no_device_error()
    assert np.array_equal(o1.float().cpu().numpy(), _run_a8w4(c))


def test_a8w4_stage1_repeats_bit_identically():
    """Two runs of the native stage-1 kernel give the same intermediate bits (stage 1
    has no atomics)."""
    from aiter_b200 import moe_op
    c = inputs.make_moe_case(8, 200, 2048, 768, 16, 4, wfmt="mxfp4")
    w1p, w1s, w2p, w2s = _prep(c)
    _, k1, _, _ = W.prepare_a8w4_native(w1p, w1s, w2p, w2s)
    tid, tw = to_dev(c["topk_ids"]), to_dev(c["topk_weights"])
    sids, sw, seids, nv, buf, pos = _moe_sorting_ext(tid, tw, 16, 2048, torch.bfloat16, 128, with_pos=True)
    a1, a1s = moe_op.moe_gather_quant_1x128(to_dev(c["hidden"], torch.bfloat16), pos, 4, sids.numel())
    outs = []
    for _ in range(2):
        a2 = torch.zeros((sids.numel(), 768), dtype=torch.float8_e4m3fn, device=dev())
        a2s = torch.zeros((768 // 128, sids.numel()), dtype=torch.float32, device=dev())
        moe_op.moe_stage1_a8w4(a1, a1s, w1p, k1, sids, seids, nv, a2, a2s, 200, 128)
        torch.cuda.synchronize()
        check_no_device_error()
        outs.append((a2.view(torch.uint8).cpu(), a2s.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


# --------------------------------------------------------------------- config 2, full size

def _torch_a8w4_tokens(hidden, w1p, w1s, w2p, w2s, tw, tid, tokens):
    """fp32 torch reference for a subset of tokens: the output rows and, per (token,
    slot), the fp8 codes of the requantised intermediate."""
    a1, _ = torch_quant_1x128(hidden[tokens])
    I = w2p.shape[2] * 2
    outs, codes = [], {}
    for i, t in enumerate(tokens.tolist()):
        acc = torch.zeros(hidden.shape[1], device=hidden.device)
        for j in range(tid.shape[1]):
            e = int(tid[t, j])
            h = W.dequant_mxfp4(w1p[e], w1s[e]) @ a1[i]
            y = (torch.nn.functional.silu(h[:I]) * h[I:]).to(torch.bfloat16)
            a2, q = torch_quant_1x128(y[None])
            codes[(t, j)] = q[0]
            acc += tw[t, j] * (W.dequant_mxfp4(w2p[e], w2s[e]) @ a2[0])
        outs.append(acc.to(torch.bfloat16).float())
    return torch.stack(outs), codes


@pytest.fixture(scope="module")
def config2_weights():
    D, I, E = 4096, 2048, 256
    g = torch.Generator(device=dev()).manual_seed(2024)
    parts = {"w1": [], "w1s": [], "w2": [], "w2s": []}
    for e0 in range(0, E, 16):
        p, s = W.quant_weight_mxfp4(torch.randn(16, 2 * I, D, device=dev(), generator=g) / D ** 0.5)
        parts["w1"].append(p)
        parts["w1s"].append(s)
        p, s = W.quant_weight_mxfp4(torch.randn(16, D, I, device=dev(), generator=g) / I ** 0.5)
        parts["w2"].append(p)
        parts["w2s"].append(s)
    return {k: torch.cat(v) for k, v in parts.items()}


@pytest.mark.parametrize("M", [64, 2048])
def test_fused_moe_a8w4_full_size_config2(M, config2_weights):
    """Config 2 at full size on 64 sampled tokens.  The intermediate is rounded to bf16
    and requantised to fp8, so a last-bit difference of the fp32 GEMM sum (another
    summation order than the reference's) moves an fp8 code by one step when the value
    sits on a rounding boundary.  Checked: the stage-1 fp8 codes of the sampled (token,
    slot) pairs equal the reference's except <= 0.05 % of them, each one code step
    apart; the outputs within rtol = atol = 2e-2 (assert_moe_close)."""
    from aiter_b200 import moe_op
    D, I, E, k = 4096, 2048, 256, 8
    cw = config2_weights
    rng = np.random.default_rng(M)
    logits = torch.from_numpy(inputs.make_logits(rng, M, E, zipf_s=1.1)).to(dev())
    tw, tid = torch.topk(torch.softmax(logits, dim=-1), k, dim=-1)
    tw = tw / tw.sum(dim=-1, keepdim=True)
    tid = tid.to(torch.int32)
    hidden = torch.from_numpy(rng.standard_normal((M, D), dtype=np.float32)).to(dev()).to(torch.bfloat16)
    out = aiter.fused_moe(hidden, cw["w1"].view(torch.float4_e2m1fn_x2), cw["w2"].view(torch.float4_e2m1fn_x2),
                          tw, tid, quant_type=aiter.QuantType.per_1x32, activation=aiter.ActivationType.Silu,
                          w1_scale=cw["w1s"].view(torch.float8_e8m0fnu), w2_scale=cw["w2s"].view(torch.float8_e8m0fnu))
    torch.cuda.synchronize()
    check_no_device_error()
    tokens = torch.randperm(M, device=dev())[:64]
    ref, ref_codes = _torch_a8w4_tokens(hidden, cw["w1"], cw["w1s"], cw["w2"], cw["w2s"], tw, tid, tokens)
    # stage 1 alone: the intermediate fp8 codes of the sampled (token, slot) pairs
    sids, sw, seids, nv, buf, pos = _moe_sorting_ext(tid, tw, E, D, torch.bfloat16, 128, with_pos=True)
    rows = sids.numel()
    a1, a1s = moe_op.moe_gather_quant_1x128(hidden, pos, k, rows)
    a2 = torch.empty((rows, I), dtype=torch.float8_e4m3fn, device=dev())
    a2s = torch.empty((I // 128, rows), dtype=torch.float32, device=dev())
    moe_op.moe_stage1_a8w4(a1, a1s, cw["w1"], W.mxfp4_moe_weight_scale_chunks(cw["w1s"]), sids, seids, nv,
                           a2, a2s, M, 128)
    torch.cuda.synchronize()
    check_no_device_error()
    sid = sids.cpu().numpy()[:int(nv[0])]
    where = {(int(t), int(j)): r for r, (t, j) in enumerate(zip(sid & 0xFFFFFF, sid >> 24)) if t < M}
    diff = total = 0
    for (t, j), q in ref_codes.items():
        got, want = a2[where[(t, j)]].float(), q.float()
        neq = got != want
        if neq.any():
            # one code step: no e4m3 value lies strictly between got and want
            lo, hi = torch.minimum(got, want)[neq], torch.maximum(got, want)[neq]
            step = (hi - lo) <= torch.maximum(lo.abs(), hi.abs()) * 0.125 + 2.0 ** -9
            assert bool(step.all()), (t, j, int(neq.sum()), got[neq][:8].tolist(), want[neq][:8].tolist())
        diff += int(neq.sum())
        total += neq.numel()
    assert diff <= 5e-4 * total, f"{diff} of {total} intermediate codes differ"
    assert_moe_close(out[tokens].float().cpu().numpy(), ref.cpu().numpy())
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("opt", ["gelu", "swiglu", "doweight", "fp16"])
def test_native_a8w4_options_match_expanded_fp8(opt):
    """Every fused_moe option on the native A8W4 kernels against the FP8 kernels run on
    the exactly expanded weights (whose options are checked against the reference's
    pipeline and the oracle in test_gpu_moe_options.py), rtol = atol = 2e-2."""
    c = inputs.make_moe_case(60, 160, 2048, 768, 16, 4, wfmt="mxfp4", zipf_s=1.1)
    w1p, w1s, w2p, w2s = _prep(c)
    w1, s1, w2, s2 = W.prepare_a8w4(w1p, w1s, w2p, w2s)
    tdt = torch.float16 if opt == "fp16" else torch.bfloat16
    act = {"gelu": aiter.ActivationType.Gelu, "swiglu": aiter.ActivationType.Swiglu}.get(opt,
                                                                                        aiter.ActivationType.Silu)
    kw = dict(activation=act, doweight_stage1=opt == "doweight")
    hidden = to_dev(c["hidden"], tdt)
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])
    native = aiter.fused_moe(hidden, w1p.view(torch.float4_e2m1fn_x2), w2p.view(torch.float4_e2m1fn_x2), tw, tid,
                             quant_type=aiter.QuantType.per_1x32, w1_scale=w1s.view(torch.float8_e8m0fnu),
                             w2_scale=w2s.view(torch.float8_e8m0fnu), **kw)
    expanded = aiter.fused_moe(hidden, w1, w2, tw, tid, quant_type=aiter.QuantType.per_1x128, w1_scale=s1,
                               w2_scale=s2, **kw)
    torch.cuda.synchronize()
    check_no_device_error()
    assert native.dtype == tdt and expanded.dtype == tdt
    assert_moe_close(native.float().cpu().numpy(), expanded.float().cpu().numpy())
