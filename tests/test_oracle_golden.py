"""Pin the CPU oracle against the reference's own outputs (tests/golden/golden.npz,
produced by tests/golden/make_golden.py from the reference's torch functions)."""
import hashlib

import numpy as np
import pytest

from conftest import golden_group
from oracle import codecs, inputs, moe, quant, routing, sorting
from routing_ulps import MAX_ULPS, ulps


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ------------------------------------------------------------------ codecs


def test_fp8_encode_matches_torch_cast(golden):
    x = golden["codec/fp8_in"]
    ref = golden["codec/fp8_out"]
    got = codecs.fp8_e4m3_encode(x)
    # NaN codes may differ in sign bit only; compare finite
    fin = (ref & 0x7F) != 0x7F
    assert np.array_equal(got[fin], ref[fin])
    assert np.all((got[~fin] & 0x7F) == 0x7F)


def test_mxfp4_decode_all_bytes(golden):
    ref = golden["codec/mxfp4_all"]            # [512]: 256 bytes -> 2 values each
    got = codecs.mxfp4_to_f32(np.arange(256, dtype=np.uint8))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_e8m0_decode_all(golden):
    ref = golden["codec/e8m0_to_f32_all"]
    got = codecs.e8m0_to_f32(np.arange(256, dtype=np.uint8))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_e8m0_encode(golden):
    got = codecs.f32_to_e8m0(golden["codec/e8m0_in"])
    assert np.array_equal(got, golden["codec/e8m0_out"])


def test_e2m1_encode_grid(golden):
    got = codecs.pack_fp4(codecs.e2m1_encode(golden["codec/e2m1_in"]))
    assert np.array_equal(got, golden["codec/e2m1_out"])


# ------------------------------------------------------------------ quantisers


def test_per_1x128_quant(golden):
    q, s = quant.per_1x128_quant(golden["quant1x128/x"])
    assert np.array_equal(s.view(np.uint32), golden["quant1x128/scale"].view(np.uint32))
    assert np.array_equal(q, golden["quant1x128/q"])


def test_per_group_quant_i8(golden):
    """int8 output, the reference per_group_quant_hip's default dtype."""
    q, s = quant.per_group_quant_i8(golden["quant1x128/x"])
    assert np.array_equal(s.view(np.uint32), golden["quant1x128_i8/scale"].view(np.uint32))
    assert np.array_equal(q, golden["quant1x128_i8/q"])


def test_weight_128x128_quant(golden):
    q, s = quant.weight_128x128_quant(golden["quant128x128/w"])
    assert np.array_equal(s.view(np.uint32), golden["quant128x128/scale"].view(np.uint32))
    assert np.array_equal(q, golden["quant128x128/q"])


def test_per_1x32_f4_quant(golden):
    q, s = quant.per_1x32_f4_quant(golden["quant1x32/x"])
    assert np.array_equal(s.reshape(-1), golden["quant1x32/scale"].reshape(-1))
    assert np.array_equal(q.reshape(-1), golden["quant1x32/q"].reshape(-1))


# ------------------------------------------------------------------ sorting


@pytest.mark.parametrize("case", ["kat_doc", "m32_e8_k2_b32", "m1_e128_k8_b128", "m100_e16_k4_b32",
                                  "m300_e128_k8_b64", "m2000_e128_k8_b128", "mask_m64_e16_k4_b32",
                                  "local_m80_e16_k4_b16"])
def test_sorting_matches_reference(golden, case):
    g = golden_group(golden, "sort")[case]
    M, E, k, B, local = [int(v) for v in g["meta"]]
    sid, sw, seid, nv = sorting.moe_sorting(g["topk_ids"], g["topk_weights"], E, B,
                                            g.get("expert_mask"), None if local < 0 else local)
    assert np.array_equal(nv, g["num_valid_ids"])
    n = int(nv[0])
    assert np.array_equal(sid[:n], g["sorted_ids"][:n])
    init = (k << 24) | M
    valid = g["sorted_ids"] != init
    assert np.array_equal(sw[valid].view(np.uint32), g["sorted_weights_valid"].view(np.uint32))
    m = g["sorted_expert_ids"] != -1
    assert np.array_equal(seid[m], g["sorted_expert_ids"][m])


def test_sorting_doc_kat_layout():
    """The worked example of csrc/include/moe_sorting_opus.h:276-298, with ids packed
    as token | slot << 24 and zero-token experts skipped."""
    ids = np.array([[0, 3, 5], [2, 3, 5], [1, 3, 5], [1, 2, 3], [1, 3, 5]], dtype=np.int32)
    w = np.arange(15, dtype=np.float32).reshape(5, 3)
    sid, sw, seid, nv = sorting.moe_sorting(ids, w, 6, 4)
    tok = sid & 0xFFFFFF
    assert list(tok[:24]) == [0, 5, 5, 5, 2, 3, 4, 5, 1, 3, 5, 5, 0, 1, 2, 3, 4, 5, 5, 5, 0, 1, 2, 4]
    assert list(seid[:6]) == [0, 1, 2, 3, 3, 5]
    assert list(nv) == [24, 5]


# ------------------------------------------------------------------ routing


def test_topk_softmax_matches_reference(golden):
    for case, g in golden_group(golden, "topk").items():
        renorm = case.endswith("_r1")
        k = g["ids"].shape[1]
        w, ids, tei = routing.topk_softmax(g["gating"], k, renorm)
        assert np.array_equal(ids, g["ids"]), case
        assert ulps(w, g["weights"]).max() <= MAX_ULPS["topk/" + case], case
        M = g["gating"].shape[0]
        assert tei[1, 0] == 1 and tei[0, 1] == M


def _sorted_by_id(ids, w):
    o = np.argsort(ids, axis=-1)
    return np.take_along_axis(ids, o, -1), np.take_along_axis(w, o, -1)


def test_grouped_topk_matches_reference(golden):
    for case, g in golden_group(golden, "gtopk").items():
        M, E, G, TG, k = [int(v) for v in g["meta"]]
        w, ids = routing.grouped_topk(g["gating"], k, G, TG, True, is_softmax=case.endswith("softmax"))
        i0, w0 = _sorted_by_id(ids, w)
        i1, w1 = _sorted_by_id(g["ids"], g["weights"])
        assert np.array_equal(i0, i1), case
        assert ulps(w0, w1).max() <= MAX_ULPS["gtopk/" + case], case


def test_biased_grouped_topk_matches_reference(golden):
    for case, g in golden_group(golden, "btopk").items():
        M, E, G, TG, k = [int(v) for v in g["meta"]]
        w, ids = routing.biased_grouped_topk(g["gating"], g["bias"], k, G, TG, True)
        i0, w0 = _sorted_by_id(ids, w)
        i1, w1 = _sorted_by_id(g["ids"], g["weights"])
        assert np.array_equal(i0, i1), case
        assert ulps(w0, w1).max() <= MAX_ULPS["btopk/" + case], case


def test_routing_exp_is_correctly_rounded_on_a_dense_sample():
    """rexp against e^x computed in double and rounded once to fp32, over the whole
    range the softmax uses (x - max in [-104, 0]) and the sigmoid's [-30, 30], plus
    the special values."""
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-104, 0, 400_000), rng.uniform(-30, 30, 400_000),
                        np.arange(-1000, 1000) / 64.0]).astype(np.float32)
    assert np.array_equal(routing.rexp(x), np.exp(x.astype(np.float64)).astype(np.float32))
    sp = routing.rexp(np.array([0.0, -np.inf, np.inf, -200.0, 200.0, np.nan], np.float32))
    assert sp[0] == 1.0 and sp[1] == 0.0 and np.isinf(sp[2]) and sp[3] == 0.0 and np.isinf(sp[4])
    assert np.isnan(sp[5])


def test_routing_ksum_is_torch_cpu_sum_order():
    """The renormalising sum's order is torch's CPU sum over a contiguous row of k
    floats, for every k the kernels accept."""
    import torch
    rng = np.random.default_rng(1)
    for k in range(1, 33):
        w = rng.random((4000, k), dtype=np.float32)
        assert np.array_equal(routing.ksum(w), torch.from_numpy(w).sum(dim=-1).numpy()), k


# ------------------------------------------------------------------ MoE pipeline


@pytest.mark.parametrize("tag,shape", [("cfg0", (0, 32, 1024, 512, 8, 2)), ("cfg0_m7", (7, 7, 1024, 256, 8, 2))])
def test_moe_fp8_blockscale_matches_reference(golden, tag, shape):
    g = golden_group(golden, "moe_fp8")[tag]
    seed, M, D, I, E, k = shape
    c = inputs.make_moe_case(seed, M, D, I, E, k)
    assert np.array_equal(c["topk_ids"], g["topk_ids"])
    assert _sha(c["w1_q"]) == bytes(g["w1q_sha"]).decode()
    assert _sha(c["w2_q"]) == bytes(g["w2q_sha"]).decode()
    assert np.array_equal(c["w1_s"].view(np.uint32), g["w1s"].view(np.uint32))
    out, st = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                           c["topk_weights"], c["topk_ids"], return_intermediate=True)
    assert np.array_equal(st["a1_q"], g["a1q"])
    assert np.array_equal(st["a1_s"].view(np.uint32), g["a1s"].view(np.uint32))
    # fp32 GEMM summation order differs between numpy and torch: bf16 results agree
    # to a bf16 ulp or so
    np.testing.assert_allclose(st["out1"], g["out1"], rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(out, g["out"], rtol=2e-2, atol=2e-2)
    assert np.mean(np.abs(out - g["out"]) > 1e-3) < 0.02


def test_moe_a8w4_matches_reference(golden):
    g = golden_group(golden, "moe_a8w4")["cfg0"]
    c = inputs.make_moe_case(11, 32, 1024, 512, 8, 2, wfmt="mxfp4")
    assert _sha(c["w1_q"]) == bytes(g["w1p_sha"]).decode()
    assert np.array_equal(c["w1_s"], g["w1e"])
    out, st = moe.fused_moe_a8w4(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                 c["topk_weights"], c["topk_ids"], return_intermediate=True)
    np.testing.assert_allclose(st["out1"], g["out1"], rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(out, g["out"], rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("case", ["s1_t37_d512_e8_k2_b32", "s2_t37_d512_e8_k2_b32", "s1_t300_d1024_e16_k4_b128",
                                  "s2_t64_d256_e32_k8_b64"])
def test_mxfp4_quant_and_moe_scale_sort_match_reference(golden, case):
    from oracle import mxfp4_sort
    g = golden_group(golden, "mxfp4sort")[case]
    T, D, E, k, B, stage = (int(v) for v in g["meta"])
    q, s = quant.per_1x32_f4_quant(g["x"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(s, g["scale"])
    scale_in = s if stage == 1 else s.reshape(T, k, D // 32)
    srt = mxfp4_sort.moe_mxfp4_sort(scale_in, g["sorted_ids"], int(g["num_valid_ids"][0]), T)
    assert srt.shape == g["sorted_scale"].shape
    assert np.array_equal(srt, g["sorted_scale"])
    # e8m0_shuffle pads with uninitialised memory: compare where the source is real
    sh = mxfp4_sort.e8m0_shuffle(s)
    rows, cols = sh.shape
    r, c = mxfp4_sort.shuffle_index(rows, cols)
    real = ((r < s.shape[0]) & (c < s.shape[1])).reshape(rows, cols)
    assert np.array_equal(sh[real], g["shuffled_scale"][real])


def test_unshuffle_weight_inverts_the_reference_shuffle(golden):
    """aiter_b200.weights.unshuffle_weight undoes the reference's shuffle_weight
    (aiter/ops/shuffle.py:7-27) for 1-byte (fp8) and 2-byte (bf16) weights."""
    import torch
    from aiter_b200.weights import unshuffle_weight
    sh = torch.from_numpy(golden["shuffle/shuffled_fp8"]).view(torch.float8_e4m3fn)
    back = unshuffle_weight(sh).view(torch.uint8).numpy()
    assert np.array_equal(back, golden["shuffle/w_u8"])
    shb = torch.from_numpy(golden["shuffle/shuffled_bf16"]).to(torch.bfloat16)
    backb = unshuffle_weight(shb).float().numpy()
    assert np.array_equal(backb, golden["shuffle/w_bf16"])
    assert not np.array_equal(golden["shuffle/shuffled_fp8"], golden["shuffle/w_u8"])


@pytest.mark.parametrize("tag,opts", [("swiglu", dict(activation="swiglu")),
                                      ("doweight", dict(doweight_stage1=True)),
                                      ("fp16", dict(dtype="fp16")),
                                      ("bias_swiglu", dict(activation="swiglu"))])
def test_moe_fp8_options_match_reference(golden, tag, opts):
    """fused_moe options of the reference pipeline: Swiglu (aiter/fused_moe.py:1473-1480),
    doweight_stage1 (top-k weight on the stage-1 GEMM output, none in stage 2), fp16
    activations / intermediate / output, and the experts' biases of both GEMMs
    (w1_bias / w2_bias of torch_moe_stage1/2, :1572-1573, 1662-1663)."""
    g = golden_group(golden, "moe_fp8_opts")[tag]
    seed = {"swiglu": 21, "doweight": 22, "fp16": 23, "bias_swiglu": 24}[tag]
    c = inputs.make_moe_case(seed, 32, 1024, 512, 8, 2)
    assert np.array_equal(c["topk_ids"], g["topk_ids"])
    if "bias1" in g:
        opts = dict(opts, bias1=g["bias1"], bias2=g["bias2"])
    hidden = c["hidden"]
    if opts.get("dtype") == "fp16":
        hidden = hidden.astype(np.float16).astype(np.float32)
    out, st = moe.fused_moe_fp8_blockscale(hidden, c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                           c["topk_weights"], c["topk_ids"], return_intermediate=True, **opts)
    assert np.array_equal(st["a1_q"], g["a1q"])
    np.testing.assert_allclose(st["out1"], g["out1"], rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(out, g["out"], rtol=2e-2, atol=2e-2)
    assert np.mean(np.abs(out - g["out"]) > 1e-3) < 0.02


@pytest.mark.parametrize("tag", ["e64_k4_bf16", "e128_k8_fp16", "e128_k1_fp32"])
def test_topk_sigmoid_oracle_matches_reference(golden, tag):
    """topk_sigmoid against the reference's torch routing (torch.topk, then sigmoid in
    fp32; op_tests/test_moe_topk_sigmoid.py:30-35)."""
    from oracle.routing import topk_sigmoid
    g = golden_group(golden, "topk_sigmoid")[tag]
    k = g["ids"].shape[1]
    w, ids = topk_sigmoid(g["logits"], k)
    assert np.array_equal(ids, g["ids"])
    assert ulps(w, g["weights"]).max() <= MAX_ULPS["topk_sigmoid/" + tag]


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
def test_silu_and_mul_oracle_matches_reference(golden, tag):
    """silu_and_mul against the reference test's torch_silu_and_mul
    (op_tests/test_activation.py:13-17, checked there with atol = rtol = 1e-2); the
    torch path rounds silu(x) to bf16 before the product, the kernel rounds once."""
    from oracle.activation import act_and_mul
    g = golden_group(golden, "silu_and_mul")[tag]
    got = act_and_mul(g["input"], "silu", tag)
    np.testing.assert_allclose(got, g["out"], rtol=1e-2, atol=1e-2)
    if tag == "fp32":
        np.testing.assert_allclose(got, g["out"], rtol=1e-6, atol=1e-6)


def test_moe_sum_oracle_rounding_rule():
    """moe_sum rounds after every slot for topk 2, 4, 5 (the reference kernel adds in the
    element type) and once otherwise (its at::sum_out fallback)."""
    from oracle.codecs import round_bf16
    from oracle.moe import moe_sum
    x = np.zeros((1, 4, 8), np.float32)
    x[0, :, 0] = [1.0, 2.0 ** -9, 2.0 ** -9, 2.0 ** -9]       # bf16 ulp at 1 is 2^-7
    assert moe_sum(x, "bf16")[0, 0] == 1.0                     # each add rounds back to 1
    x3 = np.concatenate([x, np.zeros((1, 2, 8), np.float32)], axis=1)[:, [0, 1, 2, 3, 4, 5]]
    x3[0, :, 0] = [1.0, 2.0 ** -9, 2.0 ** -9, 2.0 ** -9, 2.0 ** -9, 0.0]
    assert moe_sum(x3, "bf16")[0, 0] == round_bf16(np.float32(1.0 + 4 * 2.0 ** -9))


@pytest.mark.parametrize("tag,shape", [("cfg0", (0, 32, 1024, 512, 8, 2)), ("cfg0_m7", (7, 7, 1024, 256, 8, 2))])
def test_torch_port_of_reference_cpu_path_matches_reference(golden, tag, shape):
    """The timed CPU baseline (oracle/moe_torch.py, torch CPU ops in the reference's
    order) reproduces the reference pipeline's bf16 output bit for bit."""
    import torch
    from oracle import moe_torch
    g = golden_group(golden, "moe_fp8")[tag]
    seed, M, D, I, E, k = shape
    c = inputs.make_moe_case(seed, M, D, I, E, k)
    fp8 = lambda a: torch.from_numpy(a).view(torch.float8_e4m3fn)
    out = moe_torch.fused_moe_fp8_blockscale(
        torch.from_numpy(c["hidden"]).to(torch.bfloat16), fp8(c["w1_q"]), torch.from_numpy(c["w1_s"]),
        fp8(c["w2_q"]), torch.from_numpy(c["w2_s"]), torch.from_numpy(g["topk_weights"]),
        torch.from_numpy(g["topk_ids"]))
    assert np.array_equal(out.float().numpy(), g["out"])


def test_fp8_requant_fast_path_equals_division():
    """The stage-1 epilogue quantises x / scale through q = x * RN(1/scale) and takes the
    IEEE division only when q * (1 -/+ 2^-20) straddle an fp8 rounding boundary.  Restated
    here in fp32 numpy: wherever the two bracket codes agree they equal the codes of
    RN(x / scale), on random groups and on quotients placed exactly on fp8 midpoints."""
    rng = np.random.default_rng(3)
    f = np.float32
    enc = lambda v: codecs.fp8_e4m3_encode(np.clip(v, -448.0, 448.0).astype(f))
    for trial in range(4):
        x = (rng.standard_normal((4000, 128)) * rng.uniform(0.01, 50)).astype(f)
        amax = np.abs(x).max(axis=1, keepdims=True)
        s = (amax / f(448.0)).astype(f)
        if trial == 3:   # quotients on exact fp8 midpoints (ties) and their neighbours
            mids = ((codecs.FP8_E4M3_VALUES[1:126] + codecs.FP8_E4M3_VALUES[2:127]) / 2).astype(f)
            x[:, :64] = (rng.choice(mids, (4000, 64)) * s).astype(f)
        rs = (f(1.0) / s).astype(f)
        q = (x * rs).astype(f)
        cl = enc((q * f(1.0 - 2.0 ** -20)).astype(f))
        ch = enc((q * f(1.0 + 2.0 ** -20)).astype(f))
        exact = enc((x / s).astype(f))
        fast = cl == ch
        assert np.array_equal(cl[fast], exact[fast])
        assert fast.mean() > (0.4 if trial == 3 else 0.999)
