"""Generate golden fixtures by running the reference's own torch functions.

Usage (in a container that has the reference checkout):
    python tests/golden/make_golden.py /path/to/reference

Inputs are drawn with `oracle.inputs` / numpy seeded generators so the tests can
regenerate them bit-for-bit anywhere; the fixtures store the reference's outputs
(and the small inputs that are not regenerated).  Functions used, with their
reference locations:

* moe_sorting_native       op_tests/test_moe_sorting.py:15-70
* test_nofuse              op_tests/test_moeTopkSoftmax.py:21-41
* grouped_topk_torch       aiter/ops/topk.py:161-197
* biased_grouped_topk_torch aiter/ops/topk.py:116-158
* pertoken_quant           aiter/ops/quant.py:42-72
* per_1x32_f4_quant        aiter/ops/quant.py:75-106
* f32_to_e8m0 / e8m0_to_f32 / mxfp4_to_f32  aiter/utility/fp4_utils.py:19-69
* weight_per_128x128_quant op_tests/test_moe_2stage.py:84-110
* torch_moe_stage1/2       aiter/fused_moe.py:1483-1666
* e8m0_shuffle             aiter/utility/fp4_utils.py:72-92
* shuffle_weight           aiter/ops/shuffle.py:7-27
* run_torch (sorted MXFP4 scale layout)  op_tests/test_moe_sorting_mxfp4.py:20-43
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from ref_loader import Reference, QuantType, ActivationType  # noqa: E402
from oracle import inputs, mxfp4_sort  # noqa: E402


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def t2n(t):
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.float4_e2m1fn_x2):
        return t.view(torch.uint8).numpy().copy()
    if t.dtype == torch.bfloat16:
        return t.float().numpy().copy()
    return t.numpy().copy()


SORT_CASES = [
    # name, M, E, topk, block, mask, local
    ("kat_doc", 5, 6, 3, 4, None, None),
    ("m32_e8_k2_b32", 32, 8, 2, 32, None, None),
    ("m1_e128_k8_b128", 1, 128, 8, 128, None, None),
    ("m100_e16_k4_b32", 100, 16, 4, 32, None, None),
    ("m300_e128_k8_b64", 300, 128, 8, 64, None, None),
    ("m2000_e128_k8_b128", 2000, 128, 8, 128, None, None),
    ("mask_m64_e16_k4_b32", 64, 16, 4, 32, "mask", None),
    ("local_m80_e16_k4_b16", 80, 16, 4, 16, None, 50),
    # config 1 at full size, and config-2 routing (Zipf(1.1)-skewed experts)
    ("m4096_e128_k8_b128", 4096, 128, 8, 128, None, None),
    ("zipf_m2048_e256_k8_b128", 2048, 256, 8, 128, None, None),
]

TOPK_CASES = [
    ("m64_e8_k2", 64, 8, 2), ("m64_e128_k8", 64, 128, 8), ("m33_e256_k8", 33, 256, 8),
    ("m17_e64_k6", 17, 64, 6), ("m9_e512_k8", 9, 512, 8),
    ("zipf_m64_e256_k8", 64, 256, 8),
]


MXFP4_SORT_CASES = [
    # name, tokens, model_dim, E, topk, block, stage (1: scales per token, 2: per token and slot)
    ("s1_t37_d512_e8_k2_b32", 37, 512, 8, 2, 32, 1),
    ("s2_t37_d512_e8_k2_b32", 37, 512, 8, 2, 32, 2),
    ("s1_t300_d1024_e16_k4_b128", 300, 1024, 16, 4, 128, 1),
    ("s2_t64_d256_e32_k8_b64", 64, 256, 32, 8, 64, 2),
]


def main(root):
    ref = Reference(root)
    out = {}
    # ---------------------------------------------------------------- sorting
    for i, (name, M, E, k, B, mask, local) in enumerate(SORT_CASES):
        rng = np.random.default_rng(1000 + i)
        if name == "kat_doc":
            ids = np.array([[0, 3, 5], [2, 3, 5], [1, 3, 5], [1, 2, 3], [1, 3, 5]], dtype=np.int32)
        elif name.startswith("zipf"):
            # the k largest of N(0,1) + log p_e logits, p Zipf(1.1) over a random expert order
            lg = inputs.make_logits(rng, M, E, zipf_s=1.1)
            ids = np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)
        else:
            ids = np.stack([rng.permutation(E)[:k] for _ in range(M)]).astype(np.int32)
        w = rng.random((M, k), dtype=np.float32)
        em = None
        if mask:
            em = rng.integers(0, 2, E).astype(np.int32)
        nlt = None if local is None else torch.tensor([local], dtype=torch.int32)
        r = ref.moe_sorting_native(torch.from_numpy(ids), torch.from_numpy(w), E, B,
                                   None if em is None else torch.from_numpy(em), nlt)
        sid, sw, seid, nv = r
        p = f"sort/{name}/"
        out[p + "topk_ids"] = ids
        out[p + "topk_weights"] = w
        out[p + "meta"] = np.array([M, E, k, B, -1 if local is None else local], dtype=np.int64)
        if em is not None:
            out[p + "expert_mask"] = em
        out[p + "sorted_ids"] = t2n(sid)
        # pad weights are torch.empty in the native function: keep only valid slots
        init = (k << 24) | M
        valid = t2n(sid) != init
        out[p + "sorted_weights_valid"] = t2n(sw)[valid]
        out[p + "sorted_expert_ids"] = t2n(seid)
        out[p + "num_valid_ids"] = t2n(nv)
    # ---------------------------------------------------------------- topk softmax
    for i, (name, M, E, k) in enumerate(TOPK_CASES):
        rng = np.random.default_rng(2000 + i)
        g = inputs.make_logits(rng, M, E, zipf_s=1.1) if name.startswith("zipf") else \
            rng.standard_normal((M, E), dtype=np.float32)
        for renorm in (True, False):
            w, ids = ref.test_nofuse(torch.from_numpy(g), k, renorm)
            p = f"topk/{name}_r{int(renorm)}/"
            out[p + "gating"] = g
            out[p + "weights"] = t2n(w)
            out[p + "ids"] = t2n(ids)
    # ---------------------------------------------------------------- grouped top-k
    for i, (M, E, G, TG, k) in enumerate([(32, 256, 8, 4, 8), (16, 64, 4, 2, 6)]):
        rng = np.random.default_rng(3000 + i)
        g = rng.standard_normal((M, E), dtype=np.float32)
        bias = (0.1 * rng.standard_normal(E)).astype(np.float32)
        for func in ("softmax", "sigmoid"):
            w, ids = ref.grouped_topk_torch(torch.from_numpy(g), k, True, G, TG, func)
            p = f"gtopk/m{M}_e{E}_{func}/"
            out[p + "gating"] = g
            out[p + "meta"] = np.array([M, E, G, TG, k])
            out[p + "weights"] = t2n(w)
            out[p + "ids"] = t2n(ids)
        w, ids = ref.biased_grouped_topk_torch(torch.from_numpy(g), torch.from_numpy(bias), k, True, G, TG)
        p = f"btopk/m{M}_e{E}/"
        out[p + "gating"] = g
        out[p + "bias"] = bias
        out[p + "meta"] = np.array([M, E, G, TG, k])
        out[p + "weights"] = t2n(w)
        out[p + "ids"] = t2n(ids)
    # ---------------------------------------------------------------- quantisers / codecs
    rng = np.random.default_rng(4000)
    x = inputs.make_hidden(rng, 16, 512)
    x[3, :128] = 0.0                       # an all-zero group takes scale 1
    x[5, 7] = 1000.0                       # a dominant outlier
    q, s = ref.pertoken_quant(torch.from_numpy(x).view(16, -1, 128), quant_dtype=torch.float8_e4m3fn)
    out["quant1x128/x"] = x
    out["quant1x128/q"] = t2n(q).reshape(16, 512)
    out["quant1x128/scale"] = t2n(s).reshape(16, 4)
    q8, s8 = ref.pertoken_quant(torch.from_numpy(x).view(16, -1, 128), quant_dtype=torch.int8)
    out["quant1x128_i8/q"] = t2n(q8).reshape(16, 512)
    out["quant1x128_i8/scale"] = t2n(s8).reshape(16, 4)
    w = (rng.standard_normal((2, 256, 384), dtype=np.float32) / np.float32(np.sqrt(384))).astype(np.float32)
    wq, ws = ref.weight_per_128x128_quant(torch.from_numpy(w), torch.float8_e4m3fn)
    out["quant128x128/w"] = w
    out["quant128x128/q"] = t2n(wq)
    out["quant128x128/scale"] = t2n(ws)
    xf = (rng.standard_normal((8, 256), dtype=np.float32) * 3).astype(np.float32)
    xf[0, :32] = 0.0
    xf[1, 5] = 40.0
    fq, fs = ref.per_1x32_f4_quant(torch.from_numpy(xf))
    out["quant1x32/x"] = xf
    out["quant1x32/q"] = t2n(fq)
    out["quant1x32/scale"] = t2n(fs)
    allb = torch.arange(256, dtype=torch.uint8)
    out["codec/mxfp4_all"] = t2n(ref.mxfp4_to_f32(allb.clone()))
    out["codec/e8m0_to_f32_all"] = t2n(ref.e8m0_to_f32(allb.clone()))
    special = np.array([0.0, 1e-40, 1.0, 1.5, 1.4999999, 1.75, 3.0, 0.375, 6.0, 1e38, np.inf, np.nan,
                        2.0 ** -127, 2.0 ** -126, 5.877472e-39, 1.2e-38] +
                       list(rng.random(64, dtype=np.float32) * 100), dtype=np.float32)
    out["codec/e8m0_in"] = special
    out["codec/e8m0_out"] = t2n(ref.f32_to_e8m0(torch.from_numpy(special.copy())))
    grid = np.linspace(-8, 8, 2048 + 1, dtype=np.float32)[:2048]
    out["codec/e2m1_in"] = grid
    out["codec/e2m1_out"] = t2n(ref.f32_to_mxfp4(torch.from_numpy(grid.copy()))).reshape(-1)
    fp8in = np.concatenate([np.linspace(-500, 500, 4001, dtype=np.float32),
                            (rng.standard_normal(4096).astype(np.float32) * 10),
                            np.array([2.0 ** -10, 2.0 ** -9 * 1.5, 2.0 ** -7 * 1.0625, 464.0, 448.0], np.float32)])
    out["codec/fp8_in"] = fp8in
    out["codec/fp8_out"] = t2n(torch.from_numpy(fp8in).to(torch.float8_e4m3fn))
    # ---------------------------------------------------------------- MXFP4 activation quant + MoE scale sort
    for i, (name, T, D, E, k, B, stage) in enumerate(MXFP4_SORT_CASES):
        rng = np.random.default_rng(5000 + i)
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        w = rng.random((T, k), dtype=np.float32)
        sid, _, _, nv = ref.moe_sorting_native(torch.from_numpy(ids), torch.from_numpy(w), E, B, None, None)
        rows = T if stage == 1 else T * k
        x = torch.from_numpy((rng.standard_normal((rows, D)) * 2).astype(np.float32)).to(torch.bfloat16)
        x[1, :32] = 0                          # an all-zero group
        x[2, 40] = 300.0                       # a dominant outlier
        q, sc = ref.per_1x32_f4_quant(x)
        sc8 = sc.view(torch.uint8)
        scale_in = sc8 if stage == 1 else sc8.view(T, k, D // 32)
        srt = ref.moe_mxfp4_sort_torch(scale_in.clone(), sid.clone(), nv[0], T)
        p = f"mxfp4sort/{name}/"
        out[p + "meta"] = np.array([T, D, E, k, B, stage], dtype=np.int64)
        out[p + "x"] = t2n(x)
        out[p + "sorted_ids"] = t2n(sid)
        out[p + "num_valid_ids"] = t2n(nv)
        out[p + "q"] = t2n(q)
        out[p + "scale"] = t2n(sc8)
        out[p + "sorted_scale"] = t2n(srt)
        # e8m0_shuffle pads with torch.empty: keep only elements whose source is real
        shf = t2n(ref.e8m0_shuffle(sc8.clone()))
        r_, c_ = mxfp4_sort.shuffle_index(*shf.shape)
        real = ((r_ < sc8.shape[0]) & (c_ < sc8.shape[1])).reshape(shf.shape)
        out[p + "shuffled_scale"] = np.where(real, shf, 0).astype(np.uint8)
    # ---------------------------------------------------------------- AMD weight pre-shuffle (to undo)
    rng = np.random.default_rng(6000)
    ws = rng.integers(0, 256, (2, 64, 128), dtype=np.uint8)
    out["shuffle/w_u8"] = ws
    out["shuffle/shuffled_fp8"] = t2n(ref.shuffle_weight(torch.from_numpy(ws.copy()).view(torch.float8_e4m3fn)))
    wb = rng.standard_normal((2, 32, 64)).astype(np.float32)
    out["shuffle/w_bf16"] = t2n(torch.from_numpy(wb).to(torch.bfloat16))
    out["shuffle/shuffled_bf16"] = t2n(ref.shuffle_weight(torch.from_numpy(wb).to(torch.bfloat16)))
    # ---------------------------------------------------------------- MoE config 0 (fp8 blockscale)
    for tag, (seed, M, D, I, E, k) in {"cfg0": (0, 32, 1024, 512, 8, 2),
                                        "cfg0_m7": (7, 7, 1024, 256, 8, 2)}.items():
        case = moe_reference_fp8(ref, seed, M, D, I, E, k)
        for kk, v in case.items():
            out[f"moe_fp8/{tag}/{kk}"] = v
    for tag, (seed, opts) in {"swiglu": (21, dict(activation=ActivationType.Swiglu)),
                              "doweight": (22, dict(doweight_stage1=True)),
                              "fp16": (23, dict(dtype=torch.float16)),
                              "bias_swiglu": (24, dict(activation=ActivationType.Swiglu, bias=True))}.items():
        case = moe_reference_fp8(ref, seed, 32, 1024, 512, 8, 2, **opts)
        for kk, v in case.items():
            out[f"moe_fp8_opts/{tag}/{kk}"] = v
    for tag, (seed, M, D, I, E, k) in {"cfg0": (11, 32, 1024, 512, 8, 2)}.items():
        case = moe_reference_a8w4(ref, seed, M, D, I, E, k)
        for kk, v in case.items():
            out[f"moe_a8w4/{tag}/{kk}"] = v
    # ---------------------------------------------------------------- topk_sigmoid, silu_and_mul
    # rows of unique values, as op_tests/test_moe_topk_sigmoid.py:114-125 draws them
    for tag, (E, k, M, dt) in {"e64_k4_bf16": (64, 4, 16, torch.bfloat16),
                                "e128_k8_fp16": (128, 8, 16, torch.float16),
                                "e128_k1_fp32": (128, 1, 8, torch.float32)}.items():
        g = torch.Generator().manual_seed(E * 10 + k)
        base = torch.arange(-1, 1, 2.0 / E).repeat((M, 1)).to(dt)
        perm = torch.argsort(torch.rand(base.shape, generator=g), dim=-1)
        logits = torch.gather(base, -1, perm)
        w, ids = ref.topk_sigmoid_torch(logits.clone(), k)
        out[f"topk_sigmoid/{tag}/logits"] = logits.float().numpy()
        out[f"topk_sigmoid/{tag}/weights"] = t2n(w)
        out[f"topk_sigmoid/{tag}/ids"] = t2n(ids)
    for tag, (M, N, dt) in {"bf16": (8, 512, torch.bfloat16), "fp32": (8, 384, torch.float32)}.items():
        g = torch.Generator().manual_seed(N)
        inp = torch.randn(M, N, generator=g).to(dt)
        out[f"silu_and_mul/{tag}/input"] = inp.float().numpy()
        out[f"silu_and_mul/{tag}/out"] = ref.torch_silu_and_mul(inp).float().numpy()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", len(out), "arrays", os.path.getsize(os.path.join(HERE, "golden.npz")), "bytes")


def _float_case(seed, M, D, I, E, k, zipf=None):
    """Float inputs drawn exactly as oracle.inputs.make_moe_case draws them."""
    rng = np.random.default_rng(seed)
    hidden = inputs.make_hidden(rng, M, D)
    logits = inputs.make_logits(rng, M, E, zipf)
    from oracle import routing
    tw, tid, _ = routing.topk_softmax(logits, k, True)
    w1 = (rng.standard_normal((E, 2 * I, D), dtype=np.float32) / np.float32(np.sqrt(D))).astype(np.float32)
    w2 = (rng.standard_normal((E, D, I), dtype=np.float32) / np.float32(np.sqrt(I))).astype(np.float32)
    return hidden, tw, tid, w1, w2


def moe_reference_fp8(ref, seed, M, D, I, E, k, activation=ActivationType.Silu, doweight_stage1=False,
                      dtype=torch.bfloat16, bias=False):
    """The reference's 2-stage pipeline (op_tests/test_moe_2stage.py:187-231) with its
    options: activation, doweight_stage1 (top-k weight applied to the stage-1 GEMM output,
    not in stage 2), the activation / output dtype (bf16 or fp16) and the experts'
    biases (drawn as op_tests/test_moe_2stage.py:62,70 draws them: clamp(randn, -1, 1)
    in the activation dtype; the kernels take them as f32, :146-147)."""
    hidden, tw, tid, w1, w2 = _float_case(seed, M, D, I, E, k)
    b1 = b2 = None
    if bias:
        brng = np.random.default_rng(seed + 1000)
        b1 = torch.from_numpy(brng.standard_normal((E, 2 * I)).astype(np.float32)).to(dtype).clamp(-1.0, 1.0)
        b2 = torch.from_numpy(brng.standard_normal((E, D)).astype(np.float32)).to(dtype).clamp(-1.0, 1.0)
    fp8 = torch.float8_e4m3fn
    w1q, w1s = ref.weight_per_128x128_quant(torch.from_numpy(w1), fp8)
    w2q, w2s = ref.weight_per_128x128_quant(torch.from_numpy(w2), fp8)
    h = torch.from_numpy(hidden).to(dtype)
    a1q, a1s = ref.pertoken_quant(h.view(M, -1, 128), quant_dtype=fp8)
    a1q = a1q.view(M, D)
    a1s = a1s.squeeze(-1)
    tw_t, tid_t = torch.from_numpy(tw), torch.from_numpy(tid)
    out1 = ref.torch_moe_stage1(a1q, w1q, w2q, tw_t, tid_t, dtype=dtype,
                                activation=activation, quant_type=QuantType.per_128x128,
                                a1_scale=a1s, w1_scale=w1s, doweight=doweight_stage1, w1_bias=b1)
    a2q, a2s = ref.pertoken_quant(out1.view(M, -1, 128), quant_dtype=fp8)
    a2s = a2s.view(M, k, -1)
    out2 = ref.torch_moe_stage2(a2q.view(M, k, -1), w1q, w2q, tw_t, tid_t, dtype=dtype,
                                quant_type=QuantType.per_128x128, w2_scale=w2s, a2_scale=a2s,
                                doweight=not doweight_stage1, w2_bias=b2)
    res = dict(w1q_sha=np.frombuffer(sha(t2n(w1q)).encode(), dtype=np.uint8),
               w2q_sha=np.frombuffer(sha(t2n(w2q)).encode(), dtype=np.uint8),
               w1s=t2n(w1s), w2s=t2n(w2s), a1q=t2n(a1q), a1s=t2n(a1s),
               out1=t2n(out1), a2s=t2n(a2s), out=t2n(out2), topk_ids=tid, topk_weights=tw)
    if bias:
        res.update(bias1=b1.float().numpy(), bias2=b2.float().numpy())
    return res


def moe_reference_a8w4(ref, seed, M, D, I, E, k):
    """BASELINE-defined A8W4: fp8 1x128 activations, MXFP4 weights; composed from the
    reference's quantisers / dequantisers and its stage functions on dequantised values."""
    hidden, tw, tid, w1, w2 = _float_case(seed, M, D, I, E, k)
    fp8 = torch.float8_e4m3fn
    w1p, w1e = ref.per_1x32_f4_quant(torch.from_numpy(w1))
    w2p, w2e = ref.per_1x32_f4_quant(torch.from_numpy(w2))

    def deq(p, e, shape):
        v = ref.mxfp4_to_f32(p.view(torch.uint8).reshape(shape[0], shape[1], -1))
        s = ref.e8m0_to_f32(e.view(torch.uint8)).reshape(shape[0], shape[1], -1)
        return (v.view(shape[0], shape[1], -1, 32) * s.unsqueeze(-1)).view(shape)

    w1d = deq(w1p, w1e, w1.shape)
    w2d = deq(w2p, w2e, w2.shape)
    h = torch.from_numpy(hidden).to(torch.bfloat16)
    a1q, a1s = ref.pertoken_quant(h.view(M, -1, 128), quant_dtype=fp8)
    a1d = (a1q.float() * a1s).view(M, D)
    tw_t, tid_t = torch.from_numpy(tw), torch.from_numpy(tid)
    out1 = ref.torch_moe_stage1(a1d, w1d, w2d, tw_t, tid_t, dtype=torch.bfloat16,
                                activation=ActivationType.Silu, quant_type=QuantType.No)
    a2q, a2s = ref.pertoken_quant(out1.view(M, -1, 128), quant_dtype=fp8)
    a2d = (a2q.float() * a2s).view(M, k, I)
    out2 = ref.torch_moe_stage2(a2d, w1d, w2d, tw_t, tid_t, dtype=torch.bfloat16,
                                quant_type=QuantType.No)
    return dict(w1p_sha=np.frombuffer(sha(t2n(w1p)).encode(), dtype=np.uint8),
                w2p_sha=np.frombuffer(sha(t2n(w2p)).encode(), dtype=np.uint8),
                w1e=t2n(w1e).reshape(E, 2 * I, -1), w2e=t2n(w2e).reshape(E, D, -1),
                out1=t2n(out1), out=t2n(out2), topk_ids=tid, topk_weights=tw)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
