"""FP8 block-scale fused MoE (tcgen05 grouped GEMMs) vs the reference.

* config 0 (M=32, D=1024, I=512, E=8, k=2) against the reference's own torch
  outputs (tests/golden, torch_moe_stage1 -> requant -> torch_moe_stage2);
* shape sweeps against the numpy oracle;
* the full single-GPU config (D=4096, I=1536, E=128, k=8, M=4096) against a
  plain fp32 torch reference (its own 1x128 quantiser, dequantised weights,
  per-expert GEMMs) on a sample of tokens (the MoE is independent per token, so a
  sample checks the full-size launch).
Tolerance: rtol = atol = 2e-2 on bf16 outputs (the path's stated tolerance), plus at most
1 % of elements off by more than 1e-2 (op_tests/test_moe_2stage.py:253-269 uses
1e-2 with a mismatch ratio)."""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from aiter_b200 import weights as W
from aiter_b200.fused_moe import _moe_sorting_ext
from conftest import golden_group
from gpu_util import check_no_device_error, codes, dev, fp8_from_codes, requires_cuda, to_dev
from oracle import inputs, moe, quant

pytestmark = [pytest.mark.gpu, requires_cuda]

RTOL = ATOL = 2e-2


def assert_moe_close(out, ref, frac=0.01):
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    bad = np.abs(out - ref) > 1e-2 + 1e-2 * np.abs(ref)
    assert bad.mean() <= frac, f"{bad.mean():.4f} of elements beyond 1e-2"


def run_case_gpu(c):
    hidden = to_dev(c["hidden"], torch.bfloat16)
    w1 = fp8_from_codes(c["w1_q"])
    w2 = fp8_from_codes(c["w2_q"])
    w1s, w2s = to_dev(c["w1_s"]), to_dev(c["w2_s"])
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])
    out = aiter.fused_moe(hidden, w1, w2, tw, tid, quant_type=aiter.QuantType.per_1x128,
                          activation=aiter.ActivationType.Silu, w1_scale=w1s, w2_scale=w2s)
    torch.cuda.synchronize()
    check_no_device_error()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("tag,shape", [("cfg0", (0, 32, 1024, 512, 8, 2)), ("cfg0_m7", (7, 7, 1024, 256, 8, 2))])
def test_fused_moe_matches_reference_golden(golden, tag, shape):
    g = golden_group(golden, "moe_fp8")[tag]
    seed, M, D, I, E, k = shape
    if I % 128 or D % 256:
        pytest.skip("shape not tiled by this kernel")
    c = inputs.make_moe_case(seed, M, D, I, E, k)
    out = run_case_gpu(c)
    assert_moe_close(out, g["out"])


def test_gather_quant_sorted_rows_vs_oracle():
    """Sorted-row fp8 activations: each real row equals the oracle's 1x128 quant of
    its token (bit-exact codes and scales); padding rows are zero."""
    c = inputs.make_moe_case(0, 32, 1024, 512, 8, 2)
    a1_q, a1_s = quant.per_1x128_quant(c["hidden"])
    tid, tw = to_dev(c["topk_ids"]), to_dev(c["topk_weights"])
    sids, sw, seids, nv, buf, pos = _moe_sorting_ext(tid, tw, 8, 1024, torch.bfloat16, 128, with_pos=True)
    # every (token, slot) maps to the sorted row holding it
    p = pos.cpu().numpy().reshape(32, 2)
    sid = sids.cpu().numpy()
    assert np.array_equal(sid[p] & 0xFFFFFF, np.repeat(np.arange(32)[:, None], 2, 1))
    assert np.array_equal(sid[p] >> 24, np.repeat(np.arange(2)[None, :], 32, 0))
    for hidden, hs in ((to_dev(c["hidden"], torch.bfloat16), None), (fp8_from_codes(a1_q), to_dev(a1_s))):
        a1, a1s = aiter.moe_gather_quant_1x128(hidden, pos, 2, sids.numel(), hidden_scale=hs)
        torch.cuda.synchronize()
        n = int(nv[0])
        tok = sid[:n] & 0xFFFFFF
        q = codes(a1)[:n]
        s = a1s.cpu().numpy()[:, :n].T
        real = tok < 32
        assert np.array_equal(q[real], a1_q[tok[real]])
        assert np.array_equal(s[real].view(np.uint32), a1_s[tok[real]].view(np.uint32))


def test_stage1_intermediate_vs_oracle():
    """Stage 1 alone: fp8 codes / scales of act(gate)*up per sorted row against the
    oracle's intermediate of that (token, slot)."""
    c = inputs.make_moe_case(0, 32, 1024, 512, 8, 2)
    _, st = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                         c["topk_weights"], c["topk_ids"], return_intermediate=True)
    M, k, I = 32, 2, 512
    tid, tw = to_dev(c["topk_ids"]), to_dev(c["topk_weights"])
    sids, sw, seids, nv, buf, pos = _moe_sorting_ext(tid, tw, 8, 1024, torch.bfloat16, 128, with_pos=True)
    a1, a1s = aiter.moe_gather_quant_1x128(to_dev(c["hidden"], torch.bfloat16), pos, 2, sids.numel())
    rows = sids.numel()
    a2 = torch.empty(rows, I, dtype=torch.float8_e4m3fn, device=dev())
    a2s = torch.empty(I // 128, rows, device=dev())
    aiter.moe_stage1_fp8_blockscale(a1, a1s, fp8_from_codes(c["w1_q"]), to_dev(c["w1_s"]), sids, seids, nv,
                                    a2, a2s, M, 128)
    torch.cuda.synchronize()
    check_no_device_error()
    n = int(nv[0])
    sid = sids.cpu().numpy()[:n]
    tok, slot = sid & 0xFFFFFF, sid >> 24
    real = tok < M
    q = codes(a2)[:n][real]
    s = a2s.cpu().numpy()[:, :n].T[real]
    s_ref = st["a2_s"][tok[real], slot[real]]
    q_ref = st["a2_q"][tok[real], slot[real]]
    ref = st["out1"][tok[real], slot[real]]
    np.testing.assert_allclose(s, s_ref, rtol=1e-2)
    deq = quant.dequant_1x128(q, s)
    np.testing.assert_allclose(deq, ref, rtol=0.07, atol=0.02 * np.abs(ref).max())
    same = (q == q_ref).mean()
    assert same > 0.97, f"only {same:.3f} of fp8 codes equal"


@pytest.mark.parametrize("M", [1, 5, 64, 200])
@pytest.mark.parametrize("D,I,E,k", [(1024, 512, 8, 2), (512, 256, 16, 4), (2048, 768, 32, 8)])
def test_fused_moe_vs_oracle(M, D, I, E, k):
    c = inputs.make_moe_case(M * 13 + E, M, D, I, E, k)
    out = run_case_gpu(c)
    ref = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                       c["topk_weights"], c["topk_ids"])
    assert_moe_close(out, ref)


def test_fused_moe_gelu_vs_oracle():
    c = inputs.make_moe_case(3, 48, 1024, 512, 8, 2)
    hidden = to_dev(c["hidden"], torch.bfloat16)
    out = aiter.fused_moe(hidden, fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"]),
                          to_dev(c["topk_weights"]), to_dev(c["topk_ids"]),
                          quant_type=aiter.QuantType.per_128x128, activation=aiter.ActivationType.Gelu,
                          w1_scale=to_dev(c["w1_s"]), w2_scale=to_dev(c["w2_s"]))
    ref = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                       c["topk_weights"], c["topk_ids"], activation="gelu")
    assert_moe_close(out.float().cpu().numpy(), ref)


def test_fused_moe_preq_input_and_repeat_calls():
    """fp8 input with a1_scale skips the activation quant; two calls in a row agree
    (the output buffer is re-zeroed by sorting every call)."""
    c = inputs.make_moe_case(4, 40, 1024, 512, 8, 2)
    q, s = quant.per_1x128_quant(c["hidden"])
    args = (fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"]), to_dev(c["topk_weights"]), to_dev(c["topk_ids"]))
    kw = dict(quant_type=aiter.QuantType.per_1x128, w1_scale=to_dev(c["w1_s"]), w2_scale=to_dev(c["w2_s"]),
              a1_scale=to_dev(s))
    o1 = aiter.fused_moe(fp8_from_codes(q), *args, **kw)
    o2 = aiter.fused_moe(fp8_from_codes(q), *args, **kw)
    ref = moe.fused_moe_fp8_blockscale(c["hidden"], c["w1_q"], c["w1_s"], c["w2_q"], c["w2_s"],
                                       c["topk_weights"], c["topk_ids"])
    assert_moe_close(o1.float().cpu().numpy(), ref)
    assert_moe_close(o2.float().cpu().numpy(), ref)


# --------------------------------------------------------------------- full size


def torch_quant_1x128(x):
    """pertoken_quant over 1x128 groups in plain torch: (dequantised values, e4m3
    values).  scale = amax / 448 (1 for an all-zero group) and the codes of x / scale,
    both as IEEE divisions of two tensors, as the reference computes them on the CPU
    (on CUDA, torch turns a division by a Python scalar into a multiplication by its
    reciprocal, which can move the scale by one ulp and an exact tie to the other
    code)."""
    g = x.float().view(x.shape[0], -1, 128)
    amax = g.abs().amax(dim=-1, keepdim=True)
    sc = torch.div(amax, torch.full_like(amax, 448.0))
    sc = torch.where(sc == 0, torch.ones_like(sc), sc)
    q = torch.div(g, sc).to(torch.float8_e4m3fn)
    return (q.float() * sc).view(x.shape[0], -1), q.view(x.shape[0], -1)


def torch_reference_tokens(hidden, w1q, w1s, w2q, w2s, tw, tid, tokens):
    """fp32 torch reference of the 2-stage blockscale path for a subset of tokens."""
    a1, _ = torch_quant_1x128(hidden[tokens])
    outs = []
    I = w2q.shape[2]
    for i, t in enumerate(tokens.tolist()):
        acc = torch.zeros(hidden.shape[1], device=hidden.device)
        for j in range(tid.shape[1]):
            e = int(tid[t, j])
            w1 = W.dequant_128x128(w1q[e:e + 1], w1s[e:e + 1])[0]
            h = w1 @ a1[i]
            y = (torch.nn.functional.silu(h[:I]) * h[I:]).to(torch.bfloat16)
            a2, _ = torch_quant_1x128(y[None])
            w2 = W.dequant_128x128(w2q[e:e + 1], w2s[e:e + 1])[0]
            acc += tw[t, j] * (w2 @ a2[0])
        outs.append(acc.to(torch.bfloat16).float())
    return torch.stack(outs)


@pytest.mark.parametrize("M", [4096, 1, 16, 128])
def test_fused_moe_full_size_config1(M):
    torch.manual_seed(M)
    D, I, E, k = 4096, 1536, 128, 8
    g = torch.Generator(device=dev()).manual_seed(1234)
    w1 = torch.randn(E, 2 * I, D, device=dev(), generator=g) / D ** 0.5
    w1q, w1s = W.quant_weight_128x128(w1)
    del w1
    w2 = torch.randn(E, D, I, device=dev(), generator=g) / I ** 0.5
    w2q, w2s = W.quant_weight_128x128(w2)
    del w2
    hidden = torch.randn(M, D, device=dev(), generator=g).to(torch.bfloat16)
    logits = torch.randn(M, E, device=dev(), generator=g)
    tw, tid = aiter.fused_topk(hidden, logits, k, True)
    out = aiter.fused_moe(hidden, w1q, w2q, tw, tid, quant_type=aiter.QuantType.per_1x128,
                          w1_scale=w1s, w2_scale=w2s)
    torch.cuda.synchronize()
    check_no_device_error()
    tokens = torch.randperm(M, device=dev())[:64]
    ref = torch_reference_tokens(hidden, w1q, w1s, w2q, w2s, tw, tid, tokens)
    assert_moe_close(out[tokens].float().cpu().numpy(), ref.cpu().numpy())
    assert torch.isfinite(out.float()).all()


def test_fused_moe_traces_under_torch_compile():
    """torch.compile (dynamo + AOT autograd, no inductor codegen) traces through the
    custom op with its fake implementation and runs the same kernels."""
    c = inputs.make_moe_case(3, 16, 1024, 512, 8, 2)
    hidden = to_dev(c["hidden"], torch.bfloat16)
    w1, w2 = fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"])
    w1s, w2s = to_dev(c["w1_s"]), to_dev(c["w2_s"])
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])

    def f(x, a, b, sa, sb, w, i):
        return aiter.fused_moe(x, a, b, w, i, quant_type=aiter.QuantType.per_1x128, w1_scale=sa, w2_scale=sb)

    compiled = torch.compile(f, backend="aot_eager", fullgraph=True)
    out_c = compiled(hidden, w1, w2, w1s, w2s, tw, tid)
    out_e = f(hidden, w1, w2, w1s, w2s, tw, tid)
    torch.cuda.synchronize()
    check_no_device_error()
    assert out_c.shape == out_e.shape and out_c.dtype == torch.bfloat16
    # the stage-2 scatter-add is bf16 atomics in no fixed order
    assert torch.allclose(out_c.float(), out_e.float(), rtol=1e-2, atol=1e-2)


def test_fused_moe_expert_parallel_partials_sum_to_full():
    """Expert parallelism through `expert_mask` (the EP path of fused_moe,
    aiter/fused_moe.py:118-144 with op_tests/test_moe_ep.py): each of two simulated
    ranks holds half of the experts' weights; the masked sort maps global expert ids
    to local ones and drops tokens routed elsewhere, so the two partial outputs add up
    to the full MoE."""
    M, D, I, E, k = 64, 1024, 512, 16, 4
    c = inputs.make_moe_case(11, M, D, I, E, k)
    hidden = to_dev(c["hidden"], torch.bfloat16)
    w1, w2 = fp8_from_codes(c["w1_q"]), fp8_from_codes(c["w2_q"])
    w1s, w2s = to_dev(c["w1_s"]), to_dev(c["w2_s"])
    tw, tid = to_dev(c["topk_weights"]), to_dev(c["topk_ids"])
    kw = dict(quant_type=aiter.QuantType.per_1x128)
    full = aiter.fused_moe(hidden, w1, w2, tw, tid, w1_scale=w1s, w2_scale=w2s, **kw)
    total = torch.zeros_like(full, dtype=torch.float32)
    for r in range(2):
        lo, hi = r * E // 2, (r + 1) * E // 2
        mask = torch.zeros(E, dtype=torch.int32, device=dev())
        mask[lo:hi] = 1
        part = aiter.fused_moe(hidden, w1[lo:hi].contiguous(), w2[lo:hi].contiguous(), tw, tid, expert_mask=mask,
                               w1_scale=w1s[lo:hi].contiguous(), w2_scale=w2s[lo:hi].contiguous(), **kw)
        total += part.float()
    torch.cuda.synchronize()
    check_no_device_error()
    # the partials are bf16-rounded before the sum
    assert_moe_close(total.cpu().numpy(), full.float().cpu().numpy())


def test_fused_moe_graph_replay_matches_eager():
    """The four kernels of a step (sorting, gather-quant, stage 1, stage 2) captured in a
    CUDA graph and replayed with new routing and activations copied into the static
    inputs give the eager results (the graph replay the token sweep of bench.py times)."""
    from aiter_b200 import moe_op
    M, D, I, E, k = 96, 1024, 512, 16, 4
    cases = [inputs.make_moe_case(40 + i, M, D, I, E, k) for i in range(3)]
    c0 = cases[0]
    w1, w2 = fp8_from_codes(c0["w1_q"]), fp8_from_codes(c0["w2_q"])
    w1s, w2s = to_dev(c0["w1_s"]), to_dev(c0["w2_s"])
    hid = to_dev(c0["hidden"], torch.bfloat16).clone()
    tw, tid = to_dev(c0["topk_weights"]).clone(), to_dev(c0["topk_ids"]).clone()
    B = 128
    max_pad = M * k + E * B - k
    sid = torch.empty(max_pad, dtype=torch.int32, device=dev())
    sw = torch.empty(max_pad, dtype=torch.float32, device=dev())
    seid = torch.empty((max_pad + B - 1) // B, dtype=torch.int32, device=dev())
    nv = torch.empty(2, dtype=torch.int32, device=dev())
    pos = torch.empty(M * k, dtype=torch.int32, device=dev())
    out = torch.empty(M, D, dtype=torch.bfloat16, device=dev())
    ws_n = moe_op.moe_sorting_get_workspace_size(M, E, k, 0)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev())
    a1 = torch.empty(max_pad, D, dtype=torch.float8_e4m3fn, device=dev())
    a1s = torch.empty(D // 128, max_pad, dtype=torch.float32, device=dev())
    a2 = torch.empty(max_pad, I, dtype=torch.float8_e4m3fn, device=dev())
    a2s = torch.empty(I // 128, max_pad, dtype=torch.float32, device=dev())

    def step():
        moe_op.moe_sorting_fwd(tid, tw, sid, sw, seid, nv, out, E, B, None, None, 0, ws if ws_n else None, pos)
        moe_op.moe_gather_quant_1x128(hid, pos, k, max_pad, out=a1, out_scale=a1s)
        moe_op.moe_stage1_fp8_blockscale(a1, a1s, w1, w1s, sid, seid, nv, a2, a2s, M, B)
        moe_op.moe_stage2_fp8_blockscale(a2, a2s, w2, w2s, sid, seid, nv, sw, out, B)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # kernels loaded and attributes set before capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    for c in cases:
        hid.copy_(to_dev(c["hidden"], torch.bfloat16))
        tw.copy_(to_dev(c["topk_weights"]))
        tid.copy_(to_dev(c["topk_ids"]))
        g.replay()
        torch.cuda.synchronize()
        check_no_device_error()
        eager = aiter.fused_moe(to_dev(c["hidden"], torch.bfloat16), w1, w2, to_dev(c["topk_weights"]),
                                to_dev(c["topk_ids"]), quant_type=aiter.QuantType.per_1x128, w1_scale=w1s,
                                w2_scale=w2s)
        torch.cuda.synchronize()
        assert_moe_close(out.float().cpu().numpy(), eager.float().cpu().numpy())
    del g
