"""GPU parity of the MXFP4 activation quant and the MoE-sorted e8m0 scale layout
(dynamic_per_group_scaled_quant_fp4, mxfp4_moe_sort_hip,
fused_dynamic_mxfp4_quant_moe_sort_hip): bit-exact against the reference's torch
functions (golden vectors: per_1x32_f4_quant, e8m0_shuffle and the sorted-layout
reference of op_tests/test_moe_sorting_mxfp4.py) and against the oracle at config-2
size."""
import numpy as np
import pytest
import torch

from conftest import golden_group
from gpu_util import check_no_device_error, dev, requires_cuda, to_dev

pytestmark = [pytest.mark.gpu, requires_cuda]

CASES = ["s1_t37_d512_e8_k2_b32", "s2_t37_d512_e8_k2_b32", "s1_t300_d1024_e16_k4_b128", "s2_t64_d256_e32_k8_b64"]


def _u8(t):
    return t.view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("case", CASES)
def test_quant_sort_match_reference(golden, case):
    import aiter_b200 as aiter
    from oracle import mxfp4_sort
    g = golden_group(golden, "mxfp4sort")[case]
    T, D, E, k, B, stage = (int(v) for v in g["meta"])
    x = to_dev(g["x"], torch.bfloat16)
    sid = to_dev(g["sorted_ids"])
    nv = to_dev(g["num_valid_ids"])
    # quant, scales in row order
    q, s = aiter.per_1x32_f4_quant_hip(x)
    torch.cuda.synchronize()
    assert np.array_equal(_u8(q), g["q"])
    assert np.array_equal(_u8(s), g["scale"])
    # quant, scales in the e8m0_shuffle layout (compared where the source is real)
    q2, s2 = aiter.per_1x32_f4_quant_hip(x, shuffle=True)
    assert np.array_equal(_u8(q2), g["q"])
    sh = _u8(s2)
    r, c = mxfp4_sort.shuffle_index(*sh.shape)
    real = ((r < g["scale"].shape[0]) & (c < g["scale"].shape[1])).reshape(sh.shape)
    assert np.array_equal(sh[real], g["shuffled_scale"][real])
    # sort of the row-order scales
    scale_in = s if stage == 1 else s.view(T, k, D // 32)
    srt = aiter.mxfp4_moe_sort_fwd(scale_in, sid, nv, T, D)
    assert np.array_equal(_u8(srt), g["sorted_scale"])
    # fused quant + sort, and the Python dispatch (both branches give the same bytes)
    out = torch.empty(x.shape[0], D // 2, dtype=torch.uint8, device=dev())
    fs = torch.full_like(srt.view(torch.uint8), 0x55)
    aiter.fused_dynamic_mxfp4_quant_moe_sort_hip(out, fs, x, sid, nv, T, B)
    assert np.array_equal(out.cpu().numpy(), g["q"])
    assert np.array_equal(fs.cpu().numpy(), g["sorted_scale"])
    oq, os_ = aiter.fused_dynamic_mxfp4_quant_moe_sort(x, sid, nv, T, k, B)
    assert np.array_equal(_u8(oq), g["q"]) and np.array_equal(_u8(os_), g["sorted_scale"])
    check_no_device_error()


def test_num_rows_skips_rows_past_the_count():
    import aiter_b200 as aiter
    x = torch.randn(64, 512, device=dev()).to(torch.bfloat16)
    out = torch.full((64, 256), 0xAB, dtype=torch.uint8, device=dev())
    sc = torch.full((64, 16), 0xCD, dtype=torch.uint8, device=dev())
    n = torch.tensor([10], dtype=torch.int32, device=dev())
    aiter.dynamic_per_group_scaled_quant_fp4(out, x, sc, 32, shuffle_scale=False, num_rows=n, num_rows_factor=3)
    ref_q, ref_s = aiter.per_1x32_f4_quant_hip(x)
    assert torch.equal(out[:30], ref_q.view(torch.uint8)[:30]) and torch.equal(sc[:30], ref_s.view(torch.uint8)[:30])
    assert bool((out[30:] == 0xAB).all()) and bool((sc[30:] == 0xCD).all())


@pytest.mark.parametrize("stage", [1, 2])
def test_config2_size_against_oracle(stage):
    """Config-2 routing (E=256, top-8, Zipf-skewed) at M=2048, model_dim 4096 (stage 1) /
    inter 2048 (stage 2): the split path (quant then sort)."""
    import aiter_b200 as aiter
    from oracle import inputs, mxfp4_sort, quant, sorting
    rng = np.random.default_rng(77 + stage)
    M, E, k, B = 2048, 256, 8, 128
    D = 4096 if stage == 1 else 2048
    lg = inputs.make_logits(rng, M, E, zipf_s=1.1)
    ids = np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)
    w = rng.random((M, k), dtype=np.float32)
    sid, _, _, nv = sorting.moe_sorting(ids, w, E, B)
    rows = M if stage == 1 else M * k
    xb = torch.from_numpy((rng.standard_normal((rows, D)) * 3).astype(np.float32)).to(torch.bfloat16)
    out, sc = aiter.fused_dynamic_mxfp4_quant_moe_sort(xb.to(dev()), to_dev(sid), to_dev(nv), M, k, B)
    q_ref, s_ref = quant.per_1x32_f4_quant(xb.float().numpy())
    assert np.array_equal(_u8(out), q_ref)
    scale_in = s_ref if stage == 1 else s_ref.reshape(M, k, D // 32)
    assert np.array_equal(_u8(sc), mxfp4_sort.moe_mxfp4_sort(scale_in, sid, int(nv[0]), M))
    check_no_device_error()
