"""Routing kernels vs the oracle and the reference's torch outputs (golden).

ids are compared exactly everywhere.  Weights are compared bit for bit (as uint32)
with the oracle, which restates the kernels' arithmetic contract, and against the
reference's torch outputs within the per-case ulp table of routing_ulps.py (torch's
softmax exp approximation and its unsorted grouped top-k order; the reference's own
test allows 1e-2, op_tests/test_moeTopkSoftmax.py:124-125)."""
import numpy as np
import pytest
import torch

import aiter_b200 as aiter
from conftest import golden_group
from gpu_util import dev, requires_cuda, to_dev
from oracle import routing
from routing_ulps import MAX_ULPS, ulps


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)

pytestmark = [pytest.mark.gpu, requires_cuda]


def _run_topk(g, k, renorm, dtype=torch.float32, stride_pad=0):
    M, E = g.shape
    gt = to_dev(g, dtype)
    # strided outputs as the reference test uses (op_tests/test_moeTopkSoftmax.py:56-64)
    w = torch.empty_strided((M, k), (k + stride_pad, 1), dtype=torch.float32, device=dev())
    ids = torch.empty_strided((M, k), (k + stride_pad, 1), dtype=torch.int32, device=dev())
    tei = torch.empty_strided((M, k), (k + stride_pad, 1), dtype=torch.int32, device=dev())
    aiter.topk_softmax(w, ids, tei, gt, renorm)
    torch.cuda.synchronize()
    return w.cpu().numpy(), ids.cpu().numpy(), tei.cpu().numpy()


def test_topk_softmax_matches_reference_golden(golden):
    for case, g in golden_group(golden, "topk").items():
        renorm = case.endswith("_r1")
        k = g["ids"].shape[1]
        w, ids, tei = _run_topk(g["gating"], k, renorm, stride_pad=10)
        assert np.array_equal(ids, g["ids"]), case
        assert ulps(w, g["weights"]).max() <= MAX_ULPS["topk/" + case], case
        w0, _, _ = routing.topk_softmax(g["gating"], k, renorm)
        assert np.array_equal(bits(w), bits(w0)), case
        M = g["gating"].shape[0]
        assert np.array_equal(tei, np.arange(k)[None, :] * M + np.arange(M)[:, None])


@pytest.mark.parametrize("E,k", [(8, 2), (16, 4), (64, 6), (128, 8), (256, 8), (384, 8), (512, 8), (1, 1), (3, 2)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_topk_softmax_vs_oracle(E, k, dtype):
    rng = np.random.default_rng(E * 31 + k)
    M = 77
    g = rng.standard_normal((M, E), dtype=np.float32)
    g_cast = torch.from_numpy(g).to(dtype).float().numpy()   # the values the kernel sees
    for renorm in (True, False):
        w, ids, _ = _run_topk(g, k, renorm, dtype)
        w0, ids0, _ = routing.topk_softmax(g_cast, k, renorm)
        # bf16/fp16 logits tie often: the lower expert index wins in both
        assert np.array_equal(ids, ids0)
        assert np.array_equal(bits(w), bits(w0))


def test_topk_softmax_strided_gating_rows():
    rng = np.random.default_rng(5)
    g_full = torch.from_numpy(rng.standard_normal((40, 138), dtype=np.float32)).to(dev())
    g = g_full[:, :128]                       # row stride 138
    w = torch.empty(40, 8, device=dev())
    ids = torch.empty(40, 8, dtype=torch.int32, device=dev())
    aiter.topk_softmax(w, ids, torch.empty_like(ids), g, True)
    w0, ids0, _ = routing.topk_softmax(g.cpu().numpy(), 8, True)
    assert np.array_equal(ids.cpu().numpy(), ids0)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w0))


def test_topk_softmax_shared_expert_sigmoid():
    rng = np.random.default_rng(9)
    g = rng.standard_normal((16, 64 + 2), dtype=np.float32)
    w = torch.zeros(16, 8 + 2, device=dev())
    ids = torch.empty(16, 8, dtype=torch.int32, device=dev())
    aiter.topk_softmax(w, ids, torch.empty_like(ids), to_dev(g), True, 2, "sigmoid")
    w0, ids0, _ = routing.topk_softmax(g[:, :64], 8, True)
    assert np.array_equal(ids.cpu().numpy(), ids0)
    assert np.array_equal(bits(w.cpu().numpy()[:, :8]), bits(w0))
    assert np.array_equal(bits(w.cpu().numpy()[:, 8:]), bits(routing._sigmoid(g[:, 64:])))


def test_topk_softmax_empty_input():
    w = torch.empty(0, 8, device=dev())
    ids = torch.empty(0, 8, dtype=torch.int32, device=dev())
    aiter.topk_softmax(w, ids, torch.empty_like(ids), torch.empty(0, 128, device=dev()), True)


def _sorted(ids, w):
    o = np.argsort(ids, axis=-1)
    return np.take_along_axis(ids, o, -1), np.take_along_axis(w, o, -1)


def test_grouped_topk_matches_reference_golden(golden):
    for case, g in golden_group(golden, "gtopk").items():
        M, E, G, TG, k = [int(v) for v in g["meta"]]
        w = torch.empty(M, k, device=dev())
        ids = torch.empty(M, k, dtype=torch.int32, device=dev())
        aiter.grouped_topk(to_dev(g["gating"]), w, ids, G, TG, True, case.endswith("softmax"), 1.0)
        i0, w0 = _sorted(ids.cpu().numpy(), w.cpu().numpy())
        i1, w1 = _sorted(g["ids"], g["weights"])
        assert np.array_equal(i0, i1), case
        assert ulps(w0, w1).max() <= MAX_ULPS["gtopk/" + case], case
        wo, io = routing.grouped_topk(g["gating"], k, G, TG, True, case.endswith("softmax"))
        assert np.array_equal(ids.cpu().numpy(), io) and np.array_equal(bits(w.cpu().numpy()), bits(wo)), case


def test_biased_grouped_topk_matches_reference_golden(golden):
    for case, g in golden_group(golden, "btopk").items():
        M, E, G, TG, k = [int(v) for v in g["meta"]]
        w = torch.empty(M, k, device=dev())
        ids = torch.empty(M, k, dtype=torch.int32, device=dev())
        aiter.biased_grouped_topk(to_dev(g["gating"]), to_dev(g["bias"]), w, ids, G, TG, True, 1.0)
        i0, w0 = _sorted(ids.cpu().numpy(), w.cpu().numpy())
        i1, w1 = _sorted(g["ids"], g["weights"])
        assert np.array_equal(i0, i1), case
        assert ulps(w0, w1).max() <= MAX_ULPS["btopk/" + case], case
        wo, io = routing.biased_grouped_topk(g["gating"], g["bias"], k, G, TG, True)
        assert np.array_equal(ids.cpu().numpy(), io) and np.array_equal(bits(w.cpu().numpy()), bits(wo)), case


@pytest.mark.parametrize("scale", [1.0, 2.5])
def test_grouped_topk_deepseek_shape_vs_oracle(scale):
    rng = np.random.default_rng(77)
    M, E, G, TG, k = 300, 256, 8, 4, 8
    g = rng.standard_normal((M, E), dtype=np.float32)
    bias = (0.05 * rng.standard_normal(E)).astype(np.float32)
    w = torch.empty(M, k, device=dev())
    ids = torch.empty(M, k, dtype=torch.int32, device=dev())
    aiter.biased_grouped_topk(to_dev(g), to_dev(bias), w, ids, G, TG, True, scale)
    w0, ids0 = routing.biased_grouped_topk(g, bias, k, G, TG, True, scale)
    assert np.array_equal(ids.cpu().numpy(), ids0)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w0))
    for soft in (True, False):
        aiter.grouped_topk(to_dev(g), w, ids, G, TG, True, soft, scale)
        w0, ids0 = routing.grouped_topk(g, k, G, TG, True, soft, scale)
        assert np.array_equal(ids.cpu().numpy(), ids0)
        assert np.array_equal(bits(w.cpu().numpy()), bits(w0))
