"""bf16 tcgen05 GEMM (single GPU) and the allreduce's bounded waits.

* gemm_a16w16 vs a plain fp32 torch reference (bf16 output: rtol 1e-2, atol 1e-2
  relative to the output scale);
* an allreduce whose peers never arrive (every peer slot mapped to this rank's own
  region, so nobody writes the awaited flags) must give up after ~2 s, set the error
  word the host reads, and leave the GPU usable."""
import ctypes
import time

import pytest
import torch

from aiter_b200 import _lib
from aiter_b200.gemm import gemm_a16w16, tgemm
from gpu_util import dev, requires_cuda

pytestmark = [pytest.mark.gpu, requires_cuda]


@pytest.mark.parametrize("M", [1, 7, 128, 300, 2048])
@pytest.mark.parametrize("N,K", [(4096, 1024), (256, 4096), (512, 64)])
def test_gemm_a16w16_vs_torch(M, N, K):
    g = torch.Generator(device=dev()).manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device=dev(), generator=g).to(torch.bfloat16)
    W = torch.randn(N, K, device=dev(), generator=g).to(torch.bfloat16)
    out = gemm_a16w16(A, W)
    ref = A.float() @ W.float().t()
    torch.cuda.synchronize()
    err = (out.float() - ref).abs()
    tol = 1e-2 * ref.abs() + 1e-2 * ref.abs().max()
    assert bool((err <= tol).all()), float(err.max())


# (M, N, K) chosen so that every tile width runs: 32-wide (M=1, N=4096), 64-wide
# (N=10240), 128-wide (M=200, N=16384), 256-wide (M=2048, N=4096); plus N=96.
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (3, 96, 192), (100, 10240, 256), (200, 16384, 128),
                                   (2048, 4096, 512)])
def test_gemm_every_tile_width_vs_torch(M, N, K):
    g = torch.Generator(device=dev()).manual_seed(M + N + K)
    A = torch.randn(M, K, device=dev(), generator=g).to(torch.bfloat16)
    W = torch.randn(N, K, device=dev(), generator=g).to(torch.bfloat16)
    out = gemm_a16w16(A, W)
    ref = A.float() @ W.float().t()
    torch.cuda.synchronize()
    err = (out.float() - ref).abs()
    tol = 1e-2 * ref.abs() + 1e-2 * ref.abs().max()
    assert bool((err <= tol).all()), float(err.max())


# Cluster splits that do not divide the activation tile: N=3072 gives 24 tiles and a
# split of 6 (32- to 256-row tiles), N=1536 at M=512 gives 24 tiles of 256 rows.
@pytest.mark.parametrize("M,N,K", [(1, 3072, 1024), (60, 3072, 2048), (300, 3072, 1024), (512, 1536, 4096),
                                   (511, 1536, 1024), (33, 1536, 512)])
def test_gemm_uneven_cluster_split_vs_torch(M, N, K):
    g = torch.Generator(device=dev()).manual_seed(M + 3 * N + K)
    A = torch.randn(M, K, device=dev(), generator=g).to(torch.bfloat16)
    W = torch.randn(N, K, device=dev(), generator=g).to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), device=dev(), dtype=torch.bfloat16)
    gemm_a16w16(A, W, out)
    ref = A.float() @ W.float().t()
    torch.cuda.synchronize()
    err = (out.float() - ref).abs()
    tol = 1e-2 * ref.abs() + 1e-2 * ref.abs().max()
    assert bool((err <= tol).all()), float(err.nan_to_num(1e30).max())


def test_gemm_writes_only_its_rows_of_a_strided_output():
    A = torch.randn(5, 128, device=dev()).to(torch.bfloat16)
    W = torch.randn(256, 128, device=dev()).to(torch.bfloat16)
    big = torch.full((8, 512), 7.0, device=dev(), dtype=torch.bfloat16)
    out = big[:5, 128:384]
    gemm_a16w16(A, W, out)
    ref = (A.float() @ W.float().t()).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.allclose(out.float(), ref.float(), rtol=1e-2, atol=1e-1)
    assert bool((big[5:] == 7.0).all()) and bool((big[:, :128] == 7.0).all()) and bool((big[:, 384:] == 7.0).all())


def test_tgemm_mm_matches_gemm():
    A = torch.randn(2, 3, 256, device=dev()).to(torch.bfloat16)
    W = torch.randn(512, 256, device=dev()).to(torch.bfloat16)
    y = tgemm.mm(A, W)
    assert y.shape == (2, 3, 512)
    assert torch.equal(y.view(6, 512), gemm_a16w16(A.view(6, 256), W))


def test_allreduce_wait_times_out_when_peers_never_arrive():
    L = _lib.lib()
    L.custom_ar_device_error(1)
    ctx = ctypes.c_int64(0)
    handle = ctypes.create_string_buffer(64)
    _lib.check_status("custom_ar_init", L.custom_ar_init(0, 2, 1 << 20, 0, ctypes.byref(ctx), handle))
    try:
        _lib.check_status("custom_ar_open_loopback", L.custom_ar_open_loopback(ctx.value))
        x = torch.ones(4096, dtype=torch.bfloat16, device=dev())
        y = torch.zeros_like(x)
        a, b = _lib.to_aiter(x), _lib.to_aiter(y)
        t0 = time.time()
        _lib.check_status("custom_ar_all_reduce", L.custom_ar_all_reduce(
            ctx.value, ctypes.byref(a), ctypes.byref(b), 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        assert 1.5 < time.time() - t0 < 30
        assert L.custom_ar_device_error(1) == 1
        # the context stays usable
        z = (torch.ones(8, device=dev()) * 2).sum()
        assert float(z) == 16.0
    finally:
        L.custom_ar_dispose(ctx.value)
