"""Multi-GPU parity of the one-kernel GEMM + allreduce (custom_ar_gemm_all_reduce_fused),
one process per GPU.  Skipped with fewer than 2 GPUs.

The fused kernel pushes the same bf16 partial products the two-kernel path stages
and sums them in the same rank order, so it must return the two-kernel path's bits:
* small M (swap-AB kernel): one-shot and two-shot, forced and by size;
* large M (persistent kernel): two-shot, including a last row block that is partly
  past M and a shape whose tile count is not a multiple of the world size;
* ten calls in a row alternating with plain allreduce calls (staging buffers and
  per-CTA epochs shared with the allreduce), identical bits on every rank;
* a fused call captured in a CUDA graph, replayed with new inputs between eager calls.
"""
import os
import sys

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def _operands(M, K, N, world, seed):
    g = torch.Generator().manual_seed(seed)
    As = [torch.randn(M, K, generator=g).to(torch.bfloat16) for _ in range(world)]
    Ws = [torch.randn(N, K, generator=g).to(torch.bfloat16) for _ in range(world)]
    return As, Ws


def _same_everywhere(t, group):
    gathered = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(gathered, t, group=group)
    return all(torch.equal(g, t) for g in gathered)


def _worker(rank, world, port):
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from aiter_b200 import _lib
    from aiter_b200.dist import parallel_state as ps
    ps.init_distributed_environment(world, rank, f"tcp://127.0.0.1:{port}", rank, "nccl", timeout_s=60)
    tp = ps.initialize_model_parallel(world, local_rank=rank, ca_max_size=64 * 1024 * 1024)
    ca = tp.ca_comm
    dev = torch.device("cuda", rank)
    cases = [(1, None), (8, None), (64, False), (64, True), (200, None), (512, True), (512, None),
             (640, None), (1000, None), (2048, None)]
    for i, (M, two) in enumerate(cases):
        K, N = 8192 // world, 4096
        As, Ws = _operands(M, K, N, world, 4000 + i)
        a, w = As[rank].to(dev), Ws[rank].to(dev)
        plain = ca.gemm_all_reduce(a, w, two_shot=two)
        fused = ca.gemm_all_reduce(a, w, two_shot=two, fused=True)
        # a plain allreduce between fused calls shares the buffers and CTA epochs
        x = torch.randn(4096 * (i + 1), generator=torch.Generator().manual_seed(i)).to(torch.bfloat16).to(dev)
        xr = ca.all_reduce(x)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0, (M, two)
        assert torch.equal(fused, plain), f"M={M} two_shot={two}: fused differs from GEMM + allreduce"
        assert _same_everywhere(fused, tp.device_group), (M, two)
        ref = sum((As[r].float() @ Ws[r].float().t()) for r in range(world))
        err = (fused.float().cpu() - ref).abs()
        assert bool((err <= 2e-2 * ref.abs() + 2e-2 * ref.abs().max()).all()), (M, float(err.max()))
        xs = torch.empty(world, x.numel(), dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(xs, x, group=tp.device_group)
        acc = torch.zeros(x.numel(), dtype=torch.float32, device=dev)
        for r in range(world):  # the allreduce's rank order
            acc += xs[r].float()
        assert torch.equal(xr, acc.to(torch.bfloat16)), f"allreduce after fused call {i}"
    # N not a multiple of 256 (persistent tiles of 128 or fewer columns), odd M
    for j, (M, N) in enumerate([(777, 1536), (4096, 4096)]):
        K = 8192 // world
        As, Ws = _operands(M, K, N, world, 5000 + j)
        a, w = As[rank].to(dev), Ws[rank].to(dev)
        plain = ca.gemm_all_reduce(a, w)
        fused = ca.gemm_all_reduce(a, w, fused=True)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0, (M, N)
        assert torch.equal(fused, plain), (M, N)
    _graph_case(rank, world, dev, tp, ca)
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def _graph_case(rank, world, dev, tp, ca):
    from aiter_b200 import _lib
    from aiter_b200.dist import parallel_state as ps
    K, N = 8192 // world, 4096
    for M in (8, 1024):
        a_static = torch.zeros(M, K, dtype=torch.bfloat16, device=dev)
        w = torch.randn(N, K, generator=torch.Generator().manual_seed(9 + rank)).to(torch.bfloat16).to(dev)
        ca.gemm_all_reduce(a_static, w, fused=True)  # kernels loaded before capture
        torch.cuda.synchronize()
        with ps.graph_capture() as ctx:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=ctx.stream):
                z_static = ca.gemm_all_reduce(a_static, w, fused=True)
        for it in range(4):
            g_ = torch.Generator().manual_seed(900 + it + M)
            As = [torch.randn(M, K, generator=g_).to(torch.bfloat16) for _ in range(world)]
            a_static.copy_(As[rank].to(dev))
            g.replay()
            eager = ca.gemm_all_reduce(As[rank].to(dev), w)  # plain path after the replay
            torch.cuda.synchronize()
            assert _lib.lib().custom_ar_device_error(1) == 0
            assert torch.equal(z_static, eager), f"M={M} replay {it}"
        del g


def test_fused_gemm_allreduce_multi_gpu():
    world = min(torch.cuda.device_count(), 8)
    world = 2 if world < 4 else (4 if world < 8 else 8)
    run_ranks(_worker, world)
