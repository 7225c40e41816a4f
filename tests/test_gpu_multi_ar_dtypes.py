"""Multi-GPU parity of the IPC allreduce for fp16 and fp32 and of the fp8-quantised
allreduce (custom_ar_all_reduce_fp8), one process per GPU.  Skipped with fewer than
2 GPUs.

* fp16 / fp32: bit-exact against the fp32 rank-order sum (oracle), one- and two-shot;
* fused allreduce + RMSNorm (+ fp8 quant): the two-shot form returns the one-shot bits;
* open_fp8_quant with fp16: every rank's output bit-exact against the restatement of
  the reference's allReduceQuantFp8 (oracle/allreduce.py), including group sizes
  below 128 and a message whose pack count leaves a remainder for the last rank;
  bf16 and small fp16 messages ignore the flag (plain allreduce bits);
* IPC all-gather along dim 0 and the last dim (exact concatenation) and reduce-scatter
  (this rank's share of the rank-ordered fp32 sum, the allreduce's bits).
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def _inputs(n, world, seed, dtype):
    out = []
    for r in range(world):
        g = torch.Generator().manual_seed(seed * 100 + r)
        out.append(torch.randn(n, generator=g).to(dtype))
    return out


def _worker(rank, world, port):
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from aiter_b200 import _lib
    from aiter_b200.dist import parallel_state as ps
    from oracle.allreduce import allreduce_fp8_quant, allreduce_rank_order
    ps.init_distributed_environment(world, rank, f"tcp://127.0.0.1:{port}", rank, "nccl", timeout_s=60)
    tp = ps.initialize_model_parallel(world, local_rank=rank, ca_max_size=64 * 1024 * 1024)
    ca = tp.ca_comm
    dev = torch.device("cuda", rank)
    for i, (dtype, n, two) in enumerate([(torch.float16, 4096, None), (torch.float16, 1 << 20, True),
                                         (torch.float32, 4096, False), (torch.float32, 3 << 18, True),
                                         (torch.float16, 8, None), (torch.float32, 4, None)]):
        xs = _inputs(n, world, 10 + i, dtype)
        y = ca.all_reduce(xs[rank].to(dev), two_shot=two)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0
        want = allreduce_rank_order([x.numpy() for x in xs], xs[0].numpy().dtype)
        assert np.array_equal(y.cpu().numpy(), want), (dtype, n, two)
    # open_fp8_quant: 128-element groups; 64-element groups; a pack remainder
    npd = np.float16
    for j, n in enumerate([128 * 2048, 128 * 2048 * 3, world * 64 * 4097, 128 * 2048 + 8 * 3]):
        xs = _inputs(n, world, 50 + j, torch.float16)
        y = tp.all_reduce(xs[rank].to(dev), ca_fp8_quant=True)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0
        want = allreduce_fp8_quant([x.numpy() for x in xs])[rank]
        got = y.cpu().numpy()
        assert got.dtype == npd and np.array_equal(got, want), (n, int((got != want).sum()))
    # fused allreduce + residual + RMSNorm: two-shot (owner ranks reduce the rows, every
    # rank normalises locally) returns the one-shot kernel's bits
    for rows, hidden in ((1024, 4096), (333, 7168), (8, 16384)):
        g = torch.Generator().manual_seed(rows)
        xs = [torch.randn(rows, hidden, generator=g).to(torch.bfloat16) for _ in range(world)]
        res = torch.randn(rows, hidden, generator=g).to(torch.bfloat16).to(dev)
        wt = (torch.rand(hidden, generator=g) + 0.5).to(torch.bfloat16).to(dev)
        x = xs[rank].to(dev)
        o1, r1 = ca.fused_ar_rms(x, res, w=wt, eps=1e-6)
        o2, r2 = ca.fused_ar_rms(x, res, w=wt, eps=1e-6, two_shot=True)
        q1, _, s1 = ca.fused_ar_rms(x, res, w=wt, eps=1e-6, post_per_token_quant=True)
        q2, _, s2 = ca.fused_ar_rms(x, res, w=wt, eps=1e-6, post_per_token_quant=True, two_shot=True)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0
        assert torch.equal(r1, r2) and torch.equal(o1, o2), (rows, hidden)
        assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2), (rows, hidden)
    # the flag is ignored for bf16 and for fp16 below 128 * 2048 elements
    for dtype, n in ((torch.bfloat16, 128 * 2048), (torch.float16, 4096)):
        xs = _inputs(n, world, 70, dtype)
        y = tp.all_reduce(xs[rank].to(dev), ca_fp8_quant=True)
        z = ca.all_reduce(xs[rank].to(dev))
        torch.cuda.synchronize()
        assert torch.equal(y, z), (dtype, n)
    # IPC all-gather (dim 0 and last dim) and reduce-scatter
    for i, (dtype, shape) in enumerate([(torch.bfloat16, (64, 512)), (torch.float32, (3, 1024)),
                                        (torch.float16, (1, 8))]):
        xs = [t.reshape(shape) for t in _inputs(int(np.prod(shape)), world, 80 + i, dtype)]
        x = xs[rank].to(dev)
        g0 = ca.custom_all_gather(x, 0)
        gl = ca.custom_all_gather(x, -1)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0
        assert torch.equal(g0.cpu(), torch.cat(xs, dim=0)), (dtype, shape)
        if (shape[-1] * x.element_size()) % 16 == 0:
            assert torch.equal(gl.cpu(), torch.cat(xs, dim=-1)), (dtype, shape)
        assert torch.equal(tp.all_gather(x, use_custom=True, dim=0).cpu(), torch.cat(xs, dim=0))
    for i, (dtype, n) in enumerate([(torch.bfloat16, world * 4096), (torch.float32, world * 1000),
                                    (torch.float16, world * 8)]):
        xs = _inputs(n, world, 90 + i, dtype)
        x = xs[rank].to(dev)
        out = torch.empty(n // world, dtype=dtype, device=dev)
        assert ca.custom_reduce_scatter(x, out)
        full = ca.all_reduce(x)
        torch.cuda.synchronize()
        assert _lib.lib().custom_ar_device_error(1) == 0
        acc = torch.zeros(n, dtype=torch.float32)   # fp32 sum in rank order, rounded once
        for t in xs:
            acc += t.float()
        want = acc.to(dtype)
        seg = n // world
        assert torch.equal(out.cpu(), want[rank * seg:(rank + 1) * seg]), (dtype, n)
        assert torch.equal(out, full.reshape(-1)[rank * seg:(rank + 1) * seg])
        rs = tp.reduce_scatter_tensor(x.reshape(world, -1))
        assert torch.equal(rs.reshape(-1), out)
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_allreduce_dtypes_and_fp8_quant_multi_gpu():
    world = min(torch.cuda.device_count(), 8)
    world = 2 if world < 4 else (4 if world < 8 else 8)
    run_ranks(_worker, world)
