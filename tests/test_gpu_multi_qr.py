"""Multi-GPU parity of the quick allreduce (qr_all_reduce), one process per GPU.
Skipped with fewer than 2 GPUs.

* every level (FP, FP8, INT6, INT4) for fp16, bf16 and bf16 with cast_bf2half: each
  rank's output bit-exact against the restatement of the reference's QuickReduce
  (oracle/quick_reduce.py), with a partial last tile, a message of one 16-byte pack
  and a message of several tiles per CTA; all ranks identical;
* the reference's variable-input loop (op_tests/multigpu_tests/test_quick_all_reduce.py:
  128-170): alternating shapes of zeros and ones reduce to exactly 0 and W;
* graph capture: a captured call replayed with fresh inputs, interleaved with eager
  calls of another size;
* the communicator front-end: GroupCoordinator.all_reduce takes the quick allreduce
  when AITER_QUICK_REDUCE_QUANTIZATION names a regime and the message lies in the B200
  crossover window of the world size, else the custom one.
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

MODES = [(torch.float16, False), (torch.bfloat16, False), (torch.bfloat16, True)]


def _inputs(n, world, seed, dtype, scale=1.0):
    out = []
    for r in range(world):
        g = torch.Generator().manual_seed(seed * 100 + r)
        x = torch.randn(n, generator=g) * scale
        if n >= 256:  # an all-zero group, a tiny group and a tied group
            x[64:128] = 0
            x[128:192] = 1e-6
            x[192:256:2] = 3.0
            x[193:256:2] = -3.0
        out.append(x.to(dtype))
    return out


def _want(xs, level, dtype, cast):
    from oracle.quick_reduce import quick_allreduce
    name = "fp16" if dtype == torch.float16 else "bf16"
    return quick_allreduce([x.float().numpy() for x in xs], level, name, cast)


def _worker(rank, world, port):
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["AITER_QUICK_REDUCE_QUANTIZATION"] = "INT4"
    os.environ["AITER_QUICK_REDUCE_MAX_SIZE_BYTES_MB"] = "64"
    torch.cuda.set_device(rank)
    import aiter_b200 as aiter
    from aiter_b200.dist import parallel_state as ps
    ps.init_distributed_environment(world, rank, f"tcp://127.0.0.1:{port}", rank, "nccl", timeout_s=60)
    tp = ps.initialize_model_parallel(world, local_rank=rank, ca_max_size=16 * 1024 * 1024)
    qr = tp.qr_comm
    assert qr is not None and not qr.disabled
    dev = torch.device("cuda", rank)
    fa = qr._ptr
    cases = [(level, dtype, cast, n) for level in range(4) for dtype, cast in MODES
             for n in (8, 16384 + 8 * 9, 3 * 16384)]
    # more tiles than CTAs (every CTA loops), codec-independent: two cheap oracle cases
    big = 16384 * 600 + 64
    cases += [(3, torch.float16, False, big), (0, torch.bfloat16, False, big)]
    for i, (level, dtype, cast, n) in enumerate(cases):
        xs = _inputs(n, world, 7 * level + i, dtype, scale=(1.0, 1e-3, 300.0)[i % 3])
        inp = xs[rank].to(dev)
        out = torch.empty_like(inp)
        aiter.qr_all_reduce(fa, inp, out, level, cast)
        torch.cuda.synchronize()
        assert aiter.qr_device_error() == 0
        allo = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(allo, out, group=tp.device_group)
        assert all(torch.equal(o.view(torch.int16), out.view(torch.int16)) for o in allo)
        if rank == 0:  # identical on every rank: one rank checks the oracle
            got = out.float().cpu().numpy()
            bad = int((got != _want(xs, level, dtype, cast)).sum())
            assert bad == 0, (level, dtype, cast, n, bad)
        dist.barrier(group=tp.cpu_group)
    # the reference's variable-input loop (shortened)
    for it in range(2000):
        s2 = 1024 if it % 2 == 0 else 2048
        inp = (torch.zeros if it % 2 == 0 else torch.ones)((1024, s2), dtype=torch.float16, device=dev)
        res = torch.empty_like(inp)
        aiter.qr_all_reduce(fa, inp, res, 3, True)
        if it % 250 == 0 or it >= 1998:
            torch.cuda.synchronize()
            assert torch.all(res == (0 if it % 2 == 0 else world)), it
    assert aiter.qr_device_error() == 0
    # graph capture, replays interleaved with eager calls of another size
    n = 16384 * 40
    static_in = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    static_out = torch.empty_like(static_in)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        aiter.qr_all_reduce(fa, static_in, static_out, 2, False)  # warm-up outside capture
        with torch.cuda.graph(g, stream=s):
            aiter.qr_all_reduce(fa, static_in, static_out, 2, False)
    torch.cuda.current_stream(dev).wait_stream(s)
    for rep in range(4):
        xs = _inputs(n, world, 900 + rep, torch.bfloat16)
        static_in.copy_(xs[rank].to(dev))
        g.replay()
        ys = _inputs(5000 * 8, world, 950 + rep, torch.float16)
        e_out = torch.empty(5000 * 8, dtype=torch.float16, device=dev)
        aiter.qr_all_reduce(fa, ys[rank].to(dev), e_out, 1, False)
        torch.cuda.synchronize()
        assert aiter.qr_device_error() == 0
        assert np.array_equal(static_out.float().cpu().numpy(), _want(xs, 2, torch.bfloat16, False)), rep
        assert np.array_equal(e_out.float().cpu().numpy(), _want(ys, 1, torch.float16, False)), rep
    del g
    # front-end: with no crossover window for this world size the message stays on the
    # custom allreduce (fp32 rank-order sum rounded once); inside a window, an fp16
    # message takes the quick allreduce
    from aiter_b200.dist import quick_all_reduce as qmod
    n = (8 * 1024 * 1024) // 2
    xs = _inputs(n, world, 77, torch.float16)
    saved = dict(qmod.B200_WINDOWS)
    try:
        qmod.B200_WINDOWS.pop((world, "INT4"), None)
        y = tp.all_reduce(xs[rank].to(dev))
        torch.cuda.synchronize()
        exact = torch.zeros(n, dtype=torch.float32)
        for t in xs:
            exact += t.float()
        assert torch.equal(y.cpu(), exact.to(torch.float16))
        qmod.B200_WINDOWS[(world, "INT4")] = (1024 * 1024, 64 * 1024 * 1024)
        y = tp.all_reduce(xs[rank].to(dev))
        torch.cuda.synchronize()
        assert np.array_equal(y.float().cpu().numpy(), _want(xs, 3, torch.float16, True))
    finally:
        qmod.B200_WINDOWS.clear()
        qmod.B200_WINDOWS.update(saved)
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_quick_allreduce_multi_gpu():
    world = min(torch.cuda.device_count(), 8)
    world = 2 if world < 4 else (4 if world < 8 else 8)
    run_ranks(_worker, world)
