"""Host logic of the tensor-parallel layer on CPU ranks (gloo, world size 2/3):
IPC handle exchange, the non-custom allreduce path, eligibility, unsupported world
sizes.  No GPU is touched."""
import os
import sys

import pytest
import torch
import torch.distributed as dist

from dist_util import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _init(rank, world, port):
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank)


def _exchange(rank, world, port):
    _init(rank, world, port)
    from aiter_b200.dist.custom_all_reduce import exchange_handles
    mine = bytes([rank]) * 64
    got = exchange_handles(dist.group.WORLD, mine)
    assert got == [bytes([r]) * 64 for r in range(world)]
    dist.destroy_process_group()


def test_ipc_handle_exchange_in_rank_order():
    run_ranks(_exchange, 2)


def _bad_handle(rank, world, port):
    _init(rank, world, port)
    from aiter_b200.dist.custom_all_reduce import exchange_handles
    try:
        exchange_handles(dist.group.WORLD, b"x" * (64 if rank == 0 else 10))
        raise AssertionError("a malformed handle must be rejected")
    except RuntimeError as e:
        assert "malformed" in str(e)
    dist.destroy_process_group()


def test_malformed_handle_rejected():
    run_ranks(_bad_handle, 2)


def _group_allreduce(rank, world, port):
    _init(rank, world, port)
    from aiter_b200.dist import parallel_state as ps
    tp = ps.initialize_model_parallel(world, local_rank=rank, backend="gloo", use_custom_allreduce=False)
    x = torch.full((4, 8), float(rank + 1))
    y = tp.all_reduce(x)
    assert torch.equal(y, torch.full((4, 8), float(sum(range(1, world + 1)))))
    assert torch.equal(x, torch.full((4, 8), float(rank + 1))), "all_reduce is out of place"
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_group_coordinator_allreduce_fallback_path():
    run_ranks(_group_allreduce, 2)


def _unsupported_world(rank, world, port):
    _init(rank, world, port)
    from aiter_b200.dist.custom_all_reduce import CustomAllreduce
    ca = CustomAllreduce(dist.group.WORLD, torch.device("cpu"))
    assert ca.disabled
    assert not ca.should_custom_ar(torch.zeros(8, dtype=torch.bfloat16))
    dist.destroy_process_group()


def test_custom_allreduce_disabled_for_unsupported_world_size():
    run_ranks(_unsupported_world, 3)


def test_nccl_group_rejected_for_handle_exchange():
    from aiter_b200.dist.custom_all_reduce import CustomAllreduce

    class G:
        pass

    orig = dist.get_backend
    try:
        dist.get_backend = lambda g=None: dist.Backend.NCCL
        with pytest.raises(AssertionError, match="non-NCCL"):
            CustomAllreduce(G(), 0)
    finally:
        dist.get_backend = orig
