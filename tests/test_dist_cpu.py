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


def _group_fused_rmsnorm(rank, world, port):
    """fused_allreduce_rmsnorm(_quant) through the non-custom path: allreduce, then
    x = ar + residual (fp32), residual_out = bf16(x), out = x * w * rsqrt(mean x^2 + eps)."""
    _init(rank, world, port)
    from aiter_b200.dist import parallel_state as ps
    from aiter_b200.dist import (tensor_model_parallel_fused_allreduce_rmsnorm,
                                 tensor_model_parallel_fused_allreduce_rmsnorm_quant)
    ps.initialize_model_parallel(world, local_rank=rank, backend="gloo", use_custom_allreduce=False)
    g = torch.Generator().manual_seed(3)
    xs = [torch.randn(5, 64, generator=g).to(torch.bfloat16) for _ in range(world)]
    res = torch.randn(5, 64, generator=g).to(torch.bfloat16)
    w = (torch.rand(64, generator=g) + 0.5).to(torch.bfloat16)
    out, res_out = tensor_model_parallel_fused_allreduce_rmsnorm(xs[rank].clone(), res, w, 1e-6)
    ar = sum(x.float() for x in xs).to(torch.bfloat16)  # gloo sums bf16 in rank order too
    x = ar.float() + res.float()
    assert torch.equal(res_out, x.to(torch.bfloat16))
    ref = x * w.float() / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(out.float(), ref, rtol=1e-2, atol=1e-2)
    q, res_out2, scale = tensor_model_parallel_fused_allreduce_rmsnorm_quant(xs[rank].clone(), res, w, 1e-6)
    assert q.dtype == torch.float8_e4m3fn and scale.shape == (5, 1) and torch.equal(res_out2, res_out)
    assert torch.allclose(q.float() * scale, ref, rtol=0.07, atol=0.02 * float(ref.abs().max()))
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_group_coordinator_fused_allreduce_rmsnorm_fallback_path():
    run_ranks(_group_fused_rmsnorm, 2)


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


def _group_collectives(rank, world, port):
    """all_gather (dim 0, last, middle), reduce_scatter_tensor (divisible and flat),
    gather and the front-ends, on the non-custom path."""
    _init(rank, world, port)
    from aiter_b200.dist import communication_op as co
    from aiter_b200.dist import parallel_state as ps
    ps.initialize_model_parallel(world, local_rank=rank, backend="gloo", use_custom_allreduce=False)
    x = torch.arange(24, dtype=torch.float32).reshape(2, 3, 4) + 100 * rank
    parts = [torch.arange(24, dtype=torch.float32).reshape(2, 3, 4) + 100 * r for r in range(world)]
    for dim in (0, 1, -1):
        got = co.tensor_model_parallel_all_gather(x, dim=dim)
        assert torch.equal(got, torch.cat(parts, dim=dim)), dim
    assert torch.equal(co.tensor_model_parallel_custom_all_gather(x), torch.cat(parts, dim=0))
    y = torch.arange(12, dtype=torch.float32).reshape(4, 3) * (rank + 1)
    total = sum(torch.arange(12, dtype=torch.float32).reshape(4, 3) * (r + 1) for r in range(world))
    rs = co.tensor_model_parallel_reduce_scatter(y)
    assert rs.shape == (4 // world, 3) and torch.equal(rs, total.chunk(world, dim=0)[rank])
    z = torch.arange(6, dtype=torch.float32).reshape(3, 2) * (rank + 1)   # 3 rows: flat shares
    ztot = sum(torch.arange(6, dtype=torch.float32).reshape(3, 2) * (r + 1) for r in range(world)).reshape(-1)
    rz = co.tensor_model_parallel_reduce_scatter(z)
    assert rz.shape == (6 // world,) and torch.equal(rz, ztot.chunk(world)[rank])
    g = co.tensor_model_parallel_gather(x, dst=0, dim=0)
    assert (torch.equal(g, torch.cat(parts, dim=0)) if rank == 0 else g is None)
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_group_coordinator_collectives_fallback_path():
    run_ranks(_group_collectives, 2)


def _group_layout(rank, world, port, tp):
    """TP groups of consecutive ranks (TP fastest, as the reference's layout,
    parallel_state.py:1181-1264), the EP group equal to the TP group without data
    parallelism, the EP front-ends; pipeline / data-parallel sizes above 1 rejected."""
    _init(rank, world, port)
    from aiter_b200.dist import communication_op as co
    from aiter_b200.dist import parallel_state as ps
    for bad in (dict(pipeline_model_parallel_size=2), dict(data_parallel_size=2)):
        with pytest.raises(NotImplementedError, match="outside this library"):
            ps.initialize_model_parallel(tp, backend="gloo", local_rank=rank, use_custom_allreduce=False, **bad)
    ps.initialize_model_parallel(tp, 1, "gloo", 1, local_rank=rank, use_custom_allreduce=False)
    first = rank // tp * tp
    assert ps.get_tp_group().ranks == list(range(first, first + tp))
    assert ps.get_ep_group().ranks == ps.get_tp_group().ranks
    assert ps.get_tensor_model_parallel_world_size() == tp and ps.get_tensor_model_parallel_rank() == rank - first
    x = torch.full((2, 4), float(rank + 1))
    ep_sum = float(sum(r + 1 for r in ps.get_ep_group().ranks))
    assert torch.equal(co.expert_parallel_all_reduce(x), torch.full((2, 4), ep_sum))
    g = co.expert_parallel_all_gather(x, dim=0)
    assert torch.equal(g[:, 0], torch.tensor([float(r + 1) for r in ps.get_ep_group().ranks]).repeat_interleave(2))
    b = co.expert_parallel_broadcast(torch.full((3,), float(rank)), src=1)
    assert torch.equal(b, torch.full((3,), float(ps.get_ep_group().ranks[1])))
    ps.destroy_model_parallel()
    dist.destroy_process_group()


@pytest.mark.parametrize("tp", [2, 4])
def test_model_parallel_group_layout(tp):
    run_ranks(_group_layout, 4, tp)


def _group_ranks_and_barrier(rank, world, port):
    """End ranks, the keyword names of all_reduce, object broadcast and the barrier
    (parallel_state.py:310-327, 376-383, 928-935)."""
    _init(rank, world, port)
    from aiter_b200.dist import parallel_state as ps
    tp = ps.initialize_model_parallel(world, local_rank=rank, backend="gloo", use_custom_allreduce=False)
    assert tp.first_rank == 0 and tp.last_rank == world - 1
    assert tp.is_first_rank == (rank == 0) and tp.is_last_rank == (rank == world - 1)
    y = tp.all_reduce(torch.full((3,), float(rank)), ca_use_new=True, ca_fp8_quant=False)
    assert torch.equal(y, torch.full((3,), float(sum(range(world)))))
    assert tp.broadcast_object({"k": rank} if rank == 1 else None, src=1) == {"k": 1}
    tp.barrier()
    assert tp.prepare_communication_buffer_for_model(torch.nn.Linear(2, 2)) is None
    ps.destroy_model_parallel()
    dist.destroy_process_group()


def test_group_coordinator_ranks_objects_barrier():
    run_ranks(_group_ranks_and_barrier, 2)


def test_custom_allreduce_gather_scatter_eligibility_and_shapes():
    """The reference CustomAllreduce's host-side helpers (custom_all_reduce.py:405-553)
    on an object with no IPC context: registration is a no-op, all-gather eligibility
    and output shapes, reduce-scatter eligibility."""
    from aiter_b200.dist.custom_all_reduce import CustomAllreduce
    ca = CustomAllreduce.__new__(CustomAllreduce)
    ca.disabled, ca.world_size, ca.max_size, ca.device = False, 4, 1 << 20, torch.device("cpu")
    x = torch.empty(8, 64, dtype=torch.bfloat16)
    assert ca.register_input_buffer(x) is None and ca.register_output_buffer(x) is None
    assert ca.register_graph_buffers() is None
    assert ca.should_custom_ag(x) and ca.should_custom_ag(x, -1)
    assert ca.should_custom_ag(x, 1)                        # dim 1 is the last dim of a 2-D tensor
    assert ca.should_custom_ag(torch.empty(8, 64, 2, dtype=torch.bfloat16), 0)
    assert not ca.should_custom_ag(torch.empty(8, 64, 2, dtype=torch.bfloat16), 1)   # middle dim
    assert not ca.should_custom_ag(torch.empty(8, 3, dtype=torch.bfloat16), -1)       # 6-byte rows
    assert not ca.should_custom_ag(torch.empty(8, 64, dtype=torch.bfloat16)[:, :32])  # not contiguous
    assert not ca.should_custom_ag(torch.empty(1 << 20, dtype=torch.bfloat16))         # above max_size
    assert ca._allgather_out_shape(x, 0) == (32, 64) and ca._allgather_out_shape(x, -1) == (8, 256)
    assert ca._allgather_out_shape(torch.empty(2, 3, 4), 1) == (96,)
    assert ca._rs_eligible(torch.empty(8, 64, dtype=torch.bfloat16))
    assert not ca._rs_eligible(torch.empty(3, 8, dtype=torch.bfloat16))               # 12-byte shares
    assert not ca._rs_eligible(torch.empty(8, 64, dtype=torch.int32))                 # dtype
    ca.disabled = True
    assert not ca.should_custom_ag(x) and ca.custom_all_gather(x) is None
    assert ca.custom_reduce_scatter(x, torch.empty(2, 64, dtype=torch.bfloat16)) is False


def _world_and_helpers(rank, world, port):
    """init_distributed_environment's world group and the module helpers of
    parallel_state (parallel_state.py:985-1017, 1082-1145, 1320-1544) on gloo ranks."""
    sys.path.insert(0, ROOT)
    from aiter_b200.dist import parallel_state as ps
    ps.init_distributed_environment(world, rank, f"tcp://127.0.0.1:{port}", rank, "gloo", timeout_s=60)
    wg = ps.get_world_group()
    assert wg.ranks == list(range(world)) and wg.rank_in_group == rank and wg.ca_comm is None
    assert ps.is_global_first_rank() == (rank == 0)
    assert ps.in_the_same_node_as(wg.cpu_group, source_rank=0) == [True] * world
    ps.set_custom_all_reduce(False)
    g = ps.init_model_parallel_group([[0], [1]], rank, "gloo", group_name="solo")
    assert g.ranks == [rank] and g.unique_name == "solo" and g.ca_comm is None
    tp = ps.initialize_model_parallel(world, local_rank=rank, backend="gloo")
    assert tp.ca_comm is None
    with ps.patch_tensor_parallel_group(g):
        assert ps.get_tp_group() is g and ps.get_tensor_model_parallel_world_size() == 1
    assert ps.get_tp_group() is tp
    ps.prepare_communication_buffer_for_model(torch.nn.Linear(2, 2))
    ps.set_custom_all_reduce(True)
    ps.destroy_distributed_environment()
    assert not dist.is_initialized()


def test_world_group_and_parallel_state_helpers():
    run_ranks(_world_and_helpers, 2)
