"""CPU checks of the EP dispatch / combine oracle (oracle/ep.py) and of the Python
front-end's configuration handling (aiter_b200/dist/ep.py), against what the
reference's dispatch/combine test fixes (op_tests/multigpu_tests/
test_dispatch_combine.py:17-62, 76-171): every token reaches each rank owning one of
its experts exactly once, and combine returns the sum over ranks of the per-rank
expert outputs."""
import numpy as np
import pytest
import torch

from oracle import ep
from oracle.codecs import round_bf16


def _rank_inputs(world, T, H, k, E, seed):
    rng = np.random.default_rng(seed)
    out = []
    for r in range(world):
        ids = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
        if T > 3:
            ids[3] = -1              # a token that goes nowhere
        out.append({"tokens": rng.standard_normal((T, H)).astype(np.float32),
                    "weights": rng.random((T, k)).astype(np.float32), "ids": ids,
                    "scales": rng.random((T, H // 128)).astype(np.float32)})
    return out


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 16, 4), (8, 64, 8)])
def test_dispatch_delivers_each_token_once_per_owner(world, E, k):
    T, H = 37, 256
    inp = _rank_inputs(world, T, H, k, E, seed=world)
    recv = ep.dispatch(inp, E // world, world)
    for d in range(world):
        src = recv[d]["src"]
        assert src == sorted(src)                       # source rank, then token order
        want = [(s, t) for s in range(world) for t in range(T)
                if d in ep.destinations(inp[s]["ids"][t], E // world, world)]
        assert src == want
        for i, (s, t) in enumerate(src):
            assert np.array_equal(recv[d]["tokens"][i], inp[s]["tokens"][t])
            assert np.array_equal(recv[d]["ids"][i], inp[s]["ids"][t])
            assert np.array_equal(recv[d]["scales"][i], inp[s]["scales"][t])
    # the token whose ids are all out of range reaches nobody
    assert all((s, 3) not in recv[d]["src"] for d in range(world) for s in range(world))


def test_combine_sums_over_owner_ranks():
    world, E, k, T, H = 4, 16, 4, 20, 128
    inp = _rank_inputs(world, T, H, k, E, seed=7)
    recv = ep.dispatch(inp, E // world, world)
    # expert stand-in: rank d scales its received rows by d + 1
    outs = [np.asarray(recv[d]["tokens"], dtype=np.float32).reshape(-1, H) * (d + 1) for d in range(world)]
    y = ep.combine(outs, recv, [T] * world, round_bf16)
    for s in range(world):
        for t in range(T):
            dests = ep.destinations(inp[s]["ids"][t], E // world, world)
            want = np.zeros(H, np.float32)
            for d in dests:
                want += inp[s]["tokens"][t] * (d + 1)
            assert np.array_equal(y[s][t], round_bf16(want))


def test_config_validation():
    from aiter_b200.dist.ep import EpDispatchCombineConfig, _check_config
    good = dict(data_type=torch.float8_e4m3fn, rank=0, world_size=8, hidden_dim=7168, scale_dim=56,
                scale_type_size=4, max_token_type_size=2, max_num_inp_token_per_rank=4096,
                num_experts_per_rank=32, num_experts_per_token=8)
    _check_config(EpDispatchCombineConfig(**good))
    for bad in (dict(data_type=torch.float32), dict(scale_type_size=2), dict(world_size=16),
                dict(out_dtype=torch.float32)):
        with pytest.raises(ValueError):
            _check_config(EpDispatchCombineConfig(**{**good, **bad}))


def test_all2all_kwargs_mapping():
    from aiter_b200.dist.ep import EpAll2AllManager
    m = object.__new__(EpAll2AllManager)
    kw = m._make_all2all_kwargs(rank=1, num_ep_ranks=8, input_dtype=torch.bfloat16, quant_dtype=torch.float8_e4m3fn,
                                token_hidden_size=7168, scale_dim=56, scale_type_size=4,
                                max_num_tokens_per_dp_rank=1024, num_local_experts=32, num_experts_per_token=8,
                                gpu_per_node=8)
    assert kw["world_size"] == 8 and kw["data_type"] == torch.float8_e4m3fn and kw["max_token_type_size"] == 2
    assert kw["num_experts_per_rank"] == 32 and kw["max_num_inp_token_per_rank"] == 1024
