"""Single-GPU parity of the EP dispatch / combine kernels: all W ranks emulated as
CTA rows of cooperative launches (ep_emu_*), every rank's received arrays and
combined outputs bit-exact against oracle/ep.py."""
import numpy as np
import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU"),
]


def _inputs(world, T, H, k, E, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]) for _ in range(world)])
    ids = ids.to(torch.int32)
    if T > 3:
        ids[:, 3] = -1                        # goes nowhere
    tokens = torch.randn(world, T, H, generator=g).to(dtype)
    weights = torch.rand(world, T, k, generator=g)
    scales = torch.rand(world, T, H // 128, generator=g) if dtype == torch.float8_e4m3fn else None
    return tokens, weights, scales, ids


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 32, 8), (8, 64, 8)])
@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.bfloat16])
@pytest.mark.parametrize("T,max_tokens", [(1, 1), (37, 64), (1500, 1500)])
def test_ep_dispatch_combine_emulated(world, E, k, dtype, T, max_tokens):
    from aiter_b200.dist.ep import emulated_dispatch_combine
    from oracle import ep
    from oracle.codecs import round_bf16
    H = 512
    tokens, weights, scales, ids = _inputs(world, T, H, k, E, seed=world * 1000 + T, dtype=dtype)
    dev = torch.device("cuda", 0)

    def expert(rank, rt, rs, rids, rw, n):
        out = torch.zeros(world * max_tokens, H, dtype=torch.bfloat16, device=dev)
        out[:n] = (rt[:n].float() * (rank + 1)).to(torch.bfloat16)
        return out

    y, recv = emulated_dispatch_combine(tokens.to(dev), weights.to(dev), scales.to(dev) if scales is not None else None,
                                        ids.to(dev), E // world, expert, max_tokens=max_tokens)
    torch.cuda.synchronize()
    from aiter_b200 import _lib
    assert _lib.lib().ep_device_error(1) == 0
    per_rank = [{"tokens": tokens[r].float().numpy(), "weights": weights[r].numpy(), "ids": ids[r].numpy(),
                 **({"scales": scales[r].numpy()} if scales is not None else {})} for r in range(world)]
    want = ep.dispatch(per_rank, E // world, world)
    for d in range(world):
        n = recv[d]["recv_num"]
        assert n == len(want[d]["src"]), (d, n)
        tags = recv[d]["src"].cpu().numpy()
        assert [(int(t) >> 24, int(t) & 0xFFFFFF) for t in tags] == want[d]["src"]
        if n:
            assert np.array_equal(recv[d]["tokens"].float().cpu().numpy(), np.stack(want[d]["tokens"]))
            assert np.array_equal(recv[d]["ids"].cpu().numpy(), np.stack(want[d]["ids"]))
            assert np.array_equal(recv[d]["weights"].cpu().numpy(), np.stack(want[d]["weights"]))
            if scales is not None:
                assert np.array_equal(recv[d]["scales"].cpu().numpy(), np.stack(want[d]["scales"]))
    outs = [round_bf16(np.stack(want[d]["tokens"]).astype(np.float32) * (d + 1)) if want[d]["src"]
            else np.zeros((0, H), np.float32) for d in range(world)]
    ycomb = ep.combine(outs, want, [T] * world, round_bf16)
    for s in range(world):
        assert np.array_equal(y[s].float().cpu().numpy(), ycomb[s]), s
