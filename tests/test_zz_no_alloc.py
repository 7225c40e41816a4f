"""moe_sorting_fwd_static_scratch: the sorting entry point for callers that cannot
allocate device memory while running (a serving engine whose KV-cache pool took all
free HBM at start-up, a C host with no device allocator).  Its scratch is a 1 MiB
array built into the library instead of a caller-provided workspace.

The test calls it through the C ABI twice in a row, with different inputs that both
take the multi-CTA path (so the built-in array is really used and reused), and
checks every output bit-for-bit against the workspace-taking moe_sorting_fwd.  It
also checks that inputs needing more scratch than the array holds are rejected.
This file is collected last so that a run stopping at the first failure has already
run every other test; it passes alone in a fresh process as well."""
import numpy as np
import pytest
import torch

from aiter_b200 import _lib, moe_op
from gpu_util import dev, requires_cuda

pytestmark = [pytest.mark.gpu, requires_cuda]


def _buffers(M, k, E, B, D):
    rows = M * k + E * B - k
    return dict(
        sid=torch.full((rows,), -3, dtype=torch.int32, device=dev()),
        sw=torch.full((rows,), -3.0, dtype=torch.float32, device=dev()),
        seid=torch.full(((rows + B - 1) // B,), -3, dtype=torch.int32, device=dev()),
        nv=torch.full((2,), -3, dtype=torch.int32, device=dev()),
        buf=torch.full((M, D), 5.0, dtype=torch.bfloat16, device=dev()),
        pos=torch.full((M * k,), -3, dtype=torch.int32, device=dev()),
    )


def _run(M, E, k, B, D, seed, uses_scratch=True):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(M)]).to(torch.int32).to(dev())
    w = torch.rand(M, k, generator=g).to(dev())
    assert (moe_op.moe_sorting_get_workspace_size(M, E, k, 0) > 0) == uses_scratch
    ref = _buffers(M, k, E, B, D)
    moe_op.moe_sorting_fwd(ids, w, ref["sid"], ref["sw"], ref["seid"], ref["nv"], ref["buf"], E, B,
                           token_sorted_pos=ref["pos"])
    got = _buffers(M, k, E, B, D)
    _lib.call("moe_sorting_fwd_static_scratch", ids, w, got["sid"], got["sw"], got["seid"], got["nv"],
              got["buf"], E, B, None, None, 0, got["pos"])
    torch.cuda.synchronize()
    n = int(ref["nv"][0])
    assert torch.equal(got["nv"], ref["nv"])
    assert torch.equal(got["sid"][:n], ref["sid"][:n])
    assert torch.equal(got["sw"][:n].view(torch.int32), ref["sw"][:n].view(torch.int32))
    nb = n // B
    assert torch.equal(got["seid"][:nb], ref["seid"][:nb])
    assert torch.equal(got["pos"], ref["pos"])
    assert torch.count_nonzero(got["buf"]).item() == 0


def test_static_scratch_sort_matches_workspace_sort_twice_in_a_row():
    # the start-up call a caller makes before taking the free HBM: one token, one-CTA
    # sort; it places the library's array on the device
    _run(M=1, E=128, k=8, B=128, D=256, seed=0, uses_scratch=False)
    _run(M=4096, E=128, k=8, B=128, D=256, seed=1)      # 16 KiB of histograms
    _run(M=16384, E=256, k=8, B=128, D=128, seed=2)     # 128 KiB, reuses the array


def test_static_scratch_sort_rejects_oversized_inputs():
    M, E, k = 65536, 1024, 8                            # needs 2 MiB of histograms
    assert moe_op.moe_sorting_get_workspace_size(M, E, k, 0) > (1 << 20)
    ids = torch.zeros(M, k, dtype=torch.int32, device=dev())
    w = torch.zeros(M, k, device=dev())
    b = _buffers(1, k, E, 1, 8)
    with pytest.raises(RuntimeError, match="built-in array holds"):
        _lib.call("moe_sorting_fwd_static_scratch", ids, w, b["sid"], b["sw"], b["seid"], b["nv"], None, E, 1,
                  None, None, 0, None)
