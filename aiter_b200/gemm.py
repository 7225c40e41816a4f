"""bf16 GEMM front (the GEMM half of GEMM + allreduce; aiter/tuned_gemm.py)."""
from typing import Optional

import torch

from . import _lib


def gemm_a16w16(A: torch.Tensor, W: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = A @ W^T (A [M, K], W [N, K], bf16) on the tcgen05 kernel of libaiter_b200.so."""
    if out is None:
        out = torch.empty((A.shape[0], W.shape[0]), dtype=torch.bfloat16, device=A.device)
    _lib.call("gemm_a16w16", A, W, out)
    return out


class TunedGemm:
    """`tgemm.mm(inp, weights)` (aiter/tuned_gemm.py:506-529) for bf16 without bias."""

    def mm(self, inp, weights, bias=None, otype=None, scale_a=None, scale_b=None, scale_c=None):
        if bias is not None or scale_a is not None or scale_b is not None:
            raise NotImplementedError("bias / scaled variants are not part of this path")
        if otype not in (None, torch.bfloat16):
            raise NotImplementedError("bf16 output only")
        shp = inp.shape
        out = gemm_a16w16(inp.reshape(-1, shp[-1]).contiguous(), weights.contiguous())
        return out.view(*shp[:-1], weights.shape[0])


tgemm = TunedGemm()
