"""Gated activations, the reference's aiter.silu_and_mul / gelu_and_mul /
gelu_tanh_and_mul / scaled_silu_and_mul (aiter/ops/activation.py:10-23), which its
fused_moe uses after a split-K stage 1 (aiter/fused_moe.py:1719-1724).

input [..., 2d] holds [x | y]; out [..., d] = act(x) * y, computed in fp32 and rounded
once.  fp32 input may write fp32, bf16 or fp16; bf16 / fp16 input writes its own type.
scaled_silu_and_mul writes fp8 e4m3 of act(x) * y / scale (scale: f32 tensor of one
value, read on the device).
"""
from torch import Tensor

from . import _lib


def silu_and_mul(out: Tensor, input: Tensor) -> None:
    _lib.call("silu_and_mul", out, input)


def gelu_and_mul(out: Tensor, input: Tensor) -> None:
    _lib.call("gelu_and_mul", out, input)


def gelu_tanh_and_mul(out: Tensor, input: Tensor) -> None:
    _lib.call("gelu_tanh_and_mul", out, input)


def scaled_silu_and_mul(out: Tensor, input: Tensor, scale: Tensor) -> None:
    _lib.call("scaled_silu_and_mul", out, input, scale)
