"""Gated activations (test infrastructure only): the reference's silu_and_mul /
gelu_and_mul / gelu_tanh_and_mul / scaled_silu_and_mul
(csrc/kernels/activation_kernels.cu:24-160, 160-190 for the activation formulas,
337-360): input [..., 2d] = [x | y], out = act(x) * y computed in fp32 and rounded
once to the output type; the scaled form multiplies by 1 / scale and rounds to fp8
e4m3.  Computed here in float64 and rounded to fp32 first, so results may differ
from a device's fp32 transcendentals in the last fp32 bits (tests use tolerances).
"""
import math

import numpy as np

from .codecs import fp8_e4m3_encode, round_bf16

_ERF = np.vectorize(math.erf, otypes=[np.float64])


def act(x, kind):
    x = np.asarray(x, dtype=np.float64)
    if kind == "silu":
        return x / (1.0 + np.exp(-x))
    if kind == "gelu":
        return 0.5 * x * (1.0 + _ERF(x / math.sqrt(2.0)))
    if kind == "gelu_tanh":
        beta = math.sqrt(2.0 / math.pi)
        return 0.5 * x * (1.0 + np.tanh(beta * (x + 0.044715 * x ** 3)))
    raise ValueError(kind)


def round_out(v, dtype):
    v = np.asarray(v, dtype=np.float32)
    if dtype == "fp32":
        return v
    if dtype == "bf16":
        return round_bf16(v)
    if dtype == "fp16":
        return v.astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def act_and_mul(inp, kind, out_dtype):
    inp = np.asarray(inp, dtype=np.float32)
    d = inp.shape[-1] // 2
    x, y = inp[..., :d], inp[..., d:]
    return round_out((act(x, kind).astype(np.float32) * y).astype(np.float32), out_dtype)


def scaled_silu_and_mul(inp, scale):
    """fp8 e4m3 codes of silu(x) * y / scale (saturating at 448)."""
    inp = np.asarray(inp, dtype=np.float32)
    d = inp.shape[-1] // 2
    x, y = inp[..., :d], inp[..., d:]
    v = (act(x, "silu").astype(np.float32) * y * np.float32(1.0 / np.float32(scale))).astype(np.float32)
    return fp8_e4m3_encode(np.clip(v, -448.0, 448.0))
