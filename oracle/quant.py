"""Quantisers restated in numpy (test infrastructure only).

* `per_1x128_quant`   -- `pertoken_quant` over 128-wide groups
                         (aiter/ops/quant.py:42-72 via per_block_quant_wrapper :152-170):
                         scale = amax / 448 (0 -> 1), q = fp8(x / scale).
* `per_group_quant_i8` -- the same with int8 output: scale = amax / 127 (0 -> 1),
                         q = x / scale truncated toward zero (torch's float -> int8).
* `weight_128x128_quant` -- the 128x128 block quantiser of
                         op_tests/test_moe_2stage.py:84-110.
* `per_1x32_f4_quant` -- MXFP4 with e8m0 scales (aiter/ops/quant.py:75-106):
                         scale = e8m0(amax / 4), q = e2m1(x / scale).
"""
import numpy as np

from . import codecs

F32 = np.float32


def per_1x128_quant(x, group=128):
    """x: [..., K] float -> (codes uint8 [..., K], scale f32 [..., K/group])."""
    x = np.asarray(x, dtype=F32)
    shp = x.shape
    g = x.reshape(-1, group)
    amax = np.abs(g).max(axis=-1, keepdims=True)
    scale = (amax / F32(codecs.FP8_E4M3_MAX)).astype(F32)
    scale[scale == 0] = F32(1.0)
    y = (g / scale).astype(F32)
    q = codecs.fp8_e4m3_encode(y).reshape(shp)
    return q, scale.reshape(shp[:-1] + (shp[-1] // group,))


def per_group_quant_i8(x, group=128):
    """pertoken_quant(quant_dtype=int8) over `group`-wide groups (aiter/ops/quant.py:42-72):
    x: [..., K] float -> (int8 [..., K], scale f32 [..., K/group])."""
    x = np.asarray(x, dtype=F32)
    shp = x.shape
    g = x.reshape(-1, group)
    amax = np.abs(g).max(axis=-1, keepdims=True)
    scale = (amax / F32(127.0)).astype(F32)
    scale[scale == 0] = F32(1.0)
    y = (g / scale).astype(F32)
    q = np.trunc(y).astype(np.int8).reshape(shp)
    return q, scale.reshape(shp[:-1] + (shp[-1] // group,))


def dequant_1x128(q, scale, group=128):
    v = codecs.fp8_e4m3_decode(q)
    shp = v.shape
    return (v.reshape(-1, group) * np.asarray(scale, dtype=F32).reshape(-1, 1)).reshape(shp).astype(F32)


def weight_128x128_quant(w):
    """w: [E, N, K] -> (codes [E,N,K], scale f32 [E, N/128, K/128])."""
    w = np.asarray(w, dtype=F32)
    E, N, K = w.shape
    blk = w.reshape(E, N // 128, 128, K // 128, 128).transpose(0, 1, 3, 2, 4).reshape(E, -1, 128 * 128)
    amax = np.abs(blk).max(axis=-1, keepdims=True)
    scale = (amax / F32(codecs.FP8_E4M3_MAX)).astype(F32)
    scale[scale == 0] = F32(1.0)
    q = codecs.fp8_e4m3_encode((blk / scale).astype(F32))
    q = q.reshape(E, N // 128, K // 128, 128, 128).transpose(0, 1, 3, 2, 4).reshape(E, N, K)
    return q, scale.reshape(E, N // 128, K // 128)


def dequant_128x128(q, scale):
    v = codecs.fp8_e4m3_decode(q)
    E, N, K = v.shape
    s = np.asarray(scale, dtype=F32)
    return (v.reshape(E, N // 128, 128, K // 128, 128) * s[:, :, None, :, None]).reshape(E, N, K).astype(F32)


def per_1x32_f4_quant(x):
    """x: [..., K] -> (packed uint8 [..., K/2], e8m0 uint8 [..., K/32])."""
    x = np.asarray(x, dtype=F32)
    shp = x.shape
    g = x.reshape(-1, 32)
    amax = np.abs(g).max(axis=-1)
    e = codecs.f32_to_e8m0((amax / F32(4.0)).astype(F32))
    s = codecs.e8m0_to_f32(e)
    y = (g / s[:, None]).astype(F32)
    codes = codecs.e2m1_encode(y).reshape(shp)
    return codecs.pack_fp4(codes), e.reshape(shp[:-1] + (shp[-1] // 32,))


def dequant_mxfp4(packed, e8m0):
    v = codecs.mxfp4_to_f32(packed)
    shp = v.shape
    s = codecs.e8m0_to_f32(np.asarray(e8m0, dtype=np.uint8)).reshape(-1, 1)
    return (v.reshape(-1, 32) * s).reshape(shp).astype(F32)
