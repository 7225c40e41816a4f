"""Weight preparation on the device (host-side setup, not the hot path).

* `quant_weight_128x128`  fp8 e4m3fn weights with fp32 scales per 128x128 block,
  the quantiser of op_tests/test_moe_2stage.py:84-110 (amax / 448, 0 -> 1).
* `quant_weight_mxfp4`    e2m1 values packed two per byte (low nibble first) with
  e8m0 scales per 32 along K, the quantiser of aiter/ops/quant.py:75-106.
* `unshuffle_weight`      the inverse of the reference's `shuffle_weight`
  (aiter/ops/shuffle.py:7-27), for weights prepared for AMD's MFMA kernels.
Weights are [E, N, K] with K contiguous (no AMD pre-shuffle).
"""
import torch

from . import dtypes


@torch.no_grad()
def quant_weight_128x128(w: torch.Tensor, chunk: int = 8):
    E, N, K = w.shape
    assert N % 128 == 0 and K % 128 == 0
    q = torch.empty((E, N, K), dtype=dtypes.fp8, device=w.device)
    s = torch.empty((E, N // 128, K // 128), dtype=torch.float32, device=w.device)
    for e0 in range(0, E, chunk):
        blk = w[e0:e0 + chunk].float().view(-1, N // 128, 128, K // 128, 128)
        amax = blk.abs().amax(dim=(2, 4), keepdim=True)
        sc = amax / dtypes.FP8_MAX
        sc = torch.where(sc == 0, torch.ones_like(sc), sc)
        q[e0:e0 + chunk] = (blk / sc).to(dtypes.fp8).view(-1, N, K)
        s[e0:e0 + chunk] = sc.view(-1, N // 128, K // 128)
    return q, s


def _f32_to_e8m0(x: torch.Tensor) -> torch.Tensor:
    """Biased exponent, rounded up when mantissa bit 22 is set and (bit 21, any
    lower bit, or a non-zero exponent) -- aiter/utility/fp4_utils.py:49-58."""
    u = x.contiguous().view(torch.int32)
    exp = ((u >> 23) & 0xFF)
    rnd = ((u & 0x400000) != 0) & (((u & 0x200000) != 0) | ((u & 0x1FFFFF) != 0) | (exp > 0))
    out = exp + rnd.to(torch.int32)
    out = torch.where(exp == 0xFF, torch.full_like(out, 0xFF), out & 0xFF)
    return out.to(torch.uint8)


def _e8m0_to_f32(e: torch.Tensor) -> torch.Tensor:
    bits = e.to(torch.int32) << 23
    bits = torch.where(e == 0, torch.full_like(bits, 0x00400000), bits)
    bits = torch.where(e == 0xFF, torch.full_like(bits, 0x7F800001), bits)
    return bits.view(torch.float32)


_E2M1_POS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _e2m1_encode(y: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even onto the e2m1 grid, saturating at 6 (codes 0..15)."""
    a = y.abs().clamp(max=6.0)
    q = torch.where(a < 2.0, torch.full_like(a, 0.5), torch.where(a < 4.0, torch.ones_like(a), torch.full_like(a, 2.0)))
    r = torch.round(a / q) * q                     # torch.round is half-to-even
    r = r.clamp(max=6.0)
    grid = torch.tensor(_E2M1_POS, device=y.device)
    code = torch.searchsorted(grid, r.contiguous())
    code = code | (torch.signbit(y).to(code.dtype) << 3)
    return code.to(torch.uint8)


@torch.no_grad()
def quant_weight_mxfp4(w: torch.Tensor, chunk: int = 4):
    """-> (packed fp4x2 as uint8 [E, N, K/2], e8m0 uint8 [E, N, K/32])."""
    E, N, K = w.shape
    assert K % 32 == 0
    packed = torch.empty((E, N, K // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((E, N, K // 32), dtype=torch.uint8, device=w.device)
    for e0 in range(0, E, chunk):
        x = w[e0:e0 + chunk].float().reshape(-1, 32)
        amax = x.abs().amax(dim=1)
        e = _f32_to_e8m0(amax / 4.0)
        y = x / _e8m0_to_f32(e)[:, None]
        c = _e2m1_encode(y).view(-1, N, K)
        n = c.shape[0]
        packed[e0:e0 + n] = c[..., 0::2] | (c[..., 1::2] << 4)
        scales[e0:e0 + n] = e.view(n, N, K // 32)
    return packed, scales


def dequant_128x128(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    E, N, K = q.shape
    return (q.float().view(E, N // 128, 128, K // 128, 128) * s[:, :, None, :, None]).view(E, N, K)


def dequant_mxfp4(packed: torch.Tensor, e8m0: torch.Tensor) -> torch.Tensor:
    grid = torch.tensor(_E2M1_POS + tuple(-v for v in _E2M1_POS), device=packed.device)
    lo = grid[(packed & 0xF).long()]
    hi = grid[(packed >> 4).long()]
    v = torch.stack([lo, hi], dim=-1).flatten(-2)
    sh = v.shape
    return (v.view(*sh[:-1], sh[-1] // 32, 32) * _e8m0_to_f32(e8m0)[..., None]).view(sh)


@torch.no_grad()
def mxfp4_to_fp8_blockscale(w_fp4: torch.Tensor, w_scale: torch.Tensor, check: bool = True):
    """MXFP4 weights [E, N, K/2] (fp4x2 or uint8) + e8m0 scales [E, N, K/32] ->
    (e4m3 [E, N, K], f32 [E, N/128, K/128]) holding exactly the same values, the
    operand format of the FP8 grouped GEMMs (CUDA kernel `mxfp4_to_fp8_blockscale`).
    With `check`, raises if a 128x128 block cannot be represented exactly (its
    non-zero group exponents span more than 14 binades); this synchronises once."""
    from . import _lib
    E, N, Kh = w_fp4.shape
    K = Kh * 2
    out = torch.empty((E, N, K), dtype=dtypes.fp8, device=w_fp4.device)
    out_s = torch.empty((E, N // 128, K // 128), dtype=torch.float32, device=w_fp4.device)
    status = torch.zeros(1, dtype=torch.int32, device=w_fp4.device) if check else None
    wf = w_fp4.view(torch.uint8) if w_fp4.dtype != torch.uint8 else w_fp4
    ws = w_scale.view(torch.uint8) if w_scale.dtype != torch.uint8 else w_scale
    _lib.call("mxfp4_to_fp8_blockscale", wf.contiguous(), ws.contiguous().view(E, N, K // 32), out, out_s, status)
    if check and int(status.item()) != 0:
        raise ValueError(f"{int(status.item())} MXFP4 blocks are not exactly representable as e4m3 with one "
                         "power-of-two scale per 128x128 block")
    return out, out_s


def mxfp4_moe_weight_scale_chunks(w_scale: torch.Tensor) -> torch.Tensor:
    """e8m0 scales [E, N, K/32] of MXFP4 weights -> the chunks the native A8W4 GEMMs
    copy into tensor memory: [E, N/128, K/128, 512] uint8, per 128 weight rows x 128 K
    values the 128 x 4 scales, line r / word w / byte b = row 32w + r, K group b
    (CUDA kernel `mxfp4_moe_weight_scale_chunks`).  The role of the reference's
    e8m0_shuffle of the scales (aiter/utility/fp4_utils.py) for this GEMM."""
    from . import _lib
    ws = w_scale.view(torch.uint8) if w_scale.dtype != torch.uint8 else w_scale
    if ws.dim() != 3:
        raise ValueError("w_scale must be [E, N, K/32]")
    E, N, G = ws.shape
    out = torch.empty((E, N // 128, G * 32 // 128, 512), dtype=torch.uint8, device=ws.device)
    _lib.call("mxfp4_moe_weight_scale_chunks", ws.contiguous(), out)
    return out


def is_scale_chunks(s: torch.Tensor) -> bool:
    return s.dim() == 4 and s.shape[-1] == 512


def prepare_a8w4_native(w1_fp4, w1_scale, w2_fp4, w2_scale):
    """One-time preparation for fused_moe(..., quant_type=QuantType.per_1x32): the MXFP4
    weights unchanged, their scales as chunks (so no call rearranges them)."""
    return w1_fp4, mxfp4_moe_weight_scale_chunks(w1_scale), w2_fp4, mxfp4_moe_weight_scale_chunks(w2_scale)


def prepare_a8w4(w1_fp4, w1_scale, w2_fp4, w2_scale):
    """One-time A8W4 weight preparation (the role of the reference's shuffle_weight):
    returns (w1_fp8, w1_scale_f32, w2_fp8, w2_scale_f32) for
    fused_moe(..., quant_type=QuantType.per_1x128)."""
    w1, s1 = mxfp4_to_fp8_blockscale(w1_fp4, w1_scale)
    w2, s2 = mxfp4_to_fp8_blockscale(w2_fp4, w2_scale)
    return w1, s1, w2, s2


@torch.no_grad()
def unshuffle_weight(x: torch.Tensor, layout=(16, 16), use_int4: bool = False) -> torch.Tensor:
    """[.., N, K] weights back from the AMD MFMA tile order of `shuffle_weight`
    (aiter/ops/shuffle.py:7-27), which views the weights as
    [-1, N/BN, BN, K/BK, BK/P, P] (BN = layout[0], BK = 2 * layout[1], P = 16 bytes
    of elements, 32 for int4) and stores them permuted to (0, 1, 3, 4, 2, 5); this
    applies the inverse permutation.  The result is the [E, N, K], K-contiguous layout
    the B200 kernels take; the `is_shuffled` mark is not carried over."""
    x_type = x.dtype
    if x_type == dtypes.fp4x2:
        x = x.view(torch.uint8)
    IN, IK = layout
    BK = IK * 2
    P = 16 // x.element_size() if not use_int4 else 32
    BN = IN
    N, K = x.shape[-2], x.shape[-1]
    if N % BN or K % BK:
        raise ValueError(f"weights [{N}, {K}] are not a whole number of {BN} x {BK} shuffle tiles")
    y = x.contiguous().view(-1, N // BN, K // BK, BK // P, BN, P)
    y = y.permute(0, 1, 4, 2, 3, 5).contiguous().view(*x.shape)
    return y.view(x_type)
