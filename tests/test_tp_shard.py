"""Tensor-parallel sharding of FP8 block-scale MoE weights (CPU).

* inter_dim / tp a multiple of 128: the shard is a plain slice of the fp8 codes and
  scales (bit-exact);
* otherwise (config 3 at TP=8: 1536 / 8 = 192): the shard is re-quantised into
  shard-local 128x128 blocks after zero padding to 256; the padding must be exact
  zeros and the real part within one fp8 rounding of the original weights."""
import torch

from aiter_b200 import weights as W
from aiter_b200.dist.communication_op import shard_moe_weights_for_tp


def _weights(E, D, I, seed=0):
    g = torch.Generator().manual_seed(seed)
    w1q, w1s = W.quant_weight_128x128(torch.randn(E, 2 * I, D, generator=g) / D ** 0.5)
    w2q, w2s = W.quant_weight_128x128(torch.randn(E, D, I, generator=g) / I ** 0.5)
    return w1q, w1s, w2q, w2s


def test_aligned_shard_is_a_slice():
    E, D, I, tp = 2, 256, 512, 2
    w1q, w1s, w2q, w2s = _weights(E, D, I)
    for r in range(tp):
        a, b, c, d = shard_moe_weights_for_tp(w1q, w1s, w2q, w2s, r, tp)
        il = I // tp
        assert torch.equal(a[:, :il].view(torch.uint8), w1q[:, r * il:(r + 1) * il].view(torch.uint8))
        assert torch.equal(a[:, il:].view(torch.uint8), w1q[:, I + r * il:I + (r + 1) * il].view(torch.uint8))
        assert torch.equal(c.view(torch.uint8), w2q[:, :, r * il:(r + 1) * il].view(torch.uint8))
        assert torch.equal(b[:, :il // 128], w1s[:, r * il // 128:(r + 1) * il // 128])
        assert torch.equal(d, w2s[:, :, r * il // 128:(r + 1) * il // 128])


def test_unaligned_shard_is_padded_and_requantised():
    E, D, I, tp = 2, 256, 1536, 8
    w1q, w1s, w2q, w2s = _weights(E, D, I, seed=1)
    f1, f2 = W.dequant_128x128(w1q, w1s), W.dequant_128x128(w2q, w2s)
    il, ilp = I // tp, 256
    for r in (0, 3, 7):
        a, b, c, d = shard_moe_weights_for_tp(w1q, w1s, w2q, w2s, r, tp)
        assert a.shape == (E, 2 * ilp, D) and b.shape == (E, 2 * ilp // 128, D // 128)
        assert c.shape == (E, D, ilp) and d.shape == (E, D // 128, ilp // 128)
        l1, l2 = W.dequant_128x128(a, b), W.dequant_128x128(c, d)
        assert float(l1[:, il:ilp].abs().max()) == 0.0 and float(l1[:, ilp + il:].abs().max()) == 0.0
        assert float(l2[:, :, il:].abs().max()) == 0.0
        for got, ref in ((l1[:, :il], f1[:, r * il:(r + 1) * il]), (l1[:, ilp:ilp + il], f1[:, I + r * il:I + (r + 1) * il]),
                         (l2[:, :, :il], f2[:, :, r * il:(r + 1) * il])):
            # one e4m3 rounding (3 mantissa bits) relative to the block's amax at most
            assert float((got - ref).abs().max()) <= float(ref.abs().max()) / 16
