"""Seeded synthetic inputs with the distributions BASELINE.json names
(test infrastructure only).  No public dataset is involved: the reference's own
tests draw `torch.randn` inputs (op_tests/test_moe_2stage.py:53-73).

* activations N(0,1), rounded to bf16;
* weights N(0,1)/sqrt(K), quantised fp8 128x128 or MXFP4 1x32;
* router logits N(0,1) (plus a per-expert log-popularity bias drawn from a
  Zipf(s=1.1) law over a random expert permutation for the skewed config),
  routed with softmax -> top-k -> renormalise.
"""
import numpy as np

from . import codecs, quant, routing


def make_hidden(rng, M, D):
    return codecs.round_bf16(rng.standard_normal((M, D), dtype=np.float32))


def make_logits(rng, M, E, zipf_s=None):
    x = rng.standard_normal((M, E), dtype=np.float32)
    if zipf_s is not None:
        ranks = rng.permutation(E) + 1
        p = 1.0 / ranks.astype(np.float64) ** zipf_s
        p /= p.sum()
        x = (x + np.log(p).astype(np.float32)[None, :]).astype(np.float32)
    return x


def make_fp8_weights(rng, E, N, K):
    w = (rng.standard_normal((E, N, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)
    return quant.weight_128x128_quant(w)


def make_mxfp4_weights(rng, E, N, K):
    w = (rng.standard_normal((E, N, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)
    return quant.per_1x32_f4_quant(w)


def make_moe_case(seed, M, D, I, E, topk, wfmt="fp8", zipf_s=None):
    rng = np.random.default_rng(seed)
    hidden = make_hidden(rng, M, D)
    logits = make_logits(rng, M, E, zipf_s)
    tw, tid, _ = routing.topk_softmax(logits, topk, True)
    if wfmt == "fp8":
        w1q, w1s = make_fp8_weights(rng, E, 2 * I, D)
        w2q, w2s = make_fp8_weights(rng, E, D, I)
    else:
        w1q, w1s = make_mxfp4_weights(rng, E, 2 * I, D)
        w2q, w2s = make_mxfp4_weights(rng, E, D, I)
    return dict(hidden=hidden, logits=logits, topk_weights=tw, topk_ids=tid,
                w1_q=w1q, w1_s=w1s, w2_q=w2q, w2_s=w2s)
