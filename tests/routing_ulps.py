"""Largest distance, in fp32 units in the last place, between the routing weights of
the contract shared by the kernels and the oracle (oracle/routing.py) and the
reference's torch outputs recorded in tests/golden (torch 2.11 CPU, AVX-512 host).

ids agree exactly in every case.  The weights differ by a few ulps for two reasons,
both in torch, not in the restated order of operations:

* torch's CPU softmax evaluates exp with a faster approximation than the correctly
  rounded exp of the contract, so some e_i differ by an ulp or two, which moves the
  softmax denominator and every p_i (topk/*, gtopk/*_softmax);
* grouped_topk_torch / biased_grouped_topk_torch take their picks with
  torch.topk(sorted=False), whose output order is left to the C++ library's
  selection algorithm; the renormalising sum then adds the k weights in that order,
  while the contract adds them in descending order (gtopk/*, btopk/*).

The sigmoid path with one kept weight per call order (topk_sigmoid/*) agrees bit for
bit.  Each entry is the measured maximum; the tests fail if a case gets worse.
"""
import numpy as np

MAX_ULPS = {
    "topk/m64_e8_k2_r0": 2, "topk/m64_e8_k2_r1": 2,
    "topk/m64_e128_k8_r0": 2, "topk/m64_e128_k8_r1": 2,
    "topk/m33_e256_k8_r0": 3, "topk/m33_e256_k8_r1": 2,
    "topk/m17_e64_k6_r0": 2, "topk/m17_e64_k6_r1": 4,
    "topk/m9_e512_k8_r0": 3, "topk/m9_e512_k8_r1": 3,
    "topk/zipf_m64_e256_k8_r0": 2, "topk/zipf_m64_e256_k8_r1": 2,
    "gtopk/m32_e256_softmax": 3, "gtopk/m32_e256_sigmoid": 3,
    "gtopk/m16_e64_softmax": 3, "gtopk/m16_e64_sigmoid": 3,
    "btopk/m32_e256": 3, "btopk/m16_e64": 2,
    "topk_sigmoid/e64_k4_bf16": 0, "topk_sigmoid/e128_k8_fp16": 0, "topk_sigmoid/e128_k1_fp32": 0,
}


def ulps(a, b):
    """Elementwise distance in fp32 ulps of two arrays of non-negative fp32 values."""
    a = np.asarray(a, dtype=np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, dtype=np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)
