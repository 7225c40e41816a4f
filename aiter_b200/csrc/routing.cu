// Routing kernels: softmax top-k and grouped / biased-grouped top-k.
//
// One warp per token row.  Lane l holds experts l, l+32, l+64, ... (coalesced
// loads); selection runs k rounds of a warp arg-max in which the larger value
// wins and, on equal values, the lower expert index wins.
//
// Arithmetic contract (restated bit for bit by oracle/routing.py, and following the
// reference's torch path, op_tests/test_moeTopkSoftmax.py:21-41 and
// aiter/ops/topk.py:116-197, in torch's CPU order):
//  * exp = abd::rexp(): Cody & Waite range reduction x = n ln2 + r with ln 2 split into
//    a 21-bit head and a tail, the degree-13 Taylor polynomial of e^r in IEEE double
//    with separately rounded multiplies and adds (__dmul_rn / __dadd_rn: never
//    contracted into FMAs), times 2^n, rounded once to fp32 -- the correctly
//    rounded e^x except within ~2^-50 of an fp32 rounding boundary;
//  * softmax: max; e_i = exp(x_i - max); sum of 16-lane vectors in order (lane j
//    takes elements j, j+16, ...; a partial last vector only its first E mod 16
//    lanes), then the butterfly lane j + lane j^8, ^4, ^2, ^1 (torch's AVX-512
//    softmax); E < 16 sums element by element; p_i = e_i * (1 / sum);
//  * top-k of p (ties: lower index); renormalisation divides by the kept weights'
//    sum in the order torch's CPU sum kernel uses for a row of k floats (ksum);
//  * sigmoid(x) = 1 / (1 + exp(-x)), each step rounded to fp32.
#include <math.h>

#include "common.cuh"
#include "rexp.cuh"

namespace {

constexpr int kWarpsPerCta = 8;

struct ArgMax {
    float v;
    int i;
};

__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgMax b;
        b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
        b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
        a = better(a, b);
    }
    return a;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Softmax denominator of the routing contract over e[j] = element lane + 32 j
// (0 beyond E); every lane returns the sum.
template <int VPT>
__device__ __forceinline__ float softmax_sum(const float (&e)[VPT], int lane, int E) {
    float acc = 0.f;
    if (E < 16) {
        // element by element from e_0 (VPT == 1: lane i holds e_i)
        acc = __shfl_sync(0xffffffffu, e[0], 0);
        for (int i = 1; i < E; ++i) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, e[0], i));
        return acc;
    }
    // vector lane c = lane & 15 (lanes 0..15 accumulate); vector t = 2 j + (upper half)
    const int c = lane & 15;
    const int full = E >> 4, rem = E & 15;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const float upper = __shfl_down_sync(0xffffffffu, e[j], 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int t = 2 * j + h;
            const float v = h ? upper : e[j];
            if (t == 0) acc = v;
            else if (t < full || (t == full && c < rem)) acc = __fadd_rn(acc, v);
        }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    return __shfl_sync(0xffffffffu, acc, 0);
}

// Sum of the k kept weights (lane r holds pick r) in the order of torch's CPU sum
// over a contiguous row of k floats; every lane returns the sum.
__device__ __forceinline__ float ksum(float my_w, int k) {
    auto w = [&](int i) { return __shfl_sync(0xffffffffu, my_w, i); };
    if (k < 8) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        const int nil = k >> 2;
        for (int i = 0; i < nil; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) a[j] = __fadd_rn(a[j], w(4 * i + j));
        for (int i = 4 * nil; i < k; ++i) a[0] = __fadd_rn(a[0], w(i));
        return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), a[2]), a[3]);
    }
    const int nv = k >> 3;
    float l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) l[j] = w(j);
    for (int v = 1; v < nv; ++v)
#pragma unroll
        for (int j = 0; j < 8; ++j) l[j] = __fadd_rn(l[j], w(8 * v + j));
    float r = 0.f;
    for (int i = 8 * nv; i < k; ++i) r = __fadd_rn(r, w(i));
#pragma unroll
    for (int j = 0; j < 8; ++j) r = __fadd_rn(r, l[j]);
    return r;
}

// Arg-max over the lane's VPT values (index lane + 32*j), then across the warp.
template <int VPT>
__device__ __forceinline__ ArgMax row_argmax(const float (&v)[VPT], int lane) {
    ArgMax a{v[0], lane};
#pragma unroll
    for (int j = 1; j < VPT; ++j)
        if (v[j] > a.v) { a.v = v[j]; a.i = lane + 32 * j; }
    return warp_argmax(a);
}

template <int VPT>
__device__ __forceinline__ void knock_out(float (&v)[VPT], int lane, int idx) {
    if ((idx & 31) == lane) {
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (j == (idx >> 5)) v[j] = -INFINITY;
    }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
topk_softmax_kernel(const T* __restrict__ gating, int64_t g_stride, int M, int E, int k,
                    int num_shared, float* __restrict__ w, int64_t w_stride, int* __restrict__ ids,
                    int64_t id_stride, int* __restrict__ tei, int64_t tei_stride, int renorm) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (row >= M) return;
    const T* g = gating + (int64_t)row * g_stride;
    float v[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        int e = lane + 32 * j;
        v[j] = e < E ? abd::to_f32(g[e]) : -INFINITY;
    }
    // softmax over all routed experts
    float mx = v[0];
#pragma unroll
    for (int j = 1; j < VPT; ++j) mx = fmaxf(mx, v[j]);
    mx = warp_max(mx);
    float e[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) e[j] = (lane + 32 * j < E) ? abd::rexp(__fsub_rn(v[j], mx)) : 0.f;
    const float rz = __frcp_rn(softmax_sum<VPT>(e, lane, E));
#pragma unroll
    for (int j = 0; j < VPT; ++j) v[j] = (lane + 32 * j < E) ? __fmul_rn(e[j], rz) : -INFINITY;

    float my_p = 0.f;
    int my_id = 0;
    for (int r = 0; r < k; ++r) {
        ArgMax a = row_argmax<VPT>(v, lane);
        if (lane == r) { my_p = a.v; my_id = a.i; }
        knock_out<VPT>(v, lane, a.i);
    }
    const float denom = renorm ? ksum(my_p, k) : 1.f;
    if (lane < k) {
        w[(int64_t)row * w_stride + lane] = renorm ? __fdiv_rn(my_p, denom) : my_p;
        ids[(int64_t)row * id_stride + lane] = my_id;
        if (tei) tei[(int64_t)row * tei_stride + lane] = lane * M + row;
    }
    // shared experts: sigmoid of the trailing logits, written after the k picks
    for (int s2 = lane; s2 < num_shared; s2 += 32) {
        float x = abd::to_f32(g[E + s2]);
        w[(int64_t)row * w_stride + k + s2] = abd::rsigmoid(x);
    }
}

// Grouped top-k (softmax or sigmoid scores; optional correction bias).
// grouped_topk_torch / biased_grouped_topk_torch (aiter/ops/topk.py:116-197):
// group score = max (plain) or top-2 sum of the choice scores (biased); keep the
// topk_group best groups; experts outside them score 0.0 (masked_fill(..., 0.0));
// pick k; weights are the un-biased scores, renormalised, times the scaling factor.
template <typename T, int VPT, bool BIASED>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
grouped_topk_kernel(const T* __restrict__ gating, int64_t g_stride, const T* __restrict__ bias,
                    int M, int E, int G, int topk_group, int k, int softmax, int renorm,
                    float scaling, float* __restrict__ w, int64_t w_stride, int* __restrict__ ids,
                    int64_t id_stride) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (row >= M) return;
    const T* g = gating + (int64_t)row * g_stride;
    const int gs = E / G;
    float score[VPT], choice[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        int e = lane + 32 * j;
        score[j] = e < E ? abd::to_f32(g[e]) : -INFINITY;
    }
    if (softmax && !BIASED) {
        float mx = score[0];
#pragma unroll
        for (int j = 1; j < VPT; ++j) mx = fmaxf(mx, score[j]);
        mx = warp_max(mx);
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            score[j] = (lane + 32 * j < E) ? abd::rexp(__fsub_rn(score[j], mx)) : 0.f;
        const float rz = __frcp_rn(softmax_sum<VPT>(score, lane, E));
#pragma unroll
        for (int j = 0; j < VPT; ++j) score[j] = __fmul_rn(score[j], rz);
    } else {
#pragma unroll
        for (int j = 0; j < VPT; ++j) score[j] = abd::rsigmoid(score[j]);
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        int e = lane + 32 * j;
        float b = 0.f;
        if (BIASED && e < E) b = abd::to_f32(bias[e]);
        choice[j] = e < E ? __fadd_rn(score[j], b) : -INFINITY;
        if (e >= E) score[j] = -INFINITY;
    }
    // group scores: lane gi holds group gi's score
    float gscore = -INFINITY;
    for (int gi = 0; gi < G; ++gi) {
        ArgMax a{-INFINITY, 0x7fffffff};
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            int e = lane + 32 * j;
            if (e < E && e / gs == gi && (choice[j] > a.v || (choice[j] == a.v && e < a.i))) {
                a.v = choice[j];
                a.i = e;
            }
        }
        a = warp_argmax(a);
        float gsc = a.v;
        if (BIASED) {
            float m2 = -INFINITY;
#pragma unroll
            for (int j = 0; j < VPT; ++j) {
                int e = lane + 32 * j;
                if (e < E && e / gs == gi && e != a.i) m2 = fmaxf(m2, choice[j]);
            }
            m2 = warp_max(m2);
            gsc = __fadd_rn(a.v, m2);
        }
        if (lane == gi) gscore = gsc;
    }
    // keep the topk_group best groups (lower group index wins ties)
    unsigned keep = 0;
    {
        float gs_v = lane < G ? gscore : -INFINITY;
        for (int r = 0; r < topk_group; ++r) {
            ArgMax a = warp_argmax(ArgMax{gs_v, lane});
            keep |= 1u << a.i;
            if (lane == a.i) gs_v = -INFINITY;
        }
    }
    float tmp[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        int e = lane + 32 * j;
        tmp[j] = e < E ? (((keep >> (e / gs)) & 1u) ? choice[j] : 0.0f) : -INFINITY;
    }
    float my_w = 0.f;
    int my_id = 0;
    for (int r = 0; r < k; ++r) {
        ArgMax a = row_argmax<VPT>(tmp, lane);
        // un-biased score of the pick
        float sc = 0.f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (lane + 32 * j == a.i) sc = score[j];
        sc = __shfl_sync(0xffffffffu, sc, a.i & 31);
        if (!BIASED) sc = (((keep >> (a.i / gs)) & 1u) ? sc : 0.0f);
        if (lane == r) { my_w = sc; my_id = a.i; }
        knock_out<VPT>(tmp, lane, a.i);
    }
    const float denom = renorm ? ksum(my_w, k) : 1.f;
    if (lane < k) {
        float out = renorm ? __fdiv_rn(my_w, denom) : my_w;
        w[(int64_t)row * w_stride + lane] = __fmul_rn(out, scaling);
        ids[(int64_t)row * id_stride + lane] = my_id;
    }
}

int vpt_for(int E) {
    int v = 1;
    while (v * 32 < E) v <<= 1;
    return v;
}

template <typename T, typename Launch>
void dispatch_vpt(int vpt, Launch&& launch) {
    switch (vpt) {
        case 1: launch(std::integral_constant<int, 1>{}); break;
        case 2: launch(std::integral_constant<int, 2>{}); break;
        case 4: launch(std::integral_constant<int, 4>{}); break;
        case 8: launch(std::integral_constant<int, 8>{}); break;
        case 16: launch(std::integral_constant<int, 16>{}); break;
        case 32: launch(std::integral_constant<int, 32>{}); break;
        default: ab::fail("unsupported number of experts (max 1024)");
    }
}

template <typename Launch>
void dispatch_dtype(int dt, Launch&& launch) {
    switch (dt) {
        case AITER_DTYPE_fp32: launch(float{}); break;
        case AITER_DTYPE_bf16: launch(__nv_bfloat16{}); break;
        case AITER_DTYPE_fp16: launch(__half{}); break;
        default: ab::fail("gating_output must be fp32, bf16 or fp16, got ", ab::dtype_name(dt));
    }
}

}  // namespace

AB_ENTRY(topk_softmax,
         (aiter_tensor_t * topk_weights, aiter_tensor_t* topk_indices,
          aiter_tensor_t* token_expert_indices, aiter_tensor_t* gating_output, int need_renorm,
          int64_t num_shared_experts, const char* shared_expert_scoring_func, void* stream),
         (topk_weights, topk_indices, token_expert_indices, gating_output, need_renorm,
          num_shared_experts, shared_expert_scoring_func, stream)) {
    using namespace ab;
    need(topk_weights, "topk_weights");
    need(topk_indices, "topk_indices");
    need(gating_output, "gating_output");
    need_ndim(gating_output, 2, "gating_output");
    need_dtype(topk_weights, AITER_DTYPE_fp32, "topk_weights");
    need_dtype(topk_indices, AITER_DTYPE_i32, "topk_indices");
    AB_CHECK(gating_output->strides[1] == 1, "gating_output rows must be contiguous");
    AB_CHECK(topk_weights->strides[topk_weights->ndim - 1] == 1 &&
             topk_indices->strides[topk_indices->ndim - 1] == 1, "outputs need unit inner stride");
    const int M = (int)gating_output->shape[0];
    const int Etot = (int)gating_output->shape[1];
    const int ns = (int)num_shared_experts;
    AB_CHECK(ns >= 0 && ns < Etot, "bad num_shared_experts ", ns);
    if (ns > 0) {
        AB_CHECK(shared_expert_scoring_func && std::string(shared_expert_scoring_func) == "sigmoid",
                 "shared experts need shared_expert_scoring_func == \"sigmoid\"");
    }
    const int E = Etot - ns;
    const int k = (int)topk_indices->shape[topk_indices->ndim - 1];
    AB_CHECK(k >= 1 && k <= 32 && k <= E, "topk must be in [1, min(32, E)], got ", k);
    AB_CHECK(E <= 1024, "at most 1024 experts, got ", E);
    AB_CHECK(topk_weights->shape[topk_weights->ndim - 1] >= k + ns, "topk_weights too narrow");
    AB_CHECK(rows_of(topk_weights) >= M && rows_of(topk_indices) >= M, "outputs have fewer rows than tokens");
    int* tei = nullptr;
    int64_t tei_stride = 0;
    if (token_expert_indices && token_expert_indices->numel_ > 0) {
        need_dtype(token_expert_indices, AITER_DTYPE_i32, "token_expert_indices");
        tei = (int*)token_expert_indices->ptr;
        tei_stride = token_expert_indices->strides[0];
    }
    if (M == 0) return;
    DeviceGuard dg(gating_output->device_id);
    dim3 grid((M + kWarpsPerCta - 1) / kWarpsPerCta), block(kWarpsPerCta * 32);
    dispatch_dtype(gating_output->dtype_, [&](auto tz) {
        using T = decltype(tz);
        dispatch_vpt<T>(vpt_for(E), [&](auto vz) {
            topk_softmax_kernel<T, decltype(vz)::value><<<grid, block, 0, as_stream(stream)>>>(
                (const T*)gating_output->ptr, gating_output->strides[0], M, E, k, ns,
                (float*)topk_weights->ptr, topk_weights->strides[0], (int*)topk_indices->ptr,
                topk_indices->strides[0], tei, tei_stride, need_renorm);
        });
    });
    check_launch("topk_softmax");
}

static void grouped_common(aiter_tensor_t* gating_output, aiter_tensor_t* bias,
                           aiter_tensor_t* topk_weights, aiter_tensor_t* topk_ids, int64_t G,
                           int64_t TG, int need_renorm, int is_softmax, float scaling,
                           void* stream, bool biased) {
    using namespace ab;
    need(gating_output, "gating_output");
    need(topk_weights, "topk_weights");
    need(topk_ids, "topk_ids");
    need_ndim(gating_output, 2, "gating_output");
    need_dtype(topk_weights, AITER_DTYPE_fp32, "topk_weights");
    need_dtype(topk_ids, AITER_DTYPE_i32, "topk_ids");
    AB_CHECK(gating_output->strides[1] == 1, "gating_output rows must be contiguous");
    const int M = (int)gating_output->shape[0];
    const int E = (int)gating_output->shape[1];
    const int k = (int)topk_ids->shape[1];
    AB_CHECK(G >= 1 && G <= 32 && E % G == 0, "num_expert_group must divide E and be <= 32");
    AB_CHECK(TG >= 1 && TG <= G, "topk_group must be in [1, num_expert_group]");
    AB_CHECK(k >= 1 && k <= 32 && k <= E, "topk must be in [1, 32]");
    AB_CHECK(E <= 1024, "at most 1024 experts");
    if (biased) {
        need(bias, "correction_bias");
        AB_CHECK(bias->dtype_ == gating_output->dtype_, "correction_bias must match gating dtype");
        AB_CHECK((int)bias->numel_ == E, "correction_bias must have E elements");
    }
    if (M == 0) return;
    DeviceGuard dg(gating_output->device_id);
    dim3 grid((M + kWarpsPerCta - 1) / kWarpsPerCta), block(kWarpsPerCta * 32);
    dispatch_dtype(gating_output->dtype_, [&](auto tz) {
        using T = decltype(tz);
        dispatch_vpt<T>(vpt_for(E), [&](auto vz) {
            constexpr int V = decltype(vz)::value;
            if (biased)
                grouped_topk_kernel<T, V, true><<<grid, block, 0, as_stream(stream)>>>(
                    (const T*)gating_output->ptr, gating_output->strides[0], (const T*)bias->ptr, M, E,
                    (int)G, (int)TG, k, 0, need_renorm, scaling, (float*)topk_weights->ptr,
                    topk_weights->strides[0], (int*)topk_ids->ptr, topk_ids->strides[0]);
            else
                grouped_topk_kernel<T, V, false><<<grid, block, 0, as_stream(stream)>>>(
                    (const T*)gating_output->ptr, gating_output->strides[0], nullptr, M, E, (int)G,
                    (int)TG, k, is_softmax, need_renorm, scaling, (float*)topk_weights->ptr,
                    topk_weights->strides[0], (int*)topk_ids->ptr, topk_ids->strides[0]);
        });
    });
    check_launch("grouped_topk");
}

AB_ENTRY(grouped_topk,
         (aiter_tensor_t * gating_output, aiter_tensor_t* topk_weights, aiter_tensor_t* topk_ids,
          int64_t num_expert_group, int64_t topk_group, int need_renorm, int is_softmax,
          float routed_scaling_factor, void* stream),
         (gating_output, topk_weights, topk_ids, num_expert_group, topk_group, need_renorm,
          is_softmax, routed_scaling_factor, stream)) {
    grouped_common(gating_output, nullptr, topk_weights, topk_ids, num_expert_group, topk_group,
                   need_renorm, is_softmax, routed_scaling_factor, stream, false);
}

AB_ENTRY(biased_grouped_topk,
         (aiter_tensor_t * gating_output, aiter_tensor_t* correction_bias,
          aiter_tensor_t* topk_weights, aiter_tensor_t* topk_ids, int64_t num_expert_group,
          int64_t topk_grp, int need_renorm, float routed_scaling_factor, void* stream),
         (gating_output, correction_bias, topk_weights, topk_ids, num_expert_group, topk_grp,
          need_renorm, routed_scaling_factor, stream)) {
    grouped_common(gating_output, correction_bias, topk_weights, topk_ids, num_expert_group,
                   topk_grp, need_renorm, 0, routed_scaling_factor, stream, true);
}
