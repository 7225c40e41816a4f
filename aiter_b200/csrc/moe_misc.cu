// Small operators around the MoE path:
//   topk_sigmoid  (aiter/ops/moe_op.py:40-42 -> csrc/py_itfs_ck/topk_sigmoid_kernels.cu:15-66;
//                  torch reference op_tests/test_moe_topk_sigmoid.py:30-35): per token the k
//                  largest logits (descending; equal values: lower expert first) and
//                  sigmoid(logit) of each in fp32 -- Llama-4 style routing.
//   moe_sum       (aiter/ops/moe_op.py:45-46 -> csrc/kernels/topk_softmax_kernels.cu:737-854):
//                  out[t] = sum over the k slots of input[t, slot]; for k = 2, 4, 5 the sum runs
//                  in the element type slot by slot (one rounding per add, the reference's
//                  kernel), otherwise in fp32 with one rounding (its at::sum_out fallback).
//   silu_and_mul / gelu_and_mul / gelu_tanh_and_mul / scaled_silu_and_mul
//                 (aiter/ops/activation.py:10-23 -> csrc/kernels/activation_kernels.cu:24-160,
//                  337-360): out = act(x) * y for input [..., 2d] = [x | y], computed in fp32
//                  and rounded once to out's dtype; the scaled form multiplies by 1 / scale and
//                  writes fp8 e4m3 (saturating).  The split-K tail of the reference's
//                  fused_moe uses the first two (aiter/fused_moe.py:1719-1724).
// All are memory-bound: 16-byte vector loads and stores, grids sized to the data.
#include "common.cuh"
#include "rexp.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float beta = 0.79788456080286536f;  // sqrt(2 / pi)
    return 0.5f * x * (1.0f + tanhf(beta * (x + 0.044715f * x * x * x)));
}

enum Act : int { kSilu = 0, kGelu = 1, kGeluTanh = 2 };

template <int ACT>
__device__ __forceinline__ float act(float x) {
    if constexpr (ACT == kSilu)
        return silu_f(x);
    else if constexpr (ACT == kGelu)
        return gelu_f(x);
    else
        return gelu_tanh_f(x);
}

template <typename T>
__device__ __forceinline__ float to_f(T v) {
    if constexpr (std::is_same<T, float>::value)
        return v;
    else if constexpr (std::is_same<T, __half>::value)
        return __half2float(v);
    else
        return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f(float v) {
    if constexpr (std::is_same<T, float>::value)
        return v;
    else if constexpr (std::is_same<T, __half>::value)
        return __float2half_rn(v);
    else
        return __float2bfloat16_rn(v);
}

// ---------------------------------------------------------------- act_and_mul
// VEC elements per thread (16 bytes of the input type when d allows it, else 1).
template <typename TI, typename TO, int ACT, int VEC, bool SCALED>
__global__ void __launch_bounds__(kThreads)
act_and_mul_kernel(TO* __restrict__ out, const TI* __restrict__ in, int64_t rows, int d,
                   const float* __restrict__ scale) {
    const int64_t per_row = d / VEC;
    const int64_t total = rows * per_row;
    const float inv = SCALED ? 1.0f / scale[0] : 1.0f;
    for (int64_t q = (int64_t)blockIdx.x * kThreads + threadIdx.x; q < total; q += (int64_t)gridDim.x * kThreads) {
        const int64_t r = q / per_row;
        const int c = (int)(q % per_row) * VEC;
        const TI* xr = in + r * 2 * d + c;
        const TI* yr = xr + d;
        TI xv[VEC], yv[VEC];
        if constexpr (VEC * sizeof(TI) == 16) {
            *reinterpret_cast<uint4*>(xv) = __ldg(reinterpret_cast<const uint4*>(xr));
            *reinterpret_cast<uint4*>(yv) = __ldg(reinterpret_cast<const uint4*>(yr));
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                xv[j] = xr[j];
                yv[j] = yr[j];
            }
        }
        if constexpr (SCALED) {
            uint8_t o[VEC];
#pragma unroll
            for (int j = 0; j < VEC; ++j)
                o[j] = (uint8_t)__nv_cvt_float_to_fp8(act<ACT>(to_f(xv[j])) * to_f(yv[j]) * inv, __NV_SATFINITE,
                                                      __NV_E4M3);
            uint8_t* orow = reinterpret_cast<uint8_t*>(out) + r * d + c;
#pragma unroll
            for (int j = 0; j < VEC; ++j) orow[j] = o[j];
        } else {
            TO o[VEC];
#pragma unroll
            for (int j = 0; j < VEC; ++j) o[j] = from_f<TO>(act<ACT>(to_f(xv[j])) * to_f(yv[j]));
            TO* orow = out + r * d + c;
            if constexpr (VEC * sizeof(TO) == 16) {
                *reinterpret_cast<uint4*>(orow) = *reinterpret_cast<uint4*>(o);
            } else {
#pragma unroll
                for (int j = 0; j < VEC; ++j) orow[j] = o[j];
            }
        }
    }
}

int grid_for(int64_t work, int dev) {
    const int64_t b = (work + kThreads - 1) / kThreads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(b, 8LL * ab::num_sms(dev)));
}

template <typename TI, typename TO, int ACT, bool SCALED>
void launch_act(void* out, const void* in, int64_t rows, int d, const float* scale, int dev, cudaStream_t st) {
    constexpr int V = 16 / sizeof(TI);
    // vector path: whole 16-byte input packs, and both bases 16-byte aligned
    const bool vec = d % V == 0 && ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0;
    const int64_t work = rows * (vec ? d / V : d);
    const int g = grid_for(work, dev);
    if (vec)
        act_and_mul_kernel<TI, TO, ACT, V, SCALED><<<g, kThreads, 0, st>>>((TO*)out, (const TI*)in, rows, d, scale);
    else
        act_and_mul_kernel<TI, TO, ACT, 1, SCALED><<<g, kThreads, 0, st>>>((TO*)out, (const TI*)in, rows, d, scale);
}

template <int ACT>
void run_act(aiter_tensor_t* out, aiter_tensor_t* input, aiter_tensor_t* scale, void* stream, const char* name) {
    using namespace ab;
    need(out, "out");
    need(input, "input");
    need_contig(out, "out");
    need_contig(input, "input");
    AB_CHECK(input->ndim >= 1 && input->shape[input->ndim - 1] % 2 == 0, "input's last dim must be 2 * d");
    const int d = (int)(input->shape[input->ndim - 1] / 2);
    const int64_t rows = d > 0 ? (int64_t)input->numel_ / (2 * d) : 0;
    AB_CHECK((int64_t)out->numel_ == rows * d, "out must be [..., d]");
    const int in_dt = input->dtype_, out_dt = out->dtype_;
    AB_CHECK(in_dt == AITER_DTYPE_fp32 || in_dt == AITER_DTYPE_bf16 || in_dt == AITER_DTYPE_fp16,
             "input must be fp32, bf16 or fp16");
    if (rows == 0 || d == 0) return;
    DeviceGuard dg(input->device_id);
    cudaStream_t st = as_stream(stream);
    const int dev = input->device_id;
    if (scale) {
        need_dtype(scale, AITER_DTYPE_fp32, "scale");
        AB_CHECK(scale->numel_ >= 1, "scale must hold one value");
        AB_CHECK(out_dt == AITER_DTYPE_fp8, "scaled_act_and_mul writes fp8 outputs");
        const float* sp = (const float*)scale->ptr;
        if (in_dt == AITER_DTYPE_fp32)
            launch_act<float, uint8_t, ACT, true>(out->ptr, input->ptr, rows, d, sp, dev, st);
        else if (in_dt == AITER_DTYPE_bf16)
            launch_act<__nv_bfloat16, uint8_t, ACT, true>(out->ptr, input->ptr, rows, d, sp, dev, st);
        else
            launch_act<__half, uint8_t, ACT, true>(out->ptr, input->ptr, rows, d, sp, dev, st);
    } else if (in_dt == AITER_DTYPE_fp32) {
        if (out_dt == AITER_DTYPE_fp32)
            launch_act<float, float, ACT, false>(out->ptr, input->ptr, rows, d, nullptr, dev, st);
        else if (out_dt == AITER_DTYPE_bf16)
            launch_act<float, __nv_bfloat16, ACT, false>(out->ptr, input->ptr, rows, d, nullptr, dev, st);
        else if (out_dt == AITER_DTYPE_fp16)
            launch_act<float, __half, ACT, false>(out->ptr, input->ptr, rows, d, nullptr, dev, st);
        else
            fail("Unsupported output type for fp32 input");
    } else {
        AB_CHECK(out_dt == in_dt, "For bf16/fp16 input, output type must match input type");
        if (in_dt == AITER_DTYPE_bf16)
            launch_act<__nv_bfloat16, __nv_bfloat16, ACT, false>(out->ptr, input->ptr, rows, d, nullptr, dev, st);
        else
            launch_act<__half, __half, ACT, false>(out->ptr, input->ptr, rows, d, nullptr, dev, st);
    }
    check_launch(name);
}

// ---------------------------------------------------------------- moe_sum
// VEC elements per thread; STEPWISE: round to T after every add (k = 2, 4, 5).
template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads)
moe_sum_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t tokens, int k, int d, int stepwise) {
    const int64_t per_row = d / VEC;
    const int64_t total = tokens * per_row;
    for (int64_t q = (int64_t)blockIdx.x * kThreads + threadIdx.x; q < total; q += (int64_t)gridDim.x * kThreads) {
        const int64_t t = q / per_row;
        const int c = (int)(q % per_row) * VEC;
        float acc[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[j] = 0.0f;
        for (int s = 0; s < k; ++s) {
            const T* src = in + (t * k + s) * d + c;
            T v[VEC];
            if constexpr (VEC * sizeof(T) == 16) {
                *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(src));
            } else {
#pragma unroll
                for (int j = 0; j < VEC; ++j) v[j] = src[j];
            }
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                acc[j] += to_f(v[j]);
                if (stepwise) acc[j] = to_f(from_f<T>(acc[j]));
            }
        }
        T o[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) o[j] = from_f<T>(acc[j]);
        T* dst = out + t * d + c;
        if constexpr (VEC * sizeof(T) == 16) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(o);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) dst[j] = o[j];
        }
    }
}

template <typename T>
void launch_sum(void* out, const void* in, int64_t tokens, int k, int d, int dev, cudaStream_t st) {
    constexpr int V = 16 / sizeof(T);
    const int stepwise = (k == 2 || k == 4 || k == 5) ? 1 : 0;
    const bool vec = d % V == 0 && ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0;
    const int g = grid_for(tokens * (vec ? d / V : d), dev);
    if (vec)
        moe_sum_kernel<T, V><<<g, kThreads, 0, st>>>((T*)out, (const T*)in, tokens, k, d, stepwise);
    else
        moe_sum_kernel<T, 1><<<g, kThreads, 0, st>>>((T*)out, (const T*)in, tokens, k, d, stepwise);
}

// ---------------------------------------------------------------- topk_sigmoid
// Warp per token; each lane holds experts lane, lane + 32, ... of the row.
template <typename TI, typename TW, int PER_LANE>
__global__ void __launch_bounds__(kThreads)
topk_sigmoid_kernel(TW* __restrict__ weights, int32_t* __restrict__ ids, const TI* __restrict__ logits,
                    int64_t tokens, int E, int k) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
    for (int64_t t = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); t < tokens; t += warps) {
        float v[PER_LANE];
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
            const int e = lane + 32 * i;
            v[i] = e < E ? to_f(logits[t * E + e]) : -INFINITY;
        }
        for (int j = 0; j < k; ++j) {
            // lane-local best (lowest index among equal values: slots are visited in index order)
            float bv = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < PER_LANE; ++i) {
                const int e = lane + 32 * i;
                if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) {
                    bv = v[i];
                    bi = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                weights[t * k + j] = from_f<TW>(abd::rsigmoid(bv));
                ids[t * k + j] = bi;
            }
            if ((bi & 31) == lane) v[bi >> 5] = -INFINITY;  // taken
        }
    }
}

template <typename TI, typename TW>
void launch_topk_sigmoid(void* w, int32_t* ids, const void* logits, int64_t tokens, int E, int k, int dev,
                         cudaStream_t st) {
    const int g = grid_for(tokens * 32, dev);
    if (E <= 32)
        topk_sigmoid_kernel<TI, TW, 1><<<g, kThreads, 0, st>>>((TW*)w, ids, (const TI*)logits, tokens, E, k);
    else if (E <= 128)
        topk_sigmoid_kernel<TI, TW, 4><<<g, kThreads, 0, st>>>((TW*)w, ids, (const TI*)logits, tokens, E, k);
    else if (E <= 512)
        topk_sigmoid_kernel<TI, TW, 16><<<g, kThreads, 0, st>>>((TW*)w, ids, (const TI*)logits, tokens, E, k);
    else
        topk_sigmoid_kernel<TI, TW, 32><<<g, kThreads, 0, st>>>((TW*)w, ids, (const TI*)logits, tokens, E, k);
}

template <typename TI>
void topk_sigmoid_w(aiter_tensor_t* w, int32_t* ids, const void* logits, int64_t tokens, int E, int k, int dev,
                    cudaStream_t st) {
    if (w->dtype_ == AITER_DTYPE_fp32)
        launch_topk_sigmoid<TI, float>(w->ptr, ids, logits, tokens, E, k, dev, st);
    else if (w->dtype_ == AITER_DTYPE_bf16)
        launch_topk_sigmoid<TI, __nv_bfloat16>(w->ptr, ids, logits, tokens, E, k, dev, st);
    else
        launch_topk_sigmoid<TI, __half>(w->ptr, ids, logits, tokens, E, k, dev, st);
}

}  // namespace

AB_ENTRY(topk_sigmoid, (aiter_tensor_t * topk_weights, aiter_tensor_t* topk_indices, aiter_tensor_t* gating_output,
                        void* stream),
         (topk_weights, topk_indices, gating_output, stream)) {
    using namespace ab;
    need(topk_weights, "topk_weights");
    need(topk_indices, "topk_indices");
    need(gating_output, "gating_output");
    for (auto* t : {topk_weights, topk_indices, gating_output}) need_contig(t, "operand");
    need_ndim(gating_output, 2, "gating_output");
    need_ndim(topk_weights, 2, "topk_weights");
    need_dtype(topk_indices, AITER_DTYPE_i32, "topk_indices");
    const int in_dt = gating_output->dtype_, w_dt = topk_weights->dtype_;
    AB_CHECK(in_dt == AITER_DTYPE_fp32 || in_dt == AITER_DTYPE_bf16 || in_dt == AITER_DTYPE_fp16,
             "invalid datatype for topk_sigmoid: only fp16/bf16/fp32!");
    AB_CHECK(w_dt == AITER_DTYPE_fp32 || w_dt == AITER_DTYPE_bf16 || w_dt == AITER_DTYPE_fp16,
             "invalid datatype for topk_sigmoid: only fp16/bf16/fp32!");
    const int64_t tokens = gating_output->shape[0];
    const int E = (int)gating_output->shape[1];
    const int k = (int)topk_weights->shape[1];
    AB_CHECK(topk_weights->shape[0] == tokens && (int64_t)topk_indices->numel_ == tokens * k,
             "topk_weights / topk_indices must be [tokens, topk]");
    AB_CHECK(E >= 1 && E <= 1024 && k >= 1 && k <= E, "need 1 <= topk <= experts <= 1024");
    if (tokens == 0) return;
    DeviceGuard dg(gating_output->device_id);
    cudaStream_t st = as_stream(stream);
    int32_t* ids = (int32_t*)topk_indices->ptr;
    const int dev = gating_output->device_id;
    if (in_dt == AITER_DTYPE_fp32)
        topk_sigmoid_w<float>(topk_weights, ids, gating_output->ptr, tokens, E, k, dev, st);
    else if (in_dt == AITER_DTYPE_bf16)
        topk_sigmoid_w<__nv_bfloat16>(topk_weights, ids, gating_output->ptr, tokens, E, k, dev, st);
    else
        topk_sigmoid_w<__half>(topk_weights, ids, gating_output->ptr, tokens, E, k, dev, st);
    check_launch("topk_sigmoid");
}

AB_ENTRY(moe_sum, (aiter_tensor_t * input, aiter_tensor_t* output, void* stream), (input, output, stream)) {
    using namespace ab;
    need(input, "input");
    need(output, "output");
    need_contig(input, "input");
    need_contig(output, "output");
    AB_CHECK(input->dtype_ == output->dtype_, "input and output dtypes differ");
    AB_CHECK(input->dtype_ == AITER_DTYPE_fp32 || input->dtype_ == AITER_DTYPE_bf16 ||
                 input->dtype_ == AITER_DTYPE_fp16,
             "moe_sum supports fp32, bf16 and fp16");
    AB_CHECK(input->ndim == 3, "input must be [tokens, topk, hidden]");
    const int64_t tokens = input->shape[0];
    const int k = (int)input->shape[1];
    const int d = (int)input->shape[2];
    AB_CHECK((int64_t)output->numel_ == tokens * d, "output must be [tokens, hidden]");
    if (tokens == 0 || d == 0) return;
    DeviceGuard dg(input->device_id);
    cudaStream_t st = as_stream(stream);
    const int dev = input->device_id;
    if (input->dtype_ == AITER_DTYPE_fp32)
        launch_sum<float>(output->ptr, input->ptr, tokens, k, d, dev, st);
    else if (input->dtype_ == AITER_DTYPE_bf16)
        launch_sum<__nv_bfloat16>(output->ptr, input->ptr, tokens, k, d, dev, st);
    else
        launch_sum<__half>(output->ptr, input->ptr, tokens, k, d, dev, st);
    check_launch("moe_sum");
}

AB_ENTRY(silu_and_mul, (aiter_tensor_t * out, aiter_tensor_t* input, void* stream), (out, input, stream)) {
    run_act<kSilu>(out, input, nullptr, stream, "silu_and_mul");
}

AB_ENTRY(gelu_and_mul, (aiter_tensor_t * out, aiter_tensor_t* input, void* stream), (out, input, stream)) {
    run_act<kGelu>(out, input, nullptr, stream, "gelu_and_mul");
}

AB_ENTRY(gelu_tanh_and_mul, (aiter_tensor_t * out, aiter_tensor_t* input, void* stream), (out, input, stream)) {
    run_act<kGeluTanh>(out, input, nullptr, stream, "gelu_tanh_and_mul");
}

AB_ENTRY(scaled_silu_and_mul, (aiter_tensor_t * out, aiter_tensor_t* input, aiter_tensor_t* scale, void* stream),
         (out, input, scale, stream)) {
    ab::need(scale, "scale");
    run_act<kSilu>(out, input, scale, stream, "scaled_silu_and_mul");
}
