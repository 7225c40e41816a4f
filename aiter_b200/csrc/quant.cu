// Dynamic per-group fp8 / int8 quantisation (1 x group, group in {32, 64, 128}).
//
// Restates dynamic_per_group_scaled_quant_kernel (csrc/kernels/quant_kernels.cu:20-133)
// with the arithmetic of the reference's torch oracle `pertoken_quant`
// (aiter/ops/quant.py:42-72): scale = amax / dtype_max (scale 0 -> 1); fp8:
// q = fp8(x / scale) with round-to-nearest-even (dtype_max 448); int8: q = x / scale
// truncated toward zero, as torch's float -> int8 conversion and the reference kernel's
// static_cast (csrc/include/aiter_opus_plus.h:87-102) do (dtype_max 127).  Each group
// is handled by group/8 lanes, 8 elements (16 bytes of bf16) per lane; amax by shuffles
// inside the lane segment.
#include "common.cuh"

namespace {

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
        uint4 u = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};
template <>
struct Vec8<__half> {
    static __device__ __forceinline__ void load(const __half* p, float (&v)[8]) {
        uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};
template <>
struct Vec8<float> {
    static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
        float4 a = reinterpret_cast<const float4*>(p)[0];
        float4 b = reinterpret_cast<const float4*>(p)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
};

template <typename T, int GROUP, bool I8 = false>
__global__ void __launch_bounds__(256)
group_quant_kernel(const T* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scales,
                   int64_t ngroups, const int* __restrict__ num_rows, int64_t rows_factor_groups,
                   int shuffle, int64_t groups_per_row, int64_t nrows) {
    constexpr int LPG = GROUP / 8;  // lanes per group
    int64_t limit = ngroups;
    if (num_rows) limit = min(limit, (int64_t)max(num_rows[0], 0) * rows_factor_groups);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // round the loop bound so every lane of a segment iterates together
    const int64_t total_lanes = ((ngroups * LPG + 31) / 32) * 32;
    for (int64_t t = tid; t < total_lanes; t += stride) {
        const int64_t g = t / LPG;
        const int sub = (int)(t % LPG);
        const bool on = g < limit;
        float v[8];
        if (on) {
            Vec8<T>::load(x + g * GROUP + sub * 8, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.f;
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
        for (int o = LPG / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float scale = amax / (I8 ? 127.0f : 448.0f);
        if (scale == 0.f) scale = 1.0f;
        if (on) {
            uint32_t w[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if constexpr (I8) {
                    uint32_t b = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        b |= (uint32_t)(uint8_t)(int8_t)__float2int_rz(v[4 * i + j] / scale) << (8 * j);
                    w[i] = b;
                } else {
                    __nv_fp8x4_e4m3 p4(make_float4(v[4 * i] / scale, v[4 * i + 1] / scale,
                                                   v[4 * i + 2] / scale, v[4 * i + 3] / scale));
                    w[i] = *reinterpret_cast<uint32_t*>(&p4);
                }
            }
            *reinterpret_cast<uint2*>(q + g * GROUP + sub * 8) = make_uint2(w[0], w[1]);
            if (sub == 0) {
                int64_t si = g;
                if (shuffle) {
                    int64_t row = g / groups_per_row, col = g % groups_per_row;
                    si = col * nrows + row;
                }
                scales[si] = scale;
            }
        }
    }
}

}  // namespace

AB_ENTRY(dynamic_per_token_scaled_quant,
         (aiter_tensor_t * out, aiter_tensor_t* input, aiter_tensor_t* scales,
          aiter_tensor_t* scale_ub, int shuffle_scale, aiter_tensor_t* num_rows,
          int64_t num_rows_factor, void* stream),
         (out, input, scales, scale_ub, shuffle_scale, num_rows, num_rows_factor, stream)) {
    using namespace ab;
    need(out, "out");
    need(input, "input");
    need(scales, "scales");
    AB_CHECK(scale_ub == nullptr, "scale_ub is not supported");
    AB_CHECK(out->dtype_ == AITER_DTYPE_fp8 || out->dtype_ == AITER_DTYPE_i8, "out must be fp8 or i8, got ",
             dtype_name(out->dtype_));
    const bool i8 = out->dtype_ == AITER_DTYPE_i8;
    need_dtype(scales, AITER_DTYPE_fp32, "scales");
    need_contig(out, "out");
    need_contig(input, "input");
    need_contig(scales, "scales");
    AB_CHECK(out->numel_ == input->numel_, "out and input sizes differ");
    const int64_t group = input->shape[input->ndim - 1];
    AB_CHECK(group == 32 || group == 64 || group == 128, "group size must be 32, 64 or 128, got ", group);
    const int64_t ngroups = (int64_t)input->numel_ / group;
    AB_CHECK((int64_t)scales->numel_ >= ngroups, "scales needs ", ngroups, " elements");
    const int64_t row_len = out->shape[out->ndim - 1];
    AB_CHECK(row_len % group == 0, "row length must be a multiple of the group size");
    const int64_t gpr = row_len / group;
    const int64_t nrows = ngroups / gpr;
    if (num_rows) need_dtype(num_rows, AITER_DTYPE_i32, "num_rows");
    AB_CHECK(((uintptr_t)input->ptr & 15) == 0 && ((uintptr_t)out->ptr & 7) == 0, "misaligned buffers");
    if (ngroups == 0) return;
    DeviceGuard dg(input->device_id);
    const int dev = input->device_id;
    const int64_t lanes = ngroups * (group / 8);
    const int blocks = (int)std::min<int64_t>((lanes + 255) / 256, (int64_t)num_sms(dev) * 8);
    cudaStream_t st = as_stream(stream);
    const int* nr = num_rows ? (const int*)num_rows->ptr : nullptr;
    const int64_t factor_groups = num_rows_factor * gpr;
    auto go = [&](auto tz, auto gz) {
        using T = decltype(tz);
        constexpr int G = decltype(gz)::value;
        if (i8)
            group_quant_kernel<T, G, true><<<blocks, 256, 0, st>>>((const T*)input->ptr, (uint8_t*)out->ptr,
                                                                   (float*)scales->ptr, ngroups, nr, factor_groups,
                                                                   shuffle_scale, gpr, nrows);
        else
            group_quant_kernel<T, G><<<blocks, 256, 0, st>>>((const T*)input->ptr, (uint8_t*)out->ptr,
                                                             (float*)scales->ptr, ngroups, nr, factor_groups,
                                                             shuffle_scale, gpr, nrows);
    };
    auto by_group = [&](auto tz) {
        if (group == 128) go(tz, std::integral_constant<int, 128>{});
        else if (group == 64) go(tz, std::integral_constant<int, 64>{});
        else go(tz, std::integral_constant<int, 32>{});
    };
    switch (input->dtype_) {
        case AITER_DTYPE_bf16: by_group(__nv_bfloat16{}); break;
        case AITER_DTYPE_fp16: by_group(__half{}); break;
        case AITER_DTYPE_fp32: by_group(float{}); break;
        default: fail("input must be bf16, fp16 or fp32");
    }
    check_launch("dynamic_per_token_scaled_quant");
}

// ---------------------------------------------------------------------------
// 1x128 quantisation scattered into sorted-row order (the A operand of the stage-1
// grouped GEMM).  Token t is quantised once (the arithmetic of group_quant_kernel
// above, `pertoken_quant` over 128 groups, aiter/ops/quant.py:42-72) and stored to
// the sorted rows pos[t * topk + s] of its slots (-1 = not routed here).  Scales
// are written transposed, [K/128][rows], for coalesced reads in the GEMM
// epilogue.  With an fp8 input (`hidden_scale` given, [M, K/128]) the rows and
// scales are copied instead -- fused_moe's pre-quantised input path
// (aiter/fused_moe.py:259-265).
namespace {

template <typename T, bool PREQ>
__global__ void __launch_bounds__(256)
scatter_quant_kernel(const T* __restrict__ x, const float* __restrict__ xs, const int* __restrict__ pos,
                     uint8_t* __restrict__ q, float* __restrict__ st, int M, int K, int topk, int rows_pad) {
    // 8 lanes per 128-wide group, 16 values (one 16-byte fp8 store per sorted row) each
    const int gpr = K / 128;
    const int64_t total_lanes = (int64_t)M * gpr * 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < ((total_lanes + 31) / 32) * 32;
         t += stride) {
        const int64_t g = t >> 3;
        const int sub = (int)(t & 7);
        const bool on = t < total_lanes;
        const int tok = on ? (int)(g / gpr) : 0;
        const int c = on ? (int)(g % gpr) : 0;
        uint4 packed = make_uint4(0, 0, 0, 0);
        float scale = 0.f;
        if constexpr (PREQ) {
            if (on) {
                packed = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(x) + (int64_t)tok * K + c * 128 + sub * 16);
                scale = xs[(int64_t)tok * gpr + c];
            }
        } else {
            float v[16];
            if (on) {
                const T* src = x + (int64_t)tok * K + c * 128 + sub * 16;
                Vec8<T>::load(src, *reinterpret_cast<float(*)[8]>(&v[0]));
                Vec8<T>::load(src + 8, *reinterpret_cast<float(*)[8]>(&v[8]));
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = 0.f;
            }
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            scale = amax / 448.0f;
            if (scale == 0.f) scale = 1.0f;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                __nv_fp8x4_e4m3 p4(make_float4(v[4 * i] / scale, v[4 * i + 1] / scale, v[4 * i + 2] / scale,
                                               v[4 * i + 3] / scale));
                w[i] = *reinterpret_cast<uint32_t*>(&p4);
            }
            packed = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (!on) continue;
        for (int s = 0; s < topk; ++s) {
            const int r = pos[(int64_t)tok * topk + s];
            if (r < 0 || r >= rows_pad) continue;
            *reinterpret_cast<uint4*>(q + (int64_t)r * K + c * 128 + sub * 16) = packed;
            if (sub == 0) st[(int64_t)c * rows_pad + r] = scale;
        }
    }
}

}  // namespace

AB_ENTRY(moe_gather_quant_1x128,
         (aiter_tensor_t * hidden, aiter_tensor_t* hidden_scale, aiter_tensor_t* token_sorted_pos, int64_t topk,
          aiter_tensor_t* out, aiter_tensor_t* out_scale, void* stream),
         (hidden, hidden_scale, token_sorted_pos, topk, out, out_scale, stream)) {
    using namespace ab;
    need(hidden, "hidden");
    need(token_sorted_pos, "token_sorted_pos");
    need(out, "out");
    need(out_scale, "out_scale");
    need_ndim(hidden, 2, "hidden");
    need_contig(hidden, "hidden");
    need_contig(out, "out");
    need_contig(out_scale, "out_scale");
    need_dtype(token_sorted_pos, AITER_DTYPE_i32, "token_sorted_pos");
    need_dtype(out, AITER_DTYPE_fp8, "out");
    need_dtype(out_scale, AITER_DTYPE_fp32, "out_scale");
    const int M = (int)hidden->shape[0], K = (int)hidden->shape[1];
    AB_CHECK(topk >= 1 && (int64_t)token_sorted_pos->numel_ >= M * topk, "token_sorted_pos must be [M * topk]");
    AB_CHECK(K % 128 == 0, "hidden width must be a multiple of 128");
    AB_CHECK(out->ndim == 2 && out->shape[1] == K, "out must be [rows, K]");
    const int rows_pad = (int)out->shape[0];
    AB_CHECK((int64_t)out_scale->numel_ == (int64_t)rows_pad * (K / 128), "out_scale must be [K/128, rows]");
    AB_CHECK(((uintptr_t)hidden->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "misaligned buffers");
    const bool preq = hidden->dtype_ == AITER_DTYPE_fp8;
    if (preq) {
        need(hidden_scale, "hidden_scale");
        need_dtype(hidden_scale, AITER_DTYPE_fp32, "hidden_scale");
        need_contig(hidden_scale, "hidden_scale");
        AB_CHECK((int64_t)hidden_scale->numel_ == (int64_t)M * (K / 128), "hidden_scale must be [M, K/128]");
    }
    if (M == 0 || rows_pad == 0) return;
    DeviceGuard dg(hidden->device_id);
    const int dev = hidden->device_id;
    const int64_t lanes = (int64_t)M * (K / 128) * 8;
    const int blocks = (int)std::min<int64_t>((lanes + 255) / 256, (int64_t)num_sms(dev) * 8);
    cudaStream_t st = as_stream(stream);
    const int* pos = (const int*)token_sorted_pos->ptr;
    uint8_t* q = (uint8_t*)out->ptr;
    float* sc = (float*)out_scale->ptr;
    const int k = (int)topk;
    switch (hidden->dtype_) {
        case AITER_DTYPE_bf16:
            scatter_quant_kernel<__nv_bfloat16, false><<<blocks, 256, 0, st>>>(
                (const __nv_bfloat16*)hidden->ptr, nullptr, pos, q, sc, M, K, k, rows_pad);
            break;
        case AITER_DTYPE_fp16:
            scatter_quant_kernel<__half, false><<<blocks, 256, 0, st>>>((const __half*)hidden->ptr, nullptr, pos, q, sc,
                                                                       M, K, k, rows_pad);
            break;
        case AITER_DTYPE_fp32:
            scatter_quant_kernel<float, false><<<blocks, 256, 0, st>>>((const float*)hidden->ptr, nullptr, pos, q, sc,
                                                                      M, K, k, rows_pad);
            break;
        case AITER_DTYPE_fp8:
            scatter_quant_kernel<uint8_t, true><<<blocks, 256, 0, st>>>(
                (const uint8_t*)hidden->ptr, (const float*)hidden_scale->ptr, pos, q, sc, M, K, k, rows_pad);
            break;
        default: fail("hidden must be bf16, fp16, fp32 or fp8");
    }
    check_launch("moe_gather_quant_1x128");
}
