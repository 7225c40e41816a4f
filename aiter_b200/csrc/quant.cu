// Dynamic per-group fp8 quantisation (1 x group, group in {32, 64, 128}).
//
// Restates dynamic_per_group_scaled_quant_kernel (csrc/kernels/quant_kernels.cu:20-133)
// with the arithmetic of the reference's torch oracle `pertoken_quant`
// (aiter/ops/quant.py:42-72): scale = amax / 448 (scale 0 -> 1), q = fp8(x / scale)
// with round-to-nearest-even.  Each group is handled by group/8 lanes, 8 elements
// (16 bytes of bf16) per lane; amax by shuffles inside the lane segment.
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

template <typename T, int GROUP>
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
        float scale = amax / 448.0f;
        if (scale == 0.f) scale = 1.0f;
        if (on) {
            uint32_t w[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                __nv_fp8x4_e4m3 p4(make_float4(v[4 * i] / scale, v[4 * i + 1] / scale,
                                               v[4 * i + 2] / scale, v[4 * i + 3] / scale));
                w[i] = *reinterpret_cast<uint32_t*>(&p4);
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
    need_dtype(out, AITER_DTYPE_fp8, "out");
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
