// MXFP4 weight preparation for the A8W4 path.
//
// MXFP4 weights (e2m1 values packed two per byte, element 2i in the low nibble,
// with one e8m0 scale per 32 values along K; per_1x32_f4_quant,
// aiter/ops/quant.py:75-106, and the codecs of aiter/utility/fp4_utils.py:19-69)
// are rewritten, once, as e4m3 values with one power-of-two fp32 scale per 128x128
// block -- the operand format of the FP8 block-scale grouped GEMMs.  For a block
// whose largest non-zero group exponent is c_max, value v = m * 2^(c - 127) is
// stored as the e4m3 number m * 2^(c - c_max + 6) with block scale 2^(c_max - 133).
// e2m1 magnitudes are {0.5 .. 6} with one mantissa bit, so this is exact for
// every group whose exponent is within 14 of c_max (the smallest, 0.5 * 2^-8, is
// the e4m3 subnormal 2^-9); the largest is 6 * 2^6 = 384 <= 448.  Blocks whose
// exponents spread further, or that hold a NaN scale (code 255), are counted in
// `status` (the values are then rounded, not exact).
#include "common.cuh"

namespace {

__device__ __forceinline__ float e2m1_value(uint32_t c) {
    const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    const float v = mag[c & 7];
    return (c & 8) ? -v : v;
}

// grid: (K/128, N/128, E); 256 threads; thread t -> row t/2, K half t%2 (64 values)
__global__ void __launch_bounds__(256)
mxfp4_to_fp8_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sc, uint8_t* __restrict__ q,
                    float* __restrict__ qs, int* __restrict__ status, int N, int K) {
    __shared__ int s_max, s_min;
    const int kb = blockIdx.x, nb = blockIdx.y, e = blockIdx.z;
    const int t = threadIdx.x, r = t >> 1, half = t & 1;
    const int64_t row = (int64_t)e * N + nb * 128 + r;
    const int gpr = K / 32;                      // scale groups per row
    if (t == 0) { s_max = -1; s_min = 256; }
    __syncthreads();
    // this thread's two 32-value groups: bytes [kb*64 + half*32, +32) of the packed row
    const uint8_t* wp = w + row * (K / 2) + kb * 64 + half * 32;
    uint4 p0 = reinterpret_cast<const uint4*>(wp)[0];
    uint4 p1 = reinterpret_cast<const uint4*>(wp)[1];
    const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    int code[2];
    bool nonzero[2] = {false, false};
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        code[g] = sc[row * gpr + kb * 4 + half * 2 + g];
#pragma unroll
        for (int i = 0; i < 4; ++i) nonzero[g] |= (words[4 * g + i] & 0x77777777u) != 0u;
        if (nonzero[g]) {
            atomicMax(&s_max, code[g]);
            atomicMin(&s_min, code[g]);
        }
    }
    __syncthreads();
    const int cmax = s_max < 0 ? 127 : s_max;   // an all-zero block keeps scale 2^-6
    const bool bad = (s_max >= 0) && (cmax == 255 || cmax - s_min > 14 || cmax - 133 < -126);
    if (t == 0) {
        qs[((int64_t)e * (N / 128) + nb) * (K / 128) + kb] = ldexpf(1.0f, cmax - 133);
        if (bad && status) atomicAdd(status, 1);
    }
    uint8_t* qp = q + row * K + kb * 128 + half * 64;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const int shift = code[g] - cmax + 6;    // exponent of this group inside the block
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wd = words[4 * g + i];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint32_t nib = (wd >> (4 * (4 * j + b))) & 0xFu;
                    v[b] = ldexpf(e2m1_value(nib), shift);
                }
                __nv_fp8x4_e4m3 p4(make_float4(v[0], v[1], v[2], v[3]));
                out[2 * i + j] = *reinterpret_cast<uint32_t*>(&p4);
            }
        }
        reinterpret_cast<uint4*>(qp + g * 32)[0] = make_uint4(out[0], out[1], out[2], out[3]);
        reinterpret_cast<uint4*>(qp + g * 32)[1] = make_uint4(out[4], out[5], out[6], out[7]);
    }
}

// Scale chunks of the native A8W4 GEMMs: for every 128 weight rows x 128 K values,
// the 128 x 4 e8m0 scales as the 512 bytes tcgen05.cp moves into TMEM (32 lines of 16
// bytes; line r, word w, byte b = scale of row 32w + r, K group b), laid out
// [E, N/128, K/128, 512].  grid: (K/128, N/128, E), 128 threads; thread t = row t.
__global__ void __launch_bounds__(128)
mxfp4_scale_chunks_kernel(const uint8_t* __restrict__ sc, uint8_t* __restrict__ out, int N, int K) {
    const int kb = blockIdx.x, nb = blockIdx.y, e = blockIdx.z, t = threadIdx.x;
    const int gpr = K / 32;
    const int64_t row = (int64_t)e * N + nb * 128 + t;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(sc + row * gpr + kb * 4);  // K groups 4kb..4kb+3
    uint8_t* chunk = out + (((int64_t)e * (N / 128) + nb) * (K / 128) + kb) * 512;
    *reinterpret_cast<uint32_t*>(chunk + (t & 31) * 16 + (t >> 5) * 4) = word;
}

}  // namespace

AB_ENTRY(mxfp4_moe_weight_scale_chunks, (aiter_tensor_t * w_scale, aiter_tensor_t* out, void* stream),
         (w_scale, out, stream)) {
    using namespace ab;
    need(w_scale, "w_scale");
    need(out, "out");
    AB_CHECK(w_scale->dtype_ == AITER_DTYPE_fp8_e8m0 || w_scale->dtype_ == AITER_DTYPE_u8,
             "w_scale must be e8m0 (or its uint8 view)");
    AB_CHECK(out->dtype_ == AITER_DTYPE_fp8_e8m0 || out->dtype_ == AITER_DTYPE_u8, "out must be e8m0 or uint8");
    need_contig(w_scale, "w_scale");
    need_contig(out, "out");
    need_ndim(w_scale, 3, "w_scale");
    const int E = (int)w_scale->shape[0], N = (int)w_scale->shape[1], K = (int)w_scale->shape[2] * 32;
    AB_CHECK(N % 128 == 0 && K % 128 == 0, "N and K must be multiples of 128");
    AB_CHECK((int64_t)out->numel_ == (int64_t)E * (N / 128) * (K / 128) * 512, "out must be [E, N/128, K/128, 512]");
    AB_CHECK(((uintptr_t)w_scale->ptr & 3) == 0 && ((uintptr_t)out->ptr & 15) == 0, "misaligned buffers");
    if (E == 0) return;
    DeviceGuard dg(w_scale->device_id);
    mxfp4_scale_chunks_kernel<<<dim3(K / 128, N / 128, E), 128, 0, as_stream(stream)>>>(
        (const uint8_t*)w_scale->ptr, (uint8_t*)out->ptr, N, K);
    check_launch("mxfp4_moe_weight_scale_chunks");
}

AB_ENTRY(mxfp4_to_fp8_blockscale,
         (aiter_tensor_t * w_fp4, aiter_tensor_t* w_scale, aiter_tensor_t* out, aiter_tensor_t* out_scale,
          aiter_tensor_t* status, void* stream),
         (w_fp4, w_scale, out, out_scale, status, stream)) {
    using namespace ab;
    need(w_fp4, "w_fp4");
    need(w_scale, "w_scale");
    need(out, "out");
    need(out_scale, "out_scale");
    AB_CHECK(w_fp4->dtype_ == AITER_DTYPE_fp4x2 || w_fp4->dtype_ == AITER_DTYPE_u8 || w_fp4->dtype_ == AITER_DTYPE_i8,
             "w_fp4 must be fp4x2 (or its uint8 view)");
    AB_CHECK(w_scale->dtype_ == AITER_DTYPE_fp8_e8m0 || w_scale->dtype_ == AITER_DTYPE_u8,
             "w_scale must be e8m0 (or its uint8 view)");
    need_dtype(out, AITER_DTYPE_fp8, "out");
    need_dtype(out_scale, AITER_DTYPE_fp32, "out_scale");
    for (auto* t : {w_fp4, w_scale, out, out_scale}) need_contig(t, "operand");
    need_ndim(w_fp4, 3, "w_fp4");
    const int E = (int)w_fp4->shape[0], N = (int)w_fp4->shape[1], K = (int)w_fp4->shape[2] * 2;
    AB_CHECK(N % 128 == 0 && K % 128 == 0, "N and K must be multiples of 128");
    AB_CHECK((int64_t)w_scale->numel_ == (int64_t)E * N * (K / 32), "w_scale must be [E, N, K/32]");
    AB_CHECK(out->ndim == 3 && out->shape[0] == E && out->shape[1] == N && out->shape[2] == K, "out must be [E, N, K]");
    AB_CHECK((int64_t)out_scale->numel_ == (int64_t)E * (N / 128) * (K / 128), "out_scale must be [E, N/128, K/128]");
    AB_CHECK(((uintptr_t)w_fp4->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "misaligned buffers");
    int* st = nullptr;
    if (status) {
        need_dtype(status, AITER_DTYPE_i32, "status");
        st = (int*)status->ptr;
    }
    if (E == 0) return;
    DeviceGuard dg(w_fp4->device_id);
    dim3 grid(K / 128, N / 128, E);
    mxfp4_to_fp8_kernel<<<grid, 256, 0, as_stream(stream)>>>((const uint8_t*)w_fp4->ptr, (const uint8_t*)w_scale->ptr,
                                                            (uint8_t*)out->ptr, (float*)out_scale->ptr, st, N, K);
    check_launch("mxfp4_to_fp8_blockscale");
}
