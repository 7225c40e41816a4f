// MXFP4 activation quant and the MoE-sorted e8m0 scale layout, the inputs of an
// A4W4 MoE (fp4 activations, fp4 weights):
//   * dynamic_per_group_scaled_quant_fp4 -- per 1x32 group: e = e8m0(amax / 4) with
//     the reference's round-half-up mantissa rule, y = x / 2^(e-127), codes e2m1
//     round-to-nearest-even saturating at 6, packed two per byte low nibble first
//     (per_1x32_f4_quant, aiter/ops/quant.py:75-106; f32_to_e8m0 / e8m0_to_f32 /
//     f32_to_mxfp4, aiter/utility/fp4_utils.py:19-69,100-107); the scales either in
//     row order or in the e8m0_shuffle layout (fp4_utils.py:72-92);
//   * mxfp4_moe_sort -- the e8m0 scales gathered into moe_sorting order and
//     shuffled (mxfp4_moe_sort_hip, aiter/ops/quant.py:552-580; layout of run_torch,
//     op_tests/test_moe_sorting_mxfp4.py:20-43): sorted row p takes the scales of
//     token sorted_ids[p] & 0xFFFFFF (per-token scales) or of row token * topk + slot
//     (per-(token, slot) scales); padding slots and rows from num_valid_ids on are 0;
//   * fused_dynamic_mxfp4_quant_moe_sort -- both in one launch (aiter/ops/quant.py:
//     584-652): one block range quantises every row, the other writes the sorted
//     scales, recomputing each group's e8m0 from the input.
// The shuffled layout views a [rows, cols] scale matrix (rows % 32 == 0,
// cols % 8 == 0) as [rows/32, 2, 16, cols/8, 2, 4] and stores it permuted to
// (0, 3, 5, 2, 4, 1): element (r, c) lands at
//   ((((r/32 * cols/8 + c/8) * 4 + c%4) * 16 + r%16) * 2 + (c%8)/4) * 2 + (r%32)/16.
// Integer and byte work: every output is bit-exact against the reference's torch
// functions (tests/golden).
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

// f32_to_e8m0 (fp4_utils.py:49-58): biased exponent, +1 when mantissa bit 22 is set
// and (bit 21, any lower bit or a non-zero exponent); Inf / NaN -> 0xFF.
__device__ __forceinline__ uint32_t f32_to_e8m0(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t e = (u >> 23) & 0xFF;
    if (e == 0xFF) return 0xFF;
    const bool up = (u & 0x400000u) && ((u & 0x200000u) || (u & 0x1FFFFFu) || e > 0);
    return (e + (up ? 1u : 0u)) & 0xFF;
}

// e8m0_to_f32 (fp4_utils.py:61-69): 0 -> 2^-127, 0xFF -> NaN.
__device__ __forceinline__ float e8m0_to_f32(uint32_t e) {
    if (e == 0) return __uint_as_float(0x00400000u);
    if (e == 0xFF) return __uint_as_float(0x7F800001u);
    return __uint_as_float(e << 23);
}

// e2m1 code of y: round to nearest even on the grid {0, .5, 1, 1.5, 2, 3, 4, 6},
// saturating at 6, sign kept for zero, NaN -> 7 | sign (the rounding of the
// torchao-derived _f32_to_floatx_unpacked the reference uses).
__device__ __forceinline__ uint32_t e2m1_code(float y) {
    const uint32_t sign = (__float_as_uint(y) >> 31) << 3;
    if (isnan(y)) return 7u | sign;
    const float a = fminf(fabsf(y), 6.0f);
    const float q = a < 2.0f ? 0.5f : (a < 4.0f ? 1.0f : 2.0f);  // grid spacing: a / q is exact
    const float r = fminf(rintf(a / q) * q, 6.0f);
    const uint32_t c = r < 2.0f ? (uint32_t)(r * 2.0f) : (r < 4.0f ? (uint32_t)(r + 2.0f) : (r < 6.0f ? 6u : 7u));
    return c | sign;
}

template <typename T>
__device__ __forceinline__ void load32(const T* p, float (&v)[32]);
template <>
__device__ __forceinline__ void load32<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[32]) {
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 u = p4[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            v[8 * i + 2 * j] = f.x;
            v[8 * i + 2 * j + 1] = f.y;
        }
    }
}
template <>
__device__ __forceinline__ void load32<__half>(const __half* p, float (&v)[32]) {
    const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 u = p4[i];
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            v[8 * i + 2 * j] = f.x;
            v[8 * i + 2 * j + 1] = f.y;
        }
    }
}
template <>
__device__ __forceinline__ void load32<float>(const float* p, float (&v)[32]) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = p4[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
}

template <typename T>
__device__ __forceinline__ uint32_t group_e8m0(const T* p) {
    float v[32];
    load32<T>(p, v);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    return f32_to_e8m0(amax / 4.0f);
}

// Byte offset of scale element (r, c) in the shuffled layout of a matrix with `cols`
// columns (cols % 8 == 0).
__device__ __forceinline__ int64_t shuffled_offset(int64_t r, int64_t c, int64_t cols) {
    const int64_t a = r >> 5, f = (r >> 4) & 1, d = r & 15;
    const int64_t b = c >> 3, e = (c >> 2) & 1, cc = c & 3;
    return ((((a * (cols >> 3) + b) * 4 + cc) * 16 + d) * 2 + e) * 2 + f;
}

// One thread per 32-element group of a row: the e8m0 scale and 16 bytes of codes.
// Rows from num_rows[0] * factor on are left untouched (when num_rows is given).
template <typename T>
__device__ __forceinline__ void quant_group(const T* __restrict__ x, int64_t ldx, int64_t gpr, int64_t gi,
                                            uint8_t* __restrict__ q, int64_t ldq, uint8_t* __restrict__ scale,
                                            int64_t ld_scale, int shuffle, int64_t scale_cols) {
    const int64_t row = gi / gpr, g = gi % gpr;
    const T* p = x + row * ldx + g * 32;
    float v[32];
    load32<T>(p, v);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint32_t e = f32_to_e8m0(amax / 4.0f);
    const float s = e8m0_to_f32(e);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) packed |= e2m1_code(v[8 * i + j] / s) << (4 * j);
        w[i] = packed;
    }
    *reinterpret_cast<uint4*>(q + row * ldq + g * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    if (scale != nullptr) {
        if (shuffle) scale[shuffled_offset(row, g, scale_cols)] = (uint8_t)e;
        else scale[row * ld_scale + g] = (uint8_t)e;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
mxfp4_quant_kernel(const T* __restrict__ x, int64_t rows, int64_t ldx, int64_t gpr, uint8_t* __restrict__ q,
                   int64_t ldq, uint8_t* __restrict__ scale, int64_t ld_scale, int shuffle, int64_t scale_cols,
                   const int* __restrict__ num_rows, int64_t factor) {
    int64_t live = rows;
    if (num_rows != nullptr) live = min(rows, (int64_t)max(num_rows[0], 0) * factor);
    const int64_t total = live * gpr;
    for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < total; gi += (int64_t)gridDim.x * blockDim.x)
        quant_group<T>(x, ldx, gpr, gi, q, ldq, scale, ld_scale, shuffle, scale_cols);
}

// Scale byte of sorted row r, scale column c: from a row-order e8m0 matrix
// (`scale`, when given) or recomputed from the input rows.
template <typename T>
__device__ __forceinline__ uint32_t sorted_scale(int64_t r, int64_t c, const int* __restrict__ sorted_ids,
                                                 int64_t max_pad, int64_t nvalid, int64_t token_num, int64_t topk,
                                                 int64_t src_rows, const uint8_t* __restrict__ scale,
                                                 int64_t ld_scale, const T* __restrict__ x, int64_t ldx) {
    if (r >= nvalid || r >= max_pad) return 0;
    const uint32_t id = (uint32_t)sorted_ids[r];
    const int64_t tok = id & 0xFFFFFF;
    if (tok >= token_num) return 0;
    const int64_t src = topk > 1 ? tok * topk + (int64_t)(id >> 24) : tok;
    if (src >= src_rows) return 0;
    if (scale != nullptr) return scale[src * ld_scale + c];
    return group_e8m0<T>(x + src * ldx + c * 32);
}

// One thread per 4 consecutive bytes of the shuffled output: (e, f) in {0,1}^2 with
// f fastest, i.e. sorted rows r0 and r0 + 16, scale columns c0 and c0 + 4.
template <typename T>
__device__ __forceinline__ void sort_quad(int64_t o4, int64_t cols, uint8_t* __restrict__ out,
                                          const int* __restrict__ sorted_ids, int64_t max_pad, int64_t nvalid,
                                          int64_t token_num, int64_t topk, int64_t src_rows,
                                          const uint8_t* __restrict__ scale, int64_t ld_scale,
                                          const T* __restrict__ x, int64_t ldx) {
    const int64_t d = o4 & 15, cc = (o4 >> 4) & 3, ab = o4 >> 6;
    const int64_t b = ab % (cols >> 3), a = ab / (cols >> 3);
    uint32_t word = 0;
#pragma unroll
    for (int ef = 0; ef < 4; ++ef) {
        const int e = ef >> 1, f = ef & 1;
        const int64_t r = a * 32 + f * 16 + d, c = b * 8 + e * 4 + cc;
        word |= sorted_scale<T>(r, c, sorted_ids, max_pad, nvalid, token_num, topk, src_rows, scale, ld_scale, x, ldx)
                << (8 * ef);
    }
    reinterpret_cast<uint32_t*>(out)[o4] = word;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
mxfp4_moe_sort_kernel(uint8_t* __restrict__ out, int64_t out_rows, int64_t cols, const int* __restrict__ sorted_ids,
                      int64_t max_pad, const int* __restrict__ num_valid, int64_t token_num, int64_t topk,
                      int64_t src_rows, const uint8_t* __restrict__ scale, int64_t ld_scale, const T* __restrict__ x,
                      int64_t ldx) {
    const int64_t nvalid = num_valid[0];
    const int64_t quads = out_rows * cols / 4;
    for (int64_t o4 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o4 < quads; o4 += (int64_t)gridDim.x * blockDim.x)
        sort_quad<T>(o4, cols, out, sorted_ids, max_pad, nvalid, token_num, topk, src_rows, scale, ld_scale, x, ldx);
}

// Fused: blocks [0, qblocks) quantise every input row (codes only), the rest write
// the sorted scales from the input.
template <typename T>
__global__ void __launch_bounds__(kThreads)
mxfp4_quant_sort_kernel(const T* __restrict__ x, int64_t rows, int64_t ldx, int64_t gpr, uint8_t* __restrict__ q,
                        int64_t ldq, int qblocks, uint8_t* __restrict__ out, int64_t out_rows,
                        const int* __restrict__ sorted_ids, int64_t max_pad, const int* __restrict__ num_valid,
                        int64_t token_num, int64_t topk) {
    if ((int)blockIdx.x < qblocks) {
        const int64_t total = rows * gpr;
        for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < total; gi += (int64_t)qblocks * blockDim.x)
            quant_group<T>(x, ldx, gpr, gi, q, ldq, nullptr, 0, 0, 0);
        return;
    }
    const int64_t nvalid = num_valid[0];
    const int64_t quads = out_rows * gpr / 4;
    const int64_t nb = gridDim.x - qblocks;
    for (int64_t o4 = (int64_t)(blockIdx.x - qblocks) * blockDim.x + threadIdx.x; o4 < quads; o4 += nb * blockDim.x)
        sort_quad<T>(o4, gpr, out, sorted_ids, max_pad, nvalid, token_num, topk, rows,
                     nullptr, 0, x, ldx);
}

int grid_for(int64_t work, int dev) {
    const int64_t blocks = (work + kThreads - 1) / kThreads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)ab::num_sms(dev) * 8));
}

void check_input(const aiter_tensor_t* x, const char* name) {
    using namespace ab;
    need(x, name);
    AB_CHECK(x->dtype_ == AITER_DTYPE_bf16 || x->dtype_ == AITER_DTYPE_fp16 || x->dtype_ == AITER_DTYPE_fp32, name,
             " must be bf16, fp16 or fp32");
    AB_CHECK(x->ndim >= 1 && x->strides[x->ndim - 1] == 1, name, " rows must be contiguous");
    const int64_t cols = x->shape[x->ndim - 1];
    AB_CHECK(cols % 32 == 0, name, " width must be a multiple of 32");
    for (int d = 0; d + 2 < x->ndim; ++d)
        AB_CHECK(x->strides[d] == x->strides[d + 1] * x->shape[d + 1], name, " must be a row-major stack of rows");
    const int64_t ld = x->ndim >= 2 ? x->strides[x->ndim - 2] : cols;
    AB_CHECK((ld * (int64_t)elem_size(x->dtype_)) % 16 == 0 && ((uintptr_t)x->ptr & 15) == 0, name,
             " rows must be 16-byte aligned");
}

int64_t row_stride(const aiter_tensor_t* x) {
    const int64_t cols = x->shape[x->ndim - 1];
    return x->ndim >= 2 ? x->strides[x->ndim - 2] : cols;
}

template <typename F>
void by_dtype(int dt, F&& f) {
    if (dt == AITER_DTYPE_bf16) f((const __nv_bfloat16*)nullptr);
    else if (dt == AITER_DTYPE_fp16) f((const __half*)nullptr);
    else f((const float*)nullptr);
}

}  // namespace

AB_ENTRY(dynamic_per_group_scaled_quant_fp4,
         (aiter_tensor_t * out, aiter_tensor_t* input, aiter_tensor_t* scales, int64_t group_size, int shuffle_scale,
          aiter_tensor_t* num_rows, int64_t num_rows_factor, void* stream),
         (out, input, scales, group_size, shuffle_scale, num_rows, num_rows_factor, stream)) {
    using namespace ab;
    check_input(input, "input");
    need(out, "out");
    need(scales, "scales");
    AB_CHECK(group_size == 32, "group_size must be 32 (MXFP4), got ", group_size);
    AB_CHECK(out->dtype_ == AITER_DTYPE_fp4x2 || out->dtype_ == AITER_DTYPE_u8, "out must be fp4x2");
    AB_CHECK(scales->dtype_ == AITER_DTYPE_fp8_e8m0 || scales->dtype_ == AITER_DTYPE_u8, "scales must be e8m0");
    need_contig(out, "out");
    need_contig(scales, "scales");
    const int64_t cols = input->shape[input->ndim - 1];
    const int64_t rows = cols > 0 ? (int64_t)input->numel_ / cols : 0;
    const int64_t gpr = cols / 32;
    AB_CHECK((int64_t)out->numel_ == rows * cols / 2, "out must hold rows x cols/2 bytes");
    AB_CHECK(((uintptr_t)out->ptr & 15) == 0, "out must be 16-byte aligned");
    int64_t ld_scale = gpr, scale_cols = 0;
    if (shuffle_scale) {
        AB_CHECK(scales->ndim == 2, "shuffled scales must be 2-D");
        const int64_t sr = scales->shape[0];
        scale_cols = scales->shape[1];
        AB_CHECK(sr % 32 == 0 && sr >= rows && scale_cols % 8 == 0 && scale_cols >= gpr,
                 "shuffled scales must be [rows padded to 32, cols/32 padded to 8]");
    } else {
        AB_CHECK((int64_t)scales->numel_ == rows * gpr, "scales must be [rows, cols/32]");
    }
    const int* nr = nullptr;
    if (num_rows) {
        need_dtype(num_rows, AITER_DTYPE_i32, "num_rows");
        nr = (const int*)num_rows->ptr;
        AB_CHECK(num_rows_factor >= 1, "num_rows_factor must be >= 1");
    }
    if (rows == 0) return;
    DeviceGuard dg(input->device_id);
    const int grid = grid_for(rows * gpr, input->device_id);
    by_dtype(input->dtype_, [&](auto tag) {
        using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
        mxfp4_quant_kernel<T><<<grid, kThreads, 0, as_stream(stream)>>>(
            (const T*)input->ptr, rows, row_stride(input), gpr, (uint8_t*)out->ptr, cols / 2, (uint8_t*)scales->ptr,
            ld_scale, shuffle_scale ? 1 : 0, scale_cols, nr, num_rows_factor);
    });
    check_launch("dynamic_per_group_scaled_quant_fp4");
}

AB_ENTRY(mxfp4_moe_sort_hip,
         (aiter_tensor_t * out_scale, aiter_tensor_t* scale, aiter_tensor_t* sorted_ids, aiter_tensor_t* num_valid_ids,
          int64_t token_num, int64_t cols, void* stream),
         (out_scale, scale, sorted_ids, num_valid_ids, token_num, cols, stream)) {
    using namespace ab;
    need(out_scale, "out_scale");
    need(scale, "scale");
    need(sorted_ids, "sorted_ids");
    need(num_valid_ids, "num_valid_ids");
    need_dtype(sorted_ids, AITER_DTYPE_i32, "sorted_ids");
    need_dtype(num_valid_ids, AITER_DTYPE_i32, "num_valid_ids");
    for (aiter_tensor_t* t : {out_scale, scale})
        AB_CHECK(t->dtype_ == AITER_DTYPE_fp8_e8m0 || t->dtype_ == AITER_DTYPE_u8, "scales must be e8m0");
    need_contig(out_scale, "out_scale");
    need_contig(scale, "scale");
    AB_CHECK(cols > 0 && cols % 256 == 0, "cols must be a positive multiple of 256 (scale columns % 8 == 0)");
    AB_CHECK(token_num > 0 && token_num < (1 << 24), "bad token_num");
    const int64_t sc = cols / 32;
    AB_CHECK((int64_t)scale->numel_ % sc == 0, "scale must be [rows, cols/32]");
    const int64_t src_rows = (int64_t)scale->numel_ / sc;
    AB_CHECK(src_rows % token_num == 0, "scale rows must be token_num or token_num * topk");
    const int64_t topk = src_rows / token_num;
    const int64_t max_pad = (int64_t)sorted_ids->numel_;
    const int64_t out_rows = (max_pad + 31) / 32 * 32;
    AB_CHECK((int64_t)out_scale->numel_ == out_rows * sc, "out_scale must be [ceil(len(sorted_ids)/32)*32, cols/32]");
    AB_CHECK(((uintptr_t)out_scale->ptr & 3) == 0, "out_scale must be 4-byte aligned");
    if (out_rows == 0) return;
    DeviceGuard dg(out_scale->device_id);
    const int grid = grid_for(out_rows * sc / 4, out_scale->device_id);
    mxfp4_moe_sort_kernel<__nv_bfloat16><<<grid, kThreads, 0, as_stream(stream)>>>(
        (uint8_t*)out_scale->ptr, out_rows, sc, (const int*)sorted_ids->ptr, max_pad, (const int*)num_valid_ids->ptr,
        token_num, topk, src_rows, (const uint8_t*)scale->ptr, sc, nullptr, 0);
    check_launch("mxfp4_moe_sort_hip");
}

AB_ENTRY(fused_dynamic_mxfp4_quant_moe_sort_hip,
         (aiter_tensor_t * out, aiter_tensor_t* scales, aiter_tensor_t* input, aiter_tensor_t* sorted_ids,
          aiter_tensor_t* num_valid_ids, int64_t token_num, int64_t block_m, int64_t group_size, void* stream),
         (out, scales, input, sorted_ids, num_valid_ids, token_num, block_m, group_size, stream)) {
    using namespace ab;
    check_input(input, "input");
    need(out, "out");
    need(scales, "scales");
    need(sorted_ids, "sorted_ids");
    need(num_valid_ids, "num_valid_ids");
    need_dtype(sorted_ids, AITER_DTYPE_i32, "sorted_ids");
    need_dtype(num_valid_ids, AITER_DTYPE_i32, "num_valid_ids");
    AB_CHECK(group_size == 32, "group_size must be 32 (MXFP4), got ", group_size);
    AB_CHECK(block_m > 0, "block_m must be positive");
    AB_CHECK(out->dtype_ == AITER_DTYPE_fp4x2 || out->dtype_ == AITER_DTYPE_u8, "out must be fp4x2");
    AB_CHECK(scales->dtype_ == AITER_DTYPE_fp8_e8m0 || scales->dtype_ == AITER_DTYPE_u8, "scales must be e8m0");
    need_contig(out, "out");
    need_contig(scales, "scales");
    const int64_t cols = input->shape[input->ndim - 1];
    const int64_t rows = (int64_t)input->numel_ / cols;
    const int64_t gpr = cols / 32;
    AB_CHECK(cols % 256 == 0, "model_dim must be a multiple of 256");
    AB_CHECK(token_num > 0 && token_num < (1 << 24) && rows % token_num == 0,
             "input rows must be token_num (stage 1) or token_num * topk (stage 2)");
    AB_CHECK((int64_t)out->numel_ == rows * cols / 2 && ((uintptr_t)out->ptr & 15) == 0,
             "out must be [rows, cols/2], 16-byte aligned");
    const int64_t max_pad = (int64_t)sorted_ids->numel_;
    const int64_t out_rows = (max_pad + 31) / 32 * 32;
    AB_CHECK((int64_t)scales->numel_ == out_rows * gpr && ((uintptr_t)scales->ptr & 3) == 0,
             "scales must be [ceil(len(sorted_ids)/32)*32, cols/32], 4-byte aligned");
    if (rows == 0) return;
    DeviceGuard dg(input->device_id);
    const int qb = grid_for(rows * gpr, input->device_id);
    const int sb = grid_for(out_rows * gpr / 4, input->device_id);
    by_dtype(input->dtype_, [&](auto tag) {
        using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
        mxfp4_quant_sort_kernel<T><<<qb + sb, kThreads, 0, as_stream(stream)>>>(
            (const T*)input->ptr, rows, row_stride(input), gpr, (uint8_t*)out->ptr, cols / 2, qb,
            (uint8_t*)scales->ptr, out_rows, (const int*)sorted_ids->ptr, max_pad, (const int*)num_valid_ids->ptr,
            token_num, rows / token_num);
    });
    check_launch("fused_dynamic_mxfp4_quant_moe_sort_hip");
}
