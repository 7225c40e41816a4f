// Codecs of the quick allreduce (the quantised two-shot allreduce), shared by the
// kernel in quick_reduce.cu.  Value semantics follow the reference's QuickReduce
// codecs (csrc/include/quick_all_reduce.cuh:25-579, helpers in
// quick_all_reduce_base.h:187-355); the byte layout of an encoded row is this
// library's own.
//
// Arithmetic type T (fp16 or bf16): every operation is done in fp32 and rounded
// once to T.  For +, x and reciprocal that equals T's own correctly rounded
// operation (the fp32 intermediate has at least 2p + 2 bits for T's p-bit
// significand, so double rounding is innocuous).  fp16 results that overflow from
// finite operands saturate at +-65504, as the reference runs with FP16_OVFL set
// (quick_all_reduce_base.h:102-113).
//
// A thread holds 8 consecutive elements (16 bytes) of an "atom row" of 256
// threads.  Eight consecutive lanes (64 elements) share a pair of scales: one for
// the even elements, one for the odd ones (the two halves of a T pair in the
// reference, quick_all_reduce_base.h:319-349).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <math.h>
#include <stdint.h>

namespace qr {

enum Level : int { kFP = 0, kFP8 = 1, kINT6 = 2, kINT4 = 3 };

constexpr int kThreads = 256;                     // threads per CTA (one atom row)
constexpr int kAtoms = 8;                         // atom rows per tile
constexpr int kRowElems = kThreads * 8;           // 2048 elements per atom row
constexpr int kTileElems = kAtoms * kRowElems;    // 16384 elements per tile
constexpr int kTileBytes = kTileElems * 2;        // 32 KB of T per tile

// Encoded atom row: codes of 256 threads, then (for the quantised levels) the
// 32 scale pairs of the row's 8-lane groups.
//   FP:   16 B of T per thread                          = 4096 B
//   FP8:  8 e4m3 codes per thread (2048 B) + 32 x 4 B   = 2176 B
//   INT4: 8 nibbles per thread (1024 B) + 32 x 4 B      = 1152 B
//   INT6: low nibbles (1024 B) + high 2-bit pairs (512 B) + 32 x 4 B = 1664 B
template <int L>
struct RowLayout;
template <>
struct RowLayout<kFP> {
    static constexpr int kScaleOff = 0, kRowBytes = kThreads * 16;
};
template <>
struct RowLayout<kFP8> {
    static constexpr int kScaleOff = kThreads * 8, kRowBytes = kScaleOff + (kThreads / 8) * 4;
};
template <>
struct RowLayout<kINT4> {
    static constexpr int kScaleOff = kThreads * 4, kRowBytes = kScaleOff + (kThreads / 8) * 4;
};
template <>
struct RowLayout<kINT6> {
    static constexpr int kHiOff = kThreads * 4;
    static constexpr int kScaleOff = kHiOff + kThreads * 2, kRowBytes = kScaleOff + (kThreads / 8) * 4;
};

__host__ __device__ inline float rcp_rn(float x) {
#ifdef __CUDA_ARCH__
    return __frcp_rn(x);
#else
    return 1.0f / x;
#endif
}

template <typename T>
struct Arith;

template <>
struct Arith<__half> {
    using Pair = __half2;
    // scale epsilon and the FP8 scale factor 1/240 as fp16 bit patterns
    // (quick_all_reduce.cuh:92, :419-421)
    static constexpr uint16_t kEpsBits = 0x0001, kInv240Bits = 0x1C44;
    __host__ __device__ static float round(float f) {
        if (isfinite(f)) f = fminf(fmaxf(f, -65504.0f), 65504.0f);
        return __half2float(__float2half_rn(f));
    }
    __host__ __device__ static float from_bits(uint16_t b) {
        __half_raw r;
        r.x = b;
        return __half2float(__half(r));
    }
    __host__ __device__ static uint16_t to_bits(float f) {  // f already an fp16 value
        __half_raw r = __half(__float2half_rn(f));
        return r.x;
    }
};

template <>
struct Arith<__nv_bfloat16> {
    using Pair = __nv_bfloat162;
    static constexpr uint16_t kEpsBits = 0x33D7, kInv240Bits = 0x3B88;
    __host__ __device__ static float round(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
    __host__ __device__ static float from_bits(uint16_t b) {
        __nv_bfloat16_raw r;
        r.x = b;
        return __bfloat162float(__nv_bfloat16(r));
    }
    __host__ __device__ static uint16_t to_bits(float f) {
        __nv_bfloat16_raw r = __nv_bfloat16(__float2bfloat16_rn(f));
        return r.x;
    }
};

// Integer levels: code range [lo, hi] and the scale factor -1 / 2^(bits-1)
// (quick_all_reduce.cuh:89-98, :244-253).
template <int L>
struct IntRange;
template <>
struct IntRange<kINT4> {
    static constexpr float kLo = -8.0f, kHi = 7.0f, kFactor = -0.125f;
    static constexpr int kBias = 8;
};
template <>
struct IntRange<kINT6> {
    static constexpr float kLo = -32.0f, kHi = 31.0f, kFactor = -0.03125f;
    static constexpr int kBias = 32;
};

// Decoding scale of a group from its signed extreme m (INT levels) or its
// largest magnitude a (FP8).
template <typename T, int L>
__host__ __device__ inline float decoding_scale(float m) {
    if constexpr (L == kFP8)
        return Arith<T>::round(m * Arith<T>::from_bits(Arith<T>::kInv240Bits));
    else
        return Arith<T>::round(m * IntRange<L>::kFactor);
}

// Encoding scale T(1 / T(dec + eps)); 1/0 stays infinite.
template <typename T>
__host__ __device__ inline float encoding_scale(float dec) {
    const float s = Arith<T>::round(dec + Arith<T>::from_bits(Arith<T>::kEpsBits));
    if (s == 0.0f) return copysignf(INFINITY, s);
    return Arith<T>::round(rcp_rn(s));
}

// Code of one element for the INT levels (biased into [0, 2^bits)).
template <typename T, int L>
__host__ __device__ inline uint32_t int_code(float x, float enc) {
    float w = Arith<T>::round(x * enc);
    w = fminf(fmaxf(w, IntRange<L>::kLo), IntRange<L>::kHi);  // a NaN takes the bound
    return (uint32_t)((int)rintf(w) + IntRange<L>::kBias);
}

template <typename T, int L>
__host__ __device__ inline float int_value(uint32_t code, float dec) {
    return Arith<T>::round((float)((int)code - IntRange<L>::kBias) * dec);
}

template <typename T>
__host__ __device__ inline uint8_t fp8_code(float x, float enc) {
    const float w = Arith<T>::round(x * enc);
    return (uint8_t)__nv_cvt_float_to_fp8(w, __NV_SATFINITE, __NV_E4M3);
}

template <typename T>
__host__ __device__ inline float fp8_value(uint8_t code, float dec) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)code, __NV_E4M3);
    return Arith<T>::round(__half2float(__half(h)) * dec);
}

// One thread's encoded atom: up to 16 B of codes and its group's scale pair.
struct Enc {
    uint4 code;
    uint32_t scale;
};

// Pack / unpack one thread's 8 T values.
template <typename T>
__host__ __device__ inline uint4 pack_t(const float (&x)[8]) {
    uint32_t w[4];
    for (int i = 0; i < 4; ++i)
        w[i] = (uint32_t)Arith<T>::to_bits(x[2 * i]) | ((uint32_t)Arith<T>::to_bits(x[2 * i + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__host__ __device__ inline void unpack_t(uint4 v, float (&x)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    for (int i = 0; i < 4; ++i) {
        x[2 * i] = Arith<T>::from_bits((uint16_t)(w[i] & 0xFFFF));
        x[2 * i + 1] = Arith<T>::from_bits((uint16_t)(w[i] >> 16));
    }
}

// Encode 8 elements given the group's scales (dec_even, dec_odd), already
// reduced over the 8 lanes.
template <typename T, int L>
__host__ __device__ inline Enc encode_with(const float (&x)[8], float dec_e, float dec_o) {
    Enc e{};
    const float enc_e = encoding_scale<T>(dec_e), enc_o = encoding_scale<T>(dec_o);
    if constexpr (L == kFP8) {
        uint32_t lo = 0, hi = 0;
        for (int j = 0; j < 4; ++j) lo |= (uint32_t)fp8_code<T>(x[j], (j & 1) ? enc_o : enc_e) << (8 * j);
        for (int j = 4; j < 8; ++j) hi |= (uint32_t)fp8_code<T>(x[j], (j & 1) ? enc_o : enc_e) << (8 * (j - 4));
        e.code = make_uint4(lo, hi, 0, 0);
    } else {
        uint32_t nib = 0, top = 0;
        for (int j = 0; j < 8; ++j) {
            const uint32_t c = int_code<T, L>(x[j], (j & 1) ? enc_o : enc_e);
            nib |= (c & 0xF) << (4 * j);
            top |= (c >> 4) << (2 * j);  // INT6 only: the high two bits
        }
        e.code = make_uint4(nib, top, 0, 0);
    }
    e.scale = (uint32_t)Arith<T>::to_bits(dec_e) | ((uint32_t)Arith<T>::to_bits(dec_o) << 16);
    return e;
}

// Decode 8 elements from their codes and scale pair.
template <typename T, int L>
__host__ __device__ inline void decode(const Enc& e, float (&x)[8]) {
    if constexpr (L == kFP) {
        unpack_t<T>(e.code, x);
        return;
    } else {
        const float dec_e = Arith<T>::from_bits((uint16_t)(e.scale & 0xFFFF));
        const float dec_o = Arith<T>::from_bits((uint16_t)(e.scale >> 16));
        for (int j = 0; j < 8; ++j) {
            const float dec = (j & 1) ? dec_o : dec_e;
            if constexpr (L == kFP8) {
                const uint32_t w = j < 4 ? e.code.x : e.code.y;
                x[j] = fp8_value<T>((uint8_t)(w >> (8 * (j & 3))), dec);
            } else {
                uint32_t c = (e.code.x >> (4 * j)) & 0xF;
                if constexpr (L == kINT6) c |= ((e.code.y >> (2 * j)) & 0x3) << 4;
                x[j] = int_value<T, L>(c, dec);
            }
        }
    }
}

// Per-thread group statistics before the 8-lane reduction: the FP8 level needs
// max |x| (even, odd); the INT levels the max and min (even, odd).
struct Stats {
    float a_e, a_o, b_e, b_o;
};

template <int L>
__host__ __device__ inline Stats local_stats(const float (&x)[8]) {
    Stats s;
    if constexpr (L == kFP8) {
        s.a_e = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[2])), fmaxf(fabsf(x[4]), fabsf(x[6])));
        s.a_o = fmaxf(fmaxf(fabsf(x[1]), fabsf(x[3])), fmaxf(fabsf(x[5]), fabsf(x[7])));
        s.b_e = s.b_o = 0.0f;
    } else {
        s.a_e = fmaxf(fmaxf(x[0], x[2]), fmaxf(x[4], x[6]));
        s.a_o = fmaxf(fmaxf(x[1], x[3]), fmaxf(x[5], x[7]));
        s.b_e = fminf(fminf(x[0], x[2]), fminf(x[4], x[6]));
        s.b_o = fminf(fminf(x[1], x[3]), fminf(x[5], x[7]));
    }
    return s;
}

// Merge the statistics of two lanes.
template <int L>
__host__ __device__ inline Stats merge_stats(const Stats& p, const Stats& q) {
    Stats s;
    s.a_e = fmaxf(p.a_e, q.a_e);
    s.a_o = fmaxf(p.a_o, q.a_o);
    s.b_e = fminf(p.b_e, q.b_e);
    s.b_o = fminf(p.b_o, q.b_o);
    return s;
}

// Scales (dec_even, dec_odd) of a group from its merged statistics.
template <typename T, int L>
__host__ __device__ inline void group_scales(const Stats& s, float& dec_e, float& dec_o) {
    if constexpr (L == kFP8) {
        dec_e = decoding_scale<T, L>(s.a_e);
        dec_o = decoding_scale<T, L>(s.a_o);
    } else {
        // the signed extreme: the max when its magnitude is strictly larger, else the min
        const float m_e = fabsf(s.a_e) > fabsf(s.b_e) ? s.a_e : s.b_e;
        const float m_o = fabsf(s.a_o) > fabsf(s.b_o) ? s.a_o : s.b_o;
        dec_e = decoding_scale<T, L>(m_e);
        dec_o = decoding_scale<T, L>(m_o);
    }
}

}  // namespace qr
