// Custom allreduce over CUDA IPC peer memory (NVLink 5 / NVSwitch): the B200
// replacement of the reference's HIP-IPC CustomAllreduce
// (csrc/include/custom_all_reduce.cuh:150-555, aiter/dist/device_communicators/
// custom_all_reduce.py:243-739).
//
// Every rank owns one cudaMalloc'd region, exported with cudaIpcGetMemHandle and
// opened by every peer:
//   [ Signal (flags written by peers, own call counters) | staging 0 | 1 | 2 ]
// Eager call n stages its input in buffer n % 2 (host-side count of eager calls).
// A rank starts call n+2 (same buffer) only after the start barrier of call n+1,
// which every peer reaches only after finishing call n, so nothing a slow peer
// still reads is overwritten.  Calls captured into a CUDA graph use buffer 2, do
// not count as eager calls, and end with a third barrier: no rank leaves the call
// before every peer has finished reading its buffer, so a replay may run between
// any two eager calls or right after another replay.
//
// Epochs live in device memory: CTA b of a call increments its own counter[b]
// (only CTA b of this rank touches it, launches are stream-ordered), so replayed
// graphs and eager calls share one monotonic sequence per CTA index, identical on
// all ranks because all ranks launch the same grid for the same call.
// Barriers are per CTA: CTA b of rank r writes its epoch into flag[phase][b][r] of
// every peer (st.release.sys) and waits until its own flag[phase][b][p] has reached
// that epoch for all peers (ld.acquire.sys, wrap-safe >=, bounded).  All ranks
// partition the data identically per CTA, so CTA b only ever reads what peer CTAs b
// wrote before the barrier.
//   one-shot : copy -> barrier -> out = sum over ranks (rank order 0..W-1)
//   two-shot : copy -> barrier -> reduce own segment in place -> barrier -> gather
//              every segment from its owner.
// Sums accumulate in fp32 in rank order, so every rank gets identical bits.
// Every wait gives up after 2 s, sets the device error word and returns.
#include <mutex>
#include <vector>

#include "gemm_bf16.cuh"

namespace {

using namespace ipc;

constexpr int kMaxBlocks = 128;  // grid cap of the allreduce kernels
constexpr int kThreads = 512;
static_assert(kMaxBlocks <= kFlagBlocks, "allreduce CTAs need their own flags");

// 16-byte packs of each element type: bf16 and fp16 carry 8 values, fp32 4; sums
// accumulate in fp32 and round once to the element type.
template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
    __device__ static void acc(float (&a)[8], uint4 v) { acc8(a, v); }
    __device__ static uint4 pack(const float (&a)[8]) { return pack8(a); }
};
template <>
struct Elem<__half> {
    __device__ static void acc(float (&a)[8], uint4 v) {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            a[2 * i] += f.x;
            a[2 * i + 1] += f.y;
        }
    }
    __device__ static uint4 pack(const float (&a)[8]) {
        uint4 v;
        __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
        return v;
    }
};
template <>
struct Elem<float> {
    __device__ static void acc(float (&a)[8], uint4 v) {
        a[0] += __uint_as_float(v.x);
        a[1] += __uint_as_float(v.y);
        a[2] += __uint_as_float(v.z);
        a[3] += __uint_as_float(v.w);
    }
    __device__ static uint4 pack(const float (&a)[8]) {
        return make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
    }
};

// n16: number of 16-byte packs (8 bf16 / fp16, 4 fp32).  `in` may equal the staging buffer
// (zero-copy producers), then the copy is skipped.  W (the world size) is a
// template parameter so that the peer loops unroll and every thread keeps
// U * W independent 16-byte loads in flight (U packs per thread per step).
template <typename T, int W>
__global__ void __launch_bounds__(kThreads)
allreduce_kernel(Peers P, int rank, int buffer, const uint4* __restrict__ in, uint4* __restrict__ out,
                      int64_t n16, int two_shot, int end_barrier) {
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) {
        uint32_t* ctr = &P.sig[rank]->counter[blockIdx.x];
        s_epoch = *ctr + 1;
        *ctr = s_epoch;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    constexpr int U = W >= 8 ? 1 : 8 / W;
    uint4* mine = reinterpret_cast<uint4*>(P.buf[buffer][rank]);
    const uint4* bufs[W];
#pragma unroll
    for (int p = 0; p < W; ++p) bufs[p] = reinterpret_cast<const uint4*>(P.buf[buffer][p]);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // Packs are split into `nseg` segments and pack i of segment s always goes to
    // thread (i - lo_s) mod stride, in the copy, the reduce and the gather, on every
    // rank.  A CTA therefore only reads packs that the same CTA index wrote on the
    // peers before the barrier it waited on.
    const int nseg = two_shot ? W : 1;
    const int64_t seg = (n16 + nseg - 1) / nseg;
    if (in != mine) {
        for (int s = 0; s < nseg; ++s) {
            const int64_t lo = (int64_t)s * seg, hi = min(n16, lo + seg);
            for (int64_t i = lo + tid; i < hi; i += 4 * stride) {
                uint4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i + u * stride < hi) v[u] = in[i + u * stride];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i + u * stride < hi) mine[i + u * stride] = v[u];
            }
        }
    }
    if (!block_barrier(P, rank, W, 0, epoch)) return;
    // sum of packs [lo, hi) over ranks in rank order -> dst
    auto reduce_range = [&](int64_t lo, int64_t hi, uint4* dst) {
        for (int64_t i = lo + tid; i < hi; i += U * stride) {
            uint4 v[U][W];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int p = 0; p < W; ++p)
                    if (i + u * stride < hi) v[u][p] = ld_cg(bufs[p] + i + u * stride);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (i + u * stride < hi) {
                    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
                    for (int p = 0; p < W; ++p) Elem<T>::acc(a, v[u][p]);
                    dst[i + u * stride] = Elem<T>::pack(a);
                }
            }
        }
    };
    if (!two_shot) {
        reduce_range(0, n16, out);
        if (end_barrier) block_barrier(P, rank, W, 2, epoch);
        return;
    }
    // rank r reduces segment r in place
    reduce_range((int64_t)rank * seg, min(n16, (int64_t)(rank + 1) * seg), mine);
    if (!block_barrier(P, rank, W, 1, epoch)) return;
    for (int s = 0; s < W; ++s) {
        const int o = (rank + s) % W;  // start with the own segment, spread peer traffic
        const int64_t lo = (int64_t)o * seg, hi = min(n16, lo + seg);
        const uint4* src = bufs[0];
#pragma unroll
        for (int p = 1; p < W; ++p)
            if (p == o) src = bufs[p];  // select, keeps bufs[] in registers
        for (int64_t i = lo + tid; i < hi; i += 8 * stride) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i + u * stride < hi) v[u] = ld_cg(src + i + u * stride);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i + u * stride < hi) out[i + u * stride] = v[u];
        }
    }
    if (end_barrier) block_barrier(P, rank, W, 2, epoch);
}

// ---------------------------------------------------------------------------
// All-gather and reduce-scatter over the same staging buffers and per-CTA barriers
// (the reference's custom all-gather / reduce-scatter kernels,
// csrc/include/custom_all_reduce.cuh:678-800).  As in the allreduce, pack i of the
// staged input is copied, and later read on every rank, by thread (i - lo) mod stride,
// so a CTA reads only what the same CTA index of each peer staged before the barrier.

// out = every rank's input in rank order: dim 0 (c16 == 0: out [W, n16 packs]) or the
// last dim (c16 packs per input row: out row r = [rank 0's row r | rank 1's | ...]).
template <int W>
__global__ void __launch_bounds__(kThreads)
allgather_kernel(Peers P, int rank, int buffer, const uint4* __restrict__ in, uint4* __restrict__ out, int64_t n16,
                 int64_t c16, int end_barrier) {
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) s_epoch = next_epoch(P, rank);
    __syncthreads();
    const uint32_t epoch = s_epoch;
    uint4* mine = reinterpret_cast<uint4*>(P.buf[buffer][rank]);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (in != mine)
        for (int64_t i = tid; i < n16; i += stride) mine[i] = in[i];
    if (!block_barrier(P, rank, W, 0, epoch)) return;
#pragma unroll 1
    for (int s = 0; s < W; ++s) {
        const int p = (rank + s) % W;  // own rows first, then spread the peer traffic
        const uint4* src = reinterpret_cast<const uint4*>(P.buf[buffer][p]);
        for (int64_t i = tid; i < n16; i += 4 * stride) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i + u * stride < n16) v[u] = ld_cg(src + i + u * stride);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = i + u * stride;
                if (j < n16) {
                    const int64_t o = c16 == 0 ? (int64_t)p * n16 + j : (j / c16) * (W * c16) + p * c16 + j % c16;
                    out[o] = v[u];
                }
            }
        }
    }
    if (end_barrier) block_barrier(P, rank, W, 2, epoch);
}

// out = segment `rank` (n16 / W packs) of the sum over ranks of the inputs, summed
// in rank order in fp32 and rounded once (the first phase of the two-shot allreduce).
template <typename T, int W>
__global__ void __launch_bounds__(kThreads)
reduce_scatter_kernel(Peers P, int rank, int buffer, const uint4* __restrict__ in, uint4* __restrict__ out,
                      int64_t n16, int end_barrier) {
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) s_epoch = next_epoch(P, rank);
    __syncthreads();
    const uint32_t epoch = s_epoch;
    uint4* mine = reinterpret_cast<uint4*>(P.buf[buffer][rank]);
    const uint4* bufs[W];
#pragma unroll
    for (int p = 0; p < W; ++p) bufs[p] = reinterpret_cast<const uint4*>(P.buf[buffer][p]);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t seg = n16 / W;
    if (in != mine) {
        for (int s = 0; s < W; ++s) {
            const int64_t lo = (int64_t)s * seg;
            for (int64_t i = lo + tid; i < lo + seg; i += stride) mine[i] = in[i];
        }
    }
    if (!block_barrier(P, rank, W, 0, epoch)) return;
    const int64_t lo = (int64_t)rank * seg;
    for (int64_t i = lo + tid; i < lo + seg; i += stride) {
        uint4 v[W];
#pragma unroll
        for (int p = 0; p < W; ++p) v[p] = ld_cg(bufs[p] + i);
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int p = 0; p < W; ++p) Elem<T>::acc(a, v[p]);
        out[i - lo] = Elem<T>::pack(a);
    }
    if (end_barrier) block_barrier(P, rank, W, 2, epoch);
}

// ---------------------------------------------------------------------------
// fp8-quantised two-shot allreduce of fp16 data: the reference's allReduceQuantFp8
// (csrc/include/custom_all_reduce.cuh:1018-1088), used with open_fp8_quant for fp16
// messages of at least 128 * 2048 elements (csrc/kernels/custom_all_reduce.cu:90-96).
// The n8 packs (8 halves) are cut into W segments of n8 / W packs, the last rank
// taking the remainder.  Owner rank r sums segment r over the ranks in the rotated
// order r, r+1, ..., r-1 in fp32, rounds to fp16 and writes that to its own output;
// then it quantises the sum in groups of G = 8 * gp elements aligned to the segment
// start, scale = fp16(amax / 448), code = e4m3(x / scale) (a zero scale gives zero
// codes; the reference would produce NaN), into its staging buffer after the input
// (codes at q_off, fp16 scales at s_off).  After a barrier every rank decodes the
// other segments, fp16(code * scale).  Only the all-gather half moves fp8 (half the
// bytes); each rank's own segment is exact, the others carry the fp8 rounding.
// Pack i of segment s is handled by thread (i - lo_s) mod stride on every rank, so
// a CTA reads only what the same CTA index of each peer wrote before the barrier;
// the gp lanes of a group are consecutive lanes of one warp.
template <int W>
__global__ void __launch_bounds__(kThreads)
allreduce_fp8q_kernel(Peers P, int rank, int buffer, const uint4* __restrict__ in, uint4* __restrict__ out,
                      int64_t n8, int gp, int64_t q_off, int64_t s_off, int end_barrier) {
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) s_epoch = next_epoch(P, rank);
    __syncthreads();
    const uint32_t epoch = s_epoch;
    uint4* mine = reinterpret_cast<uint4*>(P.buf[buffer][rank]);
    const int lane = threadIdx.x & 31;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t part = n8 / W;
    auto seg_lo = [&](int s) -> int64_t { return (int64_t)s * part; };
    auto seg_hi = [&](int s) -> int64_t { return s == W - 1 ? n8 : (int64_t)(s + 1) * part; };
    if (in != mine)
        for (int s = 0; s < W; ++s)
            for (int64_t i = seg_lo(s) + tid; i < seg_hi(s); i += stride) mine[i] = in[i];
    if (!block_barrier(P, rank, W, 0, epoch)) return;
    {
        const int64_t lo = seg_lo(rank), hi = seg_hi(rank);
        uint8_t* qbase = P.buf[buffer][rank] + q_off;
        __half* sbase = reinterpret_cast<__half*>(P.buf[buffer][rank] + s_off);
        // warp-uniform trip count: every lane takes part in the group shuffles
        for (int64_t i0 = lo + tid - lane; i0 < hi; i0 += stride) {
            const int64_t i = i0 + lane;
            const bool active = i < hi;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (active) {
#pragma unroll
                for (int j = 0; j < W; ++j)
                    Elem<__half>::acc(a, ld_cg(reinterpret_cast<const uint4*>(P.buf[buffer][(rank + j) % W]) + i));
            }
            const uint4 h = Elem<__half>::pack(a);
            const __half* hv = reinterpret_cast<const __half*>(&h);
            float amax = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(__half2float(hv[e])));
            for (int o = gp >> 1; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const __half sh = __float2half_rn(amax / 448.0f);
            const float sf = __half2float(sh);
            if (active) {
                out[i] = h;
                uint32_t q[2];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    float4 f;
                    f.x = sf == 0.f ? 0.f : __half2float(hv[4 * k]) / sf;
                    f.y = sf == 0.f ? 0.f : __half2float(hv[4 * k + 1]) / sf;
                    f.z = sf == 0.f ? 0.f : __half2float(hv[4 * k + 2]) / sf;
                    f.w = sf == 0.f ? 0.f : __half2float(hv[4 * k + 3]) / sf;
                    __nv_fp8x4_e4m3 f4(f);
                    q[k] = *reinterpret_cast<uint32_t*>(&f4);
                }
                *reinterpret_cast<uint2*>(qbase + (i - lo) * 8) = make_uint2(q[0], q[1]);
                if ((i - lo) % gp == 0) sbase[(i - lo) / gp] = sh;
            }
        }
    }
    if (!block_barrier(P, rank, W, 1, epoch)) return;
    for (int d = 1; d < W; ++d) {
        const int s = (rank + d) % W;
        const int64_t lo = seg_lo(s), hi = seg_hi(s);
        const uint8_t* qsrc = P.buf[buffer][s] + q_off;
        const uint8_t* ssrc = P.buf[buffer][s] + s_off;
        for (int64_t i = lo + tid; i < hi; i += stride) {
            const uint2 qv = ld_cg8(qsrc + (i - lo) * 8);
            const unsigned short sb = *reinterpret_cast<const volatile unsigned short*>(ssrc + ((i - lo) / gp) * 2);
            const float sf = __half2float(__ushort_as_half(sb));
            const __nv_fp8x4_e4m3* q4 = reinterpret_cast<const __nv_fp8x4_e4m3*>(&qv);
            float a[8];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float4 f = static_cast<float4>(q4[k]);
                a[4 * k] = f.x * sf;
                a[4 * k + 1] = f.y * sf;
                a[4 * k + 2] = f.z * sf;
                a[4 * k + 3] = f.w * sf;
            }
            out[i] = Elem<__half>::pack(a);
        }
    }
    if (end_barrier) block_barrier(P, rank, W, 2, epoch);
}

// ---------------------------------------------------------------------------
// Allreduce fused with the residual add and RMSNorm that follow it in a TP layer
// (fused_allreduce_rmsnorm / _quant, csrc/include/custom_all_reduce.cuh:1187-1250,
// 1420-1500 in the reference).  One-shot over rows: CTA b stages and later reduces
// rows b, b + grid, ..., so it only reads rows the same CTA index of every peer
// staged before the barrier.  Per row, in fp32:
//   ar      = bf16(sum over ranks in rank order)      (the plain allreduce result)
//   x       = ar + res_inp;  res_out = bf16(x)
//   r       = rsqrt(mean(x^2) + eps)
//   out     = bf16(x * w * r)                         (QUANT: y = x * w * r, then
//             per-row fp8: scale = amax(|y|) / 448 (0 -> 1), q = fp8(y / scale))
template <int W, bool QUANT>
__global__ void __launch_bounds__(kThreads)
allreduce_rmsnorm_kernel(Peers P, int rank, int buffer, const uint4* __restrict__ in,
                         const uint4* __restrict__ res_in, uint4* __restrict__ res_out, void* __restrict__ out,
                         float* __restrict__ scale_out, const uint4* __restrict__ weight, int64_t rows, int ppr,
                         float eps, int end_barrier, int two_shot) {
    constexpr int MAXP = 4;  // packs of 8 per thread: hidden <= 4 * 8 * kThreads
    __shared__ uint32_t s_epoch;
    __shared__ float s_red[kThreads / 32];
    if (threadIdx.x == 0) {
        uint32_t* ctr = &P.sig[rank]->counter[blockIdx.x];
        s_epoch = *ctr + 1;
        *ctr = s_epoch;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    uint4* mine = reinterpret_cast<uint4*>(P.buf[buffer][rank]);
    const uint4* bufs[W];
#pragma unroll
    for (int p = 0; p < W; ++p) bufs[p] = reinterpret_cast<const uint4*>(P.buf[buffer][p]);
    if (in != mine)
        for (int64_t row = blockIdx.x; row < rows; row += gridDim.x)
            for (int p = threadIdx.x; p < ppr; p += blockDim.x) mine[row * ppr + p] = in[row * ppr + p];
    if (!block_barrier(P, rank, W, 0, epoch)) return;
    // the allreduce of pack i: every rank's staged pack summed in rank order, bf16
    auto sum_pack = [&](int64_t i) -> uint4 {
        uint4 v[W];
#pragma unroll
        for (int r = 0; r < W; ++r) v[r] = ld_cg(bufs[r] + i);
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int r = 0; r < W; ++r) acc8(a, v[r]);
        return pack8(a);
    };
    // two-shot: row b + k * grid belongs to rank k % W, which reduces it in place in its
    // staging buffer (only it reads that row of its buffer before the next barrier);
    // after the barrier every rank takes the reduced row from its owner
    if (two_shot) {
        for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
            if ((row / gridDim.x) % W != rank) continue;
            for (int p = threadIdx.x; p < ppr; p += blockDim.x) mine[row * ppr + p] = sum_pack(row * ppr + p);
        }
        if (!block_barrier(P, rank, W, 1, epoch)) return;
    }
    const float inv_n = 1.0f / (float)(ppr * 8);
    auto block_sum = [&](float v, bool is_max) -> float {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float t = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, t) : v + t;
        }
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
        __syncthreads();
        float r = is_max ? 0.f : 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = is_max ? fmaxf(r, s_red[i]) : r + s_red[i];
        __syncthreads();  // s_red is reused by the next reduction
        return r;
    };
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        float x[MAXP][8];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < MAXP; ++j) {
            const int p = threadIdx.x + j * blockDim.x;
            if (p < ppr) {
                const int64_t i = row * ppr + p;
                // the allreduce result, rounded to bf16
                const uint4 ar = two_shot ? ld_cg(bufs[(row / gridDim.x) % W] + i) : sum_pack(i);
                const uint4 rs = res_in[i];
                const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&ar);
                const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rs);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fa = __bfloat1622float2(ah[e]), fr = __bfloat1622float2(rh[e]);
                    x[j][2 * e] = fa.x + fr.x;
                    x[j][2 * e + 1] = fa.y + fr.y;
                    ss += x[j][2 * e] * x[j][2 * e] + x[j][2 * e + 1] * x[j][2 * e + 1];
                }
                res_out[i] = pack8(x[j]);
            }
        }
        const float rinv = rsqrtf(block_sum(ss, false) * inv_n + eps);
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < MAXP; ++j) {
            const int p = threadIdx.x + j * blockDim.x;
            if (p < ppr) {
                const uint4 wv = weight[p];
                const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fw = __bfloat1622float2(wh[e]);
                    x[j][2 * e] = x[j][2 * e] * fw.x * rinv;
                    x[j][2 * e + 1] = x[j][2 * e + 1] * fw.y * rinv;
                    amax = fmaxf(amax, fmaxf(fabsf(x[j][2 * e]), fabsf(x[j][2 * e + 1])));
                }
                if (!QUANT) reinterpret_cast<uint4*>(out)[row * ppr + p] = pack8(x[j]);
            }
        }
        if (QUANT) {
            amax = block_sum(amax, true);
            const float scale = amax == 0.f ? 1.f : amax / 448.0f;
#pragma unroll
            for (int j = 0; j < MAXP; ++j) {
                const int p = threadIdx.x + j * blockDim.x;
                if (p < ppr) {
                    uint32_t q[2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        __nv_fp8x4_e4m3 f4(make_float4(x[j][4 * h] / scale, x[j][4 * h + 1] / scale,
                                                       x[j][4 * h + 2] / scale, x[j][4 * h + 3] / scale));
                        q[h] = *reinterpret_cast<uint32_t*>(&f4);
                    }
                    reinterpret_cast<uint2*>(out)[row * ppr + p] = make_uint2(q[0], q[1]);
                }
            }
            if (threadIdx.x == 0) scale_out[row] = scale;
        }
    }
    if (end_barrier) block_barrier(P, rank, W, 2, epoch);
}

struct Ctx {
    int rank = 0, world = 0, device = -1;
    size_t max_bytes = 0;
    uint8_t* base = nullptr;               // own region
    std::vector<void*> opened;             // peer regions opened via IPC
    Peers peers{};
    uint32_t epoch = 0;                    // eager calls made (captured calls do not count)
    bool ready = false;
};

std::mutex g_mu;

Ctx* as_ctx(int64_t h) {
    Ctx* c = reinterpret_cast<Ctx*>(h);
    AB_CHECK(c != nullptr, "null allreduce context");
    return c;
}

constexpr int kCapturedBuffer = 2;

// Staging buffer and end barrier of a call about to be launched on `st`.  An eager
// call takes the next eager call number and alternates buffers 0 and 1 with no end
// barrier; a call captured into a CUDA graph takes buffer 2, ends with a barrier (a
// replay may run between any two eager calls, or right after another replay) and
// leaves the eager count alone.
struct Slot {
    int buffer;
    int end_barrier;
};

Slot take_slot(Ctx* c, cudaStream_t st) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    AB_CUDA(cudaStreamIsCapturing(st, &cap));
    if (cap != cudaStreamCaptureStatusNone) return {kCapturedBuffer, 1};
    c->epoch += 1;
    return {(int)(c->epoch & 1), 0};
}

bool is_capturing(cudaStream_t st) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    AB_CUDA(cudaStreamIsCapturing(st, &cap));
    return cap != cudaStreamCaptureStatusNone;
}

// Buffer the next call will take, without taking it.
int next_buffer_index(const Ctx* c, bool capturing) {
    return capturing ? kCapturedBuffer : (int)((c->epoch + 1) & 1);
}

uint8_t* staging_ptr(const Ctx* c, int buffer) { return c->base + kSignalPad + (size_t)buffer * c->max_bytes; }

}  // namespace

AB_ENTRY(custom_ar_init,
         (int64_t rank, int64_t world, int64_t max_bytes, int64_t device, int64_t* ctx_out, void* handle_out),
         (rank, world, max_bytes, device, ctx_out, handle_out)) {
    using namespace ab;
    AB_CHECK(world >= 2 && world <= kMaxRanks, "world size must be in [2, ", kMaxRanks, "]");
    AB_CHECK(rank >= 0 && rank < world, "bad rank");
    AB_CHECK(max_bytes > 0 && max_bytes % 16 == 0, "max_bytes must be a positive multiple of 16");
    AB_CHECK(ctx_out && handle_out, "null output pointers");
    DeviceGuard dg((int)device);
    Ctx* c = new Ctx();
    c->rank = (int)rank;
    c->world = (int)world;
    c->device = (int)device;
    c->max_bytes = (size_t)max_bytes;
    const size_t total = kSignalPad + 3 * (size_t)max_bytes;
    cudaError_t e = cudaMalloc(&c->base, total);
    if (e != cudaSuccess) {
        delete c;
        fail("cudaMalloc of the IPC region failed: ", cudaGetErrorString(e));
    }
    e = cudaMemset(c->base, 0, kSignalPad);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
    if (e != cudaSuccess) {
        cudaFree(c->base);
        delete c;
        fail("IPC setup failed: ", cudaGetErrorString(e));
    }
    memcpy(handle_out, &h, sizeof(h));
    *ctx_out = reinterpret_cast<int64_t>(c);
}

AB_ENTRY(custom_ar_open_peers, (int64_t ctx, const void* handles), (ctx, handles)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(!c->ready, "peers already opened");
    DeviceGuard dg(c->device);
    const cudaIpcMemHandle_t* hs = reinterpret_cast<const cudaIpcMemHandle_t*>(handles);
    for (int p = 0; p < c->world; ++p) {
        uint8_t* b = nullptr;
        if (p == c->rank) {
            b = c->base;
        } else {
            void* q = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&q, hs[p], cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                for (void* o : c->opened) cudaIpcCloseMemHandle(o);
                c->opened.clear();
                fail("cudaIpcOpenMemHandle for rank ", p, " failed: ", cudaGetErrorString(e));
            }
            c->opened.push_back(q);
            b = static_cast<uint8_t*>(q);
        }
        c->peers.sig[p] = reinterpret_cast<Signal*>(b);
        for (int k = 0; k < 3; ++k) c->peers.buf[k][p] = b + kSignalPad + (size_t)k * c->max_bytes;
    }
    c->ready = true;
}

AB_ENTRY(custom_ar_open_loopback, (int64_t ctx), (ctx)) {
    Ctx* c = as_ctx(ctx);
    AB_CHECK(!c->ready, "peers already opened");
    for (int p = 0; p < c->world; ++p) {
        c->peers.sig[p] = reinterpret_cast<Signal*>(c->base);
        for (int k = 0; k < 3; ++k) c->peers.buf[k][p] = staging_ptr(c, k);
    }
    c->ready = true;
}

// Pointer of the staging buffer the next eager call will use (zero-copy producers
// write their result there and pass it as `inp`).
AB_ENTRY(custom_ar_next_buffer, (int64_t ctx, int64_t* ptr_out, int64_t* bytes_out), (ctx, ptr_out, bytes_out)) {
    Ctx* c = as_ctx(ctx);
    *ptr_out = reinterpret_cast<int64_t>(staging_ptr(c, next_buffer_index(c, false)));
    *bytes_out = (int64_t)c->max_bytes;
}

// The same for the next call made eagerly (capturing = 0) or inside a CUDA graph
// capture (capturing != 0): captured calls have a staging buffer of their own.
AB_ENTRY(custom_ar_next_buffer_ex, (int64_t ctx, int64_t capturing, int64_t* ptr_out, int64_t* bytes_out),
         (ctx, capturing, ptr_out, bytes_out)) {
    Ctx* c = as_ctx(ctx);
    *ptr_out = reinterpret_cast<int64_t>(staging_ptr(c, next_buffer_index(c, capturing != 0)));
    *bytes_out = (int64_t)c->max_bytes;
}

AB_ENTRY(custom_ar_all_reduce,
         (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t force_two_shot, void* stream),
         (ctx, inp, out, force_two_shot, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(inp, "inp");
    need(out, "out");
    AB_CHECK(inp->dtype_ == AITER_DTYPE_bf16 || inp->dtype_ == AITER_DTYPE_fp16 || inp->dtype_ == AITER_DTYPE_fp32,
             "allreduce supports bf16, fp16 and fp32, got ", dtype_name(inp->dtype_));
    need_dtype(out, inp->dtype_, "out");
    need_contig(inp, "inp");
    need_contig(out, "out");
    AB_CHECK(inp->numel_ == out->numel_, "inp and out sizes differ");
    const size_t bytes = inp->numel_ * elem_size(inp->dtype_);
    AB_CHECK(bytes % 16 == 0, "allreduce size must be a multiple of 16 bytes");
    AB_CHECK(bytes <= c->max_bytes, "allreduce of ", bytes, " bytes exceeds the registered ", c->max_bytes);
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device, "tensor on a different device than the communicator");
    if (bytes == 0) return;
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    const Slot slot = take_slot(c, st);
    const int buffer = slot.buffer;
    const int endb = slot.end_barrier;
    const int64_t n16 = (int64_t)(bytes / 16);
    // force_two_shot: 1 = two-shot, 0 = one-shot, negative = by size.  One-shot reads
    // (W-1) x the data over NVLink, two-shot 2 (W-1)/W x plus one more barrier: with
    // two ranks one-shot always wins, with more it wins while latency dominates.
    const int64_t one_shot_max = c->world == 2 ? INT64_MAX : (c->world <= 4 ? (2 << 20) : (1 << 20));
    const bool two = force_two_shot > 0 ? true : (force_two_shot == 0 ? false : (int64_t)bytes > one_shot_max);
    // about two packs per thread per CTA: small messages still spread over CTAs
    const int64_t per_block = (int64_t)kThreads * 2;
    int grid = (int)std::min<int64_t>((n16 + per_block - 1) / per_block, std::min(kMaxBlocks, num_sms(c->device)));
    grid = std::max(grid, 1);
    const uint4* src = (const uint4*)inp->ptr;
    uint4* dst = (uint4*)out->ptr;
    const int tw = two ? 1 : 0;
#define AB_AR(TT)                                                                                               \
    switch (c->world) {                                                                                         \
        case 2: allreduce_kernel<TT, 2><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        case 3: allreduce_kernel<TT, 3><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        case 4: allreduce_kernel<TT, 4><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        case 5: allreduce_kernel<TT, 5><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        case 6: allreduce_kernel<TT, 6><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        case 7: allreduce_kernel<TT, 7><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
        default: allreduce_kernel<TT, 8><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n16, tw, endb); break; \
    }
    if (inp->dtype_ == AITER_DTYPE_bf16) {
        AB_AR(__nv_bfloat16)
    } else if (inp->dtype_ == AITER_DTYPE_fp16) {
        AB_AR(__half)
    } else {
        AB_AR(float)
    }
#undef AB_AR
    check_launch("custom_ar_all_reduce");
}

// allreduce with open_fp8_quant (the reference's all_reduce(..., open_fp8_quant=True),
// csrc/kernels/custom_all_reduce.cu:76-115): fp16 messages of at least 128 * 2048
// elements take the fp8-quantised two-shot kernel; every other message, and one whose
// codes and scales do not fit the staging buffer after the input, the plain
// allreduce (bf16 ignores the flag in the reference too).
AB_ENTRY(custom_ar_all_reduce_fp8, (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, void* stream),
         (ctx, inp, out, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(inp, "inp");
    need(out, "out");
    const int64_t numel = (int64_t)inp->numel_;
    const int64_t n8 = numel / 8;
    int gp = 1;  // packs per quant group: the largest of 16, 8, 4, 2 dividing numel / W / 8
    for (int g : {16, 8, 4, 2})
        if ((numel / c->world) % (8 * g) == 0) {
            gp = g;
            break;
        }
    const int64_t largest = n8 / c->world + n8 % c->world;
    const int64_t q_off = (numel * 2 + 255) / 256 * 256;
    const int64_t s_off = q_off + (largest * 8 + 255) / 256 * 256;
    const int64_t need_bytes = s_off + (largest / gp + 1) * 2;
    const bool quant = inp->dtype_ == AITER_DTYPE_fp16 && numel >= 128 * 2048 && numel % 8 == 0 &&
                       need_bytes <= (int64_t)c->max_bytes;
    if (!quant) {
        custom_ar_all_reduce_impl(ctx, inp, out, -1, stream);
        return;
    }
    need_dtype(out, AITER_DTYPE_fp16, "out");
    need_contig(inp, "inp");
    need_contig(out, "out");
    AB_CHECK(inp->numel_ == out->numel_, "inp and out sizes differ");
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device, "tensor on a different device than the communicator");
    DeviceGuard dg(c->device);
    const int64_t per_block = (int64_t)kThreads * 2;
    int grid = (int)std::min<int64_t>((n8 + per_block - 1) / per_block, std::min(kMaxBlocks, num_sms(c->device)));
    grid = std::max(grid, 1);
    cudaStream_t st = as_stream(stream);
    const Slot slot = take_slot(c, st);
    const int buffer = slot.buffer;
    const int endb = slot.end_barrier;
    const uint4* src = (const uint4*)inp->ptr;
    uint4* dst = (uint4*)out->ptr;
    switch (c->world) {
        case 2: allreduce_fp8q_kernel<2><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        case 3: allreduce_fp8q_kernel<3><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        case 4: allreduce_fp8q_kernel<4><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        case 5: allreduce_fp8q_kernel<5><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        case 6: allreduce_fp8q_kernel<6><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        case 7: allreduce_fp8q_kernel<7><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
        default: allreduce_fp8q_kernel<8><<<grid, kThreads, 0, st>>>(c->peers, c->rank, buffer, src, dst, n8, gp, q_off, s_off, endb); break;
    }
    check_launch("custom_ar_all_reduce_fp8");
}

// All-gather over peer memory (the reference's custom all-gather,
// aiter/dist/parallel_state.py:492-501, csrc/include/custom_all_reduce.cuh:678-740):
// inp [..] of any dtype (a multiple of 16 bytes), out = the W inputs in rank order
// along dim 0 (last_dim == 0: out [W * inp.shape[0], ...]) or along the last dim
// (last_dim != 0: out [..., W * inp.shape[-1]], rows a multiple of 16 bytes).
AB_ENTRY(custom_ar_all_gather, (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t last_dim, void* stream),
         (ctx, inp, out, last_dim, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(inp, "inp");
    need(out, "out");
    AB_CHECK(inp->dtype_ == out->dtype_, "inp and out dtypes differ");
    need_contig(inp, "inp");
    need_contig(out, "out");
    const size_t esz = elem_size(inp->dtype_);
    const size_t bytes = inp->numel_ * esz;
    AB_CHECK(out->numel_ == inp->numel_ * (size_t)c->world, "out must hold world x inp elements");
    AB_CHECK(bytes % 16 == 0, "all-gather size must be a multiple of 16 bytes");
    AB_CHECK(bytes <= c->max_bytes, "all-gather of ", bytes, " bytes exceeds the registered ", c->max_bytes);
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device && out->device_id == c->device,
             "tensor on a different device than the communicator");
    int64_t c16 = 0;
    if (last_dim) {
        AB_CHECK(inp->ndim >= 1, "inp needs a last dim");
        const int64_t rowb = inp->shape[inp->ndim - 1] * (int64_t)esz;
        AB_CHECK(rowb % 16 == 0, "rows must be a multiple of 16 bytes for a last-dim all-gather");
        c16 = rowb / 16;
    }
    if (bytes == 0) return;
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    const Slot slot = take_slot(c, st);
    const int64_t n16 = (int64_t)(bytes / 16);
    const int64_t per_block = (int64_t)kThreads * 2;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((n16 + per_block - 1) / per_block, std::min(kMaxBlocks, num_sms(c->device))));
    const uint4* src = (const uint4*)inp->ptr;
    uint4* dst = (uint4*)out->ptr;
    switch (c->world) {
        case 2: allgather_kernel<2><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        case 3: allgather_kernel<3><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        case 4: allgather_kernel<4><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        case 5: allgather_kernel<5><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        case 6: allgather_kernel<6><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        case 7: allgather_kernel<7><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
        default: allgather_kernel<8><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, c16, slot.end_barrier); break;
    }
    check_launch("custom_ar_all_gather");
}

// Reduce-scatter over peer memory (the reference's custom reduce-scatter,
// aiter/dist/parallel_state.py:511-538, csrc/include/custom_all_reduce.cuh:740-800):
// inp [n] (bf16, fp16 or fp32; n a multiple of world, every rank's share a multiple
// of 16 bytes), out [n / world] = elements [rank * n / world, (rank + 1) * n / world)
// of the sum over ranks, accumulated in fp32 in rank order (identical to the same
// elements of custom_ar_all_reduce's result).
AB_ENTRY(custom_ar_reduce_scatter, (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, void* stream),
         (ctx, inp, out, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(inp, "inp");
    need(out, "out");
    AB_CHECK(inp->dtype_ == AITER_DTYPE_bf16 || inp->dtype_ == AITER_DTYPE_fp16 || inp->dtype_ == AITER_DTYPE_fp32,
             "reduce-scatter supports bf16, fp16 and fp32, got ", dtype_name(inp->dtype_));
    need_dtype(out, inp->dtype_, "out");
    need_contig(inp, "inp");
    need_contig(out, "out");
    const size_t esz = elem_size(inp->dtype_);
    const size_t bytes = inp->numel_ * esz;
    AB_CHECK(inp->numel_ % (size_t)c->world == 0 && out->numel_ == inp->numel_ / (size_t)c->world,
             "out must hold inp.numel / world elements");
    AB_CHECK((bytes / (size_t)c->world) % 16 == 0, "every rank's share must be a multiple of 16 bytes");
    AB_CHECK(bytes <= c->max_bytes, "reduce-scatter of ", bytes, " bytes exceeds the registered ", c->max_bytes);
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device && out->device_id == c->device,
             "tensor on a different device than the communicator");
    if (bytes == 0) return;
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    const Slot slot = take_slot(c, st);
    const int64_t n16 = (int64_t)(bytes / 16);
    const int64_t per_block = (int64_t)kThreads * 2;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((n16 / c->world + per_block - 1) / per_block, std::min(kMaxBlocks, num_sms(c->device))));
    const uint4* src = (const uint4*)inp->ptr;
    uint4* dst = (uint4*)out->ptr;
#define AB_RS(TT)                                                                                                  \
    switch (c->world) {                                                                                            \
        case 2: reduce_scatter_kernel<TT, 2><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        case 3: reduce_scatter_kernel<TT, 3><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        case 4: reduce_scatter_kernel<TT, 4><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        case 5: reduce_scatter_kernel<TT, 5><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        case 6: reduce_scatter_kernel<TT, 6><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        case 7: reduce_scatter_kernel<TT, 7><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
        default: reduce_scatter_kernel<TT, 8><<<grid, kThreads, 0, st>>>(c->peers, c->rank, slot.buffer, src, dst, n16, slot.end_barrier); break; \
    }
    if (inp->dtype_ == AITER_DTYPE_bf16) {
        AB_RS(__nv_bfloat16)
    } else if (inp->dtype_ == AITER_DTYPE_fp16) {
        AB_RS(__half)
    } else {
        AB_RS(float)
    }
#undef AB_RS
    check_launch("custom_ar_reduce_scatter");
}

AB_ENTRY(custom_ar_dispose, (int64_t ctx), (ctx)) {
    Ctx* c = as_ctx(ctx);
    {
        ab::DeviceGuard dg(c->device);
        cudaDeviceSynchronize();
        for (void* o : c->opened) cudaIpcCloseMemHandle(o);
        if (c->base) cudaFree(c->base);
    }
    delete c;
}

// Error word of the allreduce context: peer waits of every IPC kernel, folded with
// the mbarrier waits of the fused GEMM + allreduce kernels (this unit's copy).
extern "C" int custom_ar_device_error(int clear) {
    int v = 0, m = 0;
    if (cudaMemcpyFromSymbol(&v, g_ar_error, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMemcpyFromSymbol(&m, sm100::g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        int z = 0;
        cudaMemcpyToSymbol(g_ar_error, &z, sizeof(int));
        cudaMemcpyToSymbol(sm100::g_device_error, &z, sizeof(int));
    }
    return v ? v : m;
}

// GEMM + allreduce: y = allreduce_over_ranks(A @ W^T).  The bf16 GEMM writes its
// tile results straight into the staging buffer the allreduce reads next
// (no copy), then the allreduce runs on the same stream.  The reference has no fused
// entry; this equals tensor_model_parallel_all_reduce(tgemm.mm(A, W))
// (aiter/dist/communication_op.py:30-37, aiter/tuned_gemm.py:506-529).
AB_ENTRY(custom_ar_gemm_all_reduce,
         (int64_t ctx, aiter_tensor_t* a, aiter_tensor_t* w, aiter_tensor_t* out, int64_t force_two_shot,
          void* stream),
         (ctx, a, w, out, force_two_shot, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(a, "A");
    need(w, "W");
    need(out, "out");
    need_ndim(a, 2, "A");
    need_ndim(w, 2, "W");
    const int64_t M = a->shape[0], N = w->shape[0];
    AB_CHECK(out->ndim == 2 && out->shape[0] == M && out->shape[1] == N, "out must be [M, N]");
    AB_CHECK((size_t)(M * N * 2) <= c->max_bytes, "GEMM output of ", M * N * 2, " bytes exceeds the registered ",
             c->max_bytes);
    aiter_tensor_t stage{};
    stage.ptr = staging_ptr(c, next_buffer_index(c, is_capturing(as_stream(stream))));
    stage.numel_ = (size_t)(M * N);
    stage.ndim = 2;
    stage.shape[0] = M;
    stage.shape[1] = N;
    stage.strides[0] = N;
    stage.strides[1] = 1;
    stage.dtype_ = AITER_DTYPE_bf16;
    stage.device_id = c->device;
    if (gemm_a16w16(a, w, &stage, stream) != 0) fail(std::string(aiter_get_last_error() ? aiter_get_last_error() : "gemm failed"));
    custom_ar_all_reduce_impl(ctx, &stage, out, force_two_shot, stream);
}

// allreduce(inp) + res_inp -> res_out, RMSNorm(res_out) * w -> out (bf16), or with
// `out` fp8 and `scale_out` [rows] f32: the per-row fp8 quant of the normalised row.
namespace {
void run_allreduce_rmsnorm(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* res_inp, aiter_tensor_t* res_out,
                           aiter_tensor_t* out, aiter_tensor_t* weight, float eps, aiter_tensor_t* scale_out,
                           int64_t force_two_shot, void* stream) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    for (aiter_tensor_t* t : {inp, res_inp, res_out, out, weight}) need(t, "tensor");
    for (aiter_tensor_t* t : {inp, res_inp, res_out, weight}) need_dtype(t, AITER_DTYPE_bf16, "bf16 operand");
    for (aiter_tensor_t* t : {inp, res_inp, res_out, out, weight}) need_contig(t, "operand");
    const bool quant = scale_out != nullptr;
    need_dtype(out, quant ? AITER_DTYPE_fp8 : AITER_DTYPE_bf16, "out");
    AB_CHECK(inp->ndim >= 1, "inp must have a hidden dimension");
    const int64_t hidden = inp->shape[inp->ndim - 1];
    const int64_t rows = hidden > 0 ? (int64_t)inp->numel_ / hidden : 0;
    AB_CHECK(hidden % 8 == 0 && hidden <= 4 * 8 * kThreads, "hidden size must be a multiple of 8 and at most ",
             4 * 8 * kThreads);
    AB_CHECK((int64_t)weight->numel_ == hidden, "weight must have `hidden` elements");
    for (aiter_tensor_t* t : {res_inp, res_out, out})
        AB_CHECK(t->numel_ == inp->numel_, "inp, res_inp, res_out and out must have the same number of elements");
    if (quant) {
        need_dtype(scale_out, AITER_DTYPE_fp32, "scale_out");
        need_contig(scale_out, "scale_out");
        AB_CHECK((int64_t)scale_out->numel_ == rows, "scale_out must hold one scale per row");
    }
    const size_t bytes = inp->numel_ * 2;
    AB_CHECK(bytes <= c->max_bytes, "allreduce of ", bytes, " bytes exceeds the registered ", c->max_bytes);
    for (aiter_tensor_t* t : {inp, res_inp, res_out, out, weight})
        AB_CHECK(((uintptr_t)t->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device, "tensor on a different device than the communicator");
    if (rows == 0) return;
    DeviceGuard dg(c->device);
    const int ppr = (int)(hidden / 8);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(rows, std::min(kMaxBlocks, num_sms(c->device))));
    cudaStream_t st = as_stream(stream);
    const Slot slot = take_slot(c, st);
    const int buffer = slot.buffer;
    const int endb = slot.end_barrier;
    const uint4* src = (const uint4*)inp->ptr;
    // one-shot reads (W-1) x the rows over NVLink, two-shot 2 (W-1)/W x plus a barrier:
    // the size cut-over of the plain allreduce
    const int64_t one_shot_max = c->world == 2 ? INT64_MAX : (c->world <= 4 ? (2 << 20) : (1 << 20));
    const int tw = force_two_shot > 0 ? 1 : (force_two_shot == 0 ? 0 : ((int64_t)bytes > one_shot_max ? 1 : 0));
#define AB_ARRMS(WW)                                                                                              \
    do {                                                                                                          \
        if (quant)                                                                                                \
            allreduce_rmsnorm_kernel<WW, true><<<grid, kThreads, 0, st>>>(                                        \
                c->peers, c->rank, buffer, src, (const uint4*)res_inp->ptr, (uint4*)res_out->ptr, out->ptr,       \
                (float*)scale_out->ptr, (const uint4*)weight->ptr, rows, ppr, eps, endb, tw);                     \
        else                                                                                                      \
            allreduce_rmsnorm_kernel<WW, false><<<grid, kThreads, 0, st>>>(                                       \
                c->peers, c->rank, buffer, src, (const uint4*)res_inp->ptr, (uint4*)res_out->ptr, out->ptr,       \
                nullptr, (const uint4*)weight->ptr, rows, ppr, eps, endb, tw);                                    \
    } while (0)
    switch (c->world) {
        case 2: AB_ARRMS(2); break;
        case 3: AB_ARRMS(3); break;
        case 4: AB_ARRMS(4); break;
        case 5: AB_ARRMS(5); break;
        case 6: AB_ARRMS(6); break;
        case 7: AB_ARRMS(7); break;
        default: AB_ARRMS(8); break;
    }
#undef AB_ARRMS
    check_launch("custom_ar_allreduce_rmsnorm");
}
}  // namespace

AB_ENTRY(custom_ar_allreduce_rmsnorm,
         (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* res_inp, aiter_tensor_t* res_out, aiter_tensor_t* out,
          aiter_tensor_t* weight, float eps, aiter_tensor_t* scale_out, void* stream),
         (ctx, inp, res_inp, res_out, out, weight, eps, scale_out, stream)) {
    run_allreduce_rmsnorm(ctx, inp, res_inp, res_out, out, weight, eps, scale_out, 0, stream);
}

// The same with the one-/two-shot choice: force_two_shot 1 = two-shot (rows reduced
// by an owner rank, every rank takes them from it and normalises locally), 0 =
// one-shot, negative = by size as custom_ar_all_reduce.  Both give the same bits.
AB_ENTRY(custom_ar_allreduce_rmsnorm_ex,
         (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* res_inp, aiter_tensor_t* res_out, aiter_tensor_t* out,
          aiter_tensor_t* weight, float eps, aiter_tensor_t* scale_out, int64_t force_two_shot, void* stream),
         (ctx, inp, res_inp, res_out, out, weight, eps, scale_out, force_two_shot, stream)) {
    run_allreduce_rmsnorm(ctx, inp, res_inp, res_out, out, weight, eps, scale_out, force_two_shot, stream);
}

// GEMM + allreduce in one kernel: y = allreduce_over_ranks(A @ W^T) with the GEMM
// pushing its output over NVLink into the peers' staging buffers while its MMAs run
// (gemm_bf16.cuh): one-shot (every rank gets every rank's rows, then sums them) for
// small messages, two-shot (owner rank sums each piece, every rank pulls it) above
// the same size cut-over as custom_ar_all_reduce.  Same result bits as
// custom_ar_gemm_all_reduce.  Falls back to that two-kernel path when the pushed
// images do not fit one staging buffer or the grid exceeds the per-CTA flags.
AB_ENTRY(custom_ar_gemm_all_reduce_fused,
         (int64_t ctx, aiter_tensor_t* a, aiter_tensor_t* w, aiter_tensor_t* out, int64_t force_two_shot,
          void* stream),
         (ctx, a, w, out, force_two_shot, stream)) {
    using namespace ab;
    Ctx* c = as_ctx(ctx);
    AB_CHECK(c->ready, "custom_ar_open_peers has not been called");
    need(a, "A");
    need(w, "W");
    need(out, "out");
    need_dtype(a, AITER_DTYPE_bf16, "A");
    need_dtype(w, AITER_DTYPE_bf16, "W");
    need_dtype(out, AITER_DTYPE_bf16, "out");
    need_ndim(a, 2, "A");
    need_ndim(w, 2, "W");
    need_contig(a, "A");
    need_contig(w, "W");
    const int64_t M = a->shape[0], K = a->shape[1], N = w->shape[0];
    AB_CHECK(w->shape[1] == K, "W must be [N, K] with the K of A");
    AB_CHECK(out->ndim == 2 && out->shape[0] == M && out->shape[1] == N && out->strides[1] == 1,
             "out must be [M, N] with contiguous rows");
    AB_CHECK(K % g16::BK == 0 && N % 32 == 0, "need K % 64 == 0 and N % 32 == 0");
    AB_CHECK(out->strides[0] % 8 == 0 && ((uintptr_t)out->ptr & 15) == 0, "out rows must be 16-byte aligned");
    AB_CHECK(a->device_id == c->device && w->device_id == c->device && out->device_id == c->device,
             "tensor on a different device than the communicator");
    const int64_t n_bytes = M * N * 2;
    AB_CHECK(n_bytes <= (int64_t)c->max_bytes, "GEMM output of ", n_bytes, " bytes exceeds the registered ",
             c->max_bytes);
    if (M == 0) return;
    const int sms = num_sms(c->device);
    int mode = g16::kTwoShot;
    int64_t slot = 0;
    bool eligible = false;
    if (M <= g16::kSwabMaxM && N % 128 == 0) {
        const int grid = g16::swab_grid((int)M, (int)N, (int)(K / g16::BK), sms);
        const int64_t one_shot_max = c->world == 2 ? INT64_MAX : (c->world <= 4 ? (2 << 20) : (1 << 20));
        const bool two = force_two_shot > 0 ? true : (force_two_shot == 0 ? false : n_bytes > one_shot_max);
        mode = two ? g16::kTwoShot : g16::kOneShot;
        slot = n_bytes;  // every slot is an [M, N] image
        eligible = grid <= kFlagBlocks && (int64_t)c->world * slot <= (int64_t)c->max_bytes;
    } else {
        int tiles = 0;
        slot = g16::twoshot_slot_bytes((int)M, (int)N, c->world, sms, &tiles);
        eligible = force_two_shot != 0 && std::min(tiles, sms) <= kFlagBlocks &&
                   (int64_t)c->world * slot <= (int64_t)c->max_bytes;
    }
    if (!eligible) {
        custom_ar_gemm_all_reduce_impl(ctx, a, w, out, force_two_shot, stream);
        return;
    }
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    const Slot sl = take_slot(c, st);
    g16::FuseArgs F{c->peers, c->rank, c->world, sl.buffer, sl.end_barrier, slot};
    if (mode == g16::kOneShot)
        g16::run<g16::kOneShot>(a, w, (__nv_bfloat16*)out->ptr, out->strides[0], F, c->device, st);
    else
        g16::run<g16::kTwoShot>(a, w, (__nv_bfloat16*)out->ptr, out->strides[0], F, c->device, st);
    check_launch("custom_ar_gemm_all_reduce_fused");
}
