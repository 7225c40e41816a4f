// CUDA-IPC peer-memory layout and primitives (NVLink 5 / NVSwitch), shared by the
// allreduce kernels and the GEMM kernels that push their output tiles to peers.
//
// Every rank owns one cudaMalloc'd region, exported with cudaIpcGetMemHandle and
// opened by every peer:
//   [ Signal (flags written by peers, own call counters) | staging 0 | 1 | 2 ]
// Eager calls alternate between staging 0 and 1 (a rank cannot reach call k+2, which
// rewrites call k's buffer, before every peer has entered call k+1, i.e. finished
// reading call k).  Calls captured into a CUDA graph use staging 2 only and end with
// a barrier, so a replay, whenever it runs, never shares a buffer with the eager
// call before or after it, nor a replay with the next one.
// Flags are epochs: CTA b of a call takes the next value of its own counter[b]
// (only CTA b of this rank touches it and launches are stream-ordered), so every
// rank, making the same calls with the same grids, counts the same epochs per CTA
// index, in eager calls and graph replays alike.  Flags are compared with a
// wrap-safe >= because a fast peer may already have stored a later epoch.
#pragma once
#include "common.cuh"

namespace ipc {

constexpr int kMaxRanks = 8;
constexpr int kFlagBlocks = 256;  // CTA indices that own flags and a call counter
constexpr size_t kSignalPad = 64 * 1024;

struct Signal {
    uint32_t flag[3][kFlagBlocks][kMaxRanks];  // barriers [start | mid | end], slot = writer rank
    uint32_t counter[kFlagBlocks];            // own calls per CTA index (never read by peers)
    uint32_t push[kFlagBlocks][kMaxRanks];    // GEMM+AR: tiles of peer CTA b that reached this rank
    uint32_t ready[kFlagBlocks];              // GEMM+AR: tiles this rank's CTA b has reduced (peers read)
};
static_assert(sizeof(Signal) <= kSignalPad, "signal block exceeds its pad");

struct Peers {
    Signal* sig[kMaxRanks];      // every rank's signal block
    uint8_t* buf[3][kMaxRanks];  // every rank's staging buffers [eager 0 | eager 1 | captured]
};

// Error word of the peer waits (read with custom_ar_device_error()): 1 = a peer did
// not arrive within the wait limit.  One copy per translation unit including this
// header; the allreduce unit, which launches every IPC kernel, exports the reader.
static __device__ int g_ar_error;

constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_cg(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_cg8(const void* p) {
    uint2 v;
    asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// Bounded wait until the epoch word at `p` reaches `target` (wrap-safe).  Returns
// false and sets the error word when it did not within the limit.
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t target) {
    if ((int32_t)(ld_acquire_sys(p) - target) >= 0) return true;
    const uint64_t t0 = abd::globaltimer_ns();
    uint32_t n = 0;
    while ((int32_t)(ld_acquire_sys(p) - target) < 0) {
        if ((++n & 255) == 0 && abd::globaltimer_ns() - t0 > kWaitNs) {
            atomicExch(&g_ar_error, 1);
            return false;
        }
    }
    return true;
}

// Takes this CTA's epoch for the current call (thread 0 only).
__device__ __forceinline__ uint32_t next_epoch(const Peers& P, int rank) {
    uint32_t* ctr = &P.sig[rank]->counter[blockIdx.x];
    const uint32_t e = *ctr + 1;
    *ctr = e;
    return e;
}

// Cross-rank barrier of CTA index blockIdx.x: every thread of the CTA calls it.
// CTA b of rank r stores the epoch into flag[phase][b][r] of every peer and waits
// until its own flag[phase][b][p] has reached it for all p.  Returns false (and sets
// the error word) when a peer did not arrive in time.
__device__ __forceinline__ bool block_barrier(const Peers& P, int rank, int world, int phase, uint32_t epoch) {
    __syncthreads();
    bool ok = true;
    if (threadIdx.x < world) {
        // publish: everything this CTA wrote before is visible to peers first
        __threadfence_system();
        st_release_sys(&P.sig[threadIdx.x]->flag[phase][blockIdx.x][rank], epoch);
        ok = wait_epoch(&P.sig[rank]->flag[phase][blockIdx.x][threadIdx.x], epoch);
    }
    return __syncthreads_and(ok ? 1 : 0) != 0;
}

__device__ __forceinline__ void acc8(float (&a)[8], uint4 v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        a[2 * i] += f.x;
        a[2 * i + 1] += f.y;
    }
}

__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    return v;
}

__device__ __forceinline__ void acc4(float (&a)[4], uint2 v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        a[2 * i] += f.x;
        a[2 * i + 1] += f.y;
    }
}

__device__ __forceinline__ uint2 pack4(const float (&a)[4]) {
    uint2 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 2; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    return v;
}

// Packed progress value of a GEMM+AR call: the CTA's epoch in the high 16 bits and
// the number of tiles done (1-based index of the CTA's j-th tile) in the low 16.
// Consecutive calls differ by at least 1 << 16, so a wrap-safe compare orders them.
__device__ __forceinline__ uint32_t progress(uint32_t epoch, int j) { return (epoch << 16) | (uint32_t)(j + 1); }

}  // namespace ipc
