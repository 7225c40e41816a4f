// bf16 GEMM y = A @ W^T on tcgen05 (kind::f16, fp32 accumulate in TMEM): the GEMM
// half of the tensor-parallel GEMM + allreduce (tgemm.mm / gemm_a16w16,
// aiter/tuned_gemm.py:224-308,506-529; weights [N, K], the F.linear convention).
//
// Two kernels, each templated on a fusion mode:
//   kPlain    the product goes to `out` (gemm_a16w16), or to the staging buffer
//             of the IPC allreduce, which then reduces it without a copy;
//   kOneShot  (small M) every CTA pushes its output rows to every rank's staging
//             buffer over NVLink, a per-CTA cross-rank barrier, then each rank
//             sums the W copies of those rows in rank order into `out`;
//   kTwoShot  every output piece is pushed only to its owner rank; the owner sums
//             the W copies in rank order in place and publishes it, every rank
//             then pulls it into `out`.
// In the fused modes the transfer of a tile overlaps the MMAs of the next ones and
// the allreduce needs no launch of its own.  Sums accumulate bf16 partials in fp32
// in rank order, exactly as allreduce_bf16_kernel does, so a fused call returns the
// same bits as the GEMM followed by the allreduce, on every rank.
//
// This header holds the kernel templates; gemm_bf16.cu instantiates the plain ones,
// allreduce.cu the fused ones (which report through the allreduce error word).
#pragma once
#include "ipc.cuh"
#include "sm100.cuh"

namespace {
namespace g16 {

constexpr int BM = 128, BK = 64;
constexpr int A_TILE = BM * BK * 2;
constexpr int NUM_THREADS = 384;
constexpr int kSwabMaxM = 512;  // up to this many rows: the swap-AB split-K kernel

enum Fuse : int { kPlain = 0, kOneShot = 1, kTwoShot = 2 };

// Peer context of a fused call.  Staging buffer `buffer` of rank p holds one slot
// of `slot_bytes` per source rank: slot s = what rank s pushed to p.
struct FuseArgs {
    ipc::Peers P;
    int rank, world, buffer, end_barrier;
    int64_t slot_bytes;
};

// Tile width BN (32 .. 256): small M uses narrow tiles so that more SMs stream the
// weights; large M uses 256-wide tiles for operand reuse.
template <int BN>
struct GCfg {
    static constexpr int B_TILE = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_TILE + B_TILE;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
    static constexpr int BAR_BYTES = 256;
    static constexpr int CPT = BN / 2;            // columns per epilogue thread
    static constexpr int CC = CPT < 64 ? CPT : 64;  // columns per push chunk (fused)
    static constexpr int PUSH_BYTES = 8 * 32 * CC * 2;  // per epilogue warp: 32 rows x CC bf16
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
    static constexpr int SMEM_BYTES_FUSED = SMEM_BYTES + PUSH_BYTES;
    static constexpr int TILE_BYTES = BM * BN * 2;  // one bf16 output tile in a staging slot
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    // kind::f16 instruction descriptor: D f32, A/B bf16, both K-major
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
    static_assert(SMEM_BYTES_FUSED <= 227 * 1024, "shared memory");
    static_assert(CPT % CC == 0 && CC % 16 == 0, "push chunks");
};

struct Args {
    __nv_bfloat16* out;
    int64_t ldo;
    int M, N, num_kb, m_tiles, n_tiles;
};

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Barrier of the 8 epilogue warps: lane 0 of each warp arrives after the warp's
// writes, then every lane waits (bounded) for the phase.
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) sm100::mbar_arrive(bar);
    return __all_sync(0xffffffffu, sm100::mbar_wait(bar, parity, abort_flag));
}

// Lane 0 waits (bounded) for a peer's progress word, the warp shares the outcome.
__device__ __forceinline__ bool warp_wait_epoch(const uint32_t* p, uint32_t target) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = ipc::wait_epoch(p, target) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// Persistent kernel, one CTA per SM, 384 threads:
//   warp 0     TMA producer: A box 128 x 64 (128 B rows), W box 128 x 64 twice,
//              128-byte swizzle, 4-stage ring of 48 KB;
//   warp 1     TMEM allocator + single-thread MMA issuer (M=128, N=BN, K=16 x 4
//              per 64-wide K block), accumulating the whole K of a tile in one
//              TMEM slab; two slabs alternate between tiles so the epilogue of
//              tile t overlaps the MMAs of tile t+1;
//   warps 4-11 epilogue: TMEM -> registers -> bf16 -> global (rows >= M skipped).
// kTwoShot: tile t (the j-th of this CTA; every rank runs the same schedule) is
// owned by rank t % W and lands in the owner's slot [this rank], at packed index
// t / W.  The epilogue stages each warp's 32 x CC piece in shared memory and
// stores whole row segments to the owner; after the tile, warp 4 raises
// push[b][rank] on the owner to progress(epoch, j).  After its last tile the CTA
// reduces the tiles it owns (waiting for every rank's push of them) in place into
// its own slot and raises ready[b] per tile; then it pulls every tile of its list
// from the owner into `out`.
template <int BN, int FUSE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args args,
                 const FuseArgs F) {
    using namespace sm100;
    using C = GCfg<BN>;
    static_assert(FUSE == kPlain || FUSE == kTwoShot, "the persistent kernel fuses the two-shot allreduce");
    constexpr int STAGES = C::STAGES, STAGE_BYTES = C::STAGE_BYTES, CPT = C::CPT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint64_t* ebar = reinterpret_cast<uint64_t*>(tmem_slot + 2);  // fused: epilogue-warp barrier
    uint32_t* s_epoch = reinterpret_cast<uint32_t*>(ebar + 1);
    uint8_t* push_smem = smem + STAGES * STAGE_BYTES + C::BAR_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&tfull[s], 1);
            mbar_init(&tempty[s], 8);
        }
        *abort_flag = 0;
        if (FUSE != kPlain) {
            mbar_init(ebar, 8);
            *s_epoch = ipc::next_epoch(F.P, F.rank);
        }
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_tiles = args.m_tiles * args.n_tiles;
    const uint32_t epoch = FUSE != kPlain ? *s_epoch : 0u;
    bool fused_ok = true;  // epilogue: every wait of the fused phases succeeded

    if (warp < 4) {
        setmaxnreg_dec<40>();
        if (warp == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                // n fastest: concurrently running CTAs share the A rows in L2
                const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
                for (int kb = 0; kb < args.num_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag));
                    if (!ok) break;
                    if (lane == 0) {
                        mbar_expect_tx(&full[s], STAGE_BYTES);
                        uint8_t* a = smem + s * STAGE_BYTES;
                        uint8_t* b = a + A_TILE;
                        // the tensor maps address bytes: a 64-element bf16 K block is 128 bytes
                        const int kx = kb * BK * 2;
                        tma_load_2d(a, &tmA, &full[s], kx, m_blk * BM);
#pragma unroll
                        for (int j = 0; j < (BN + 127) / 128; ++j)
                            tma_load_2d(b + j * 128 * BK * 2, &tmB, &full[s], kx, n_blk * BN + j * 128);
                    }
                    __syncwarp();
                }
            }
            if (!ok) {
                for (int d = 0; d < STAGES && it - 1 - d >= 0; ++d) {
                    const int j = it - 1 - d;
                    mbar_wait(&full[j % STAGES], (j / STAGES) & 1, abort_flag, 200000000ull, false);
                }
            }
        } else if (warp == 1) {
            if (lane == 0) {
                int it = 0, t = 0;
                bool ok = true;
                for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
                    const int as = t & 1;
                    if (!mbar_wait(&tempty[as], ((t >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d = tmem_base + as * BN;
                    for (int kb = 0; kb < args.num_kb; ++kb, ++it) {
                        const int s = it % STAGES;
                        if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint8_t* a = smem + s * STAGE_BYTES;
                        const uint64_t adesc = smem_desc_sw128(a);
                        const uint64_t bdesc = smem_desc_sw128(a + A_TILE);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            mma_bf16(d, adesc + 2 * kk, bdesc + 2 * kk, C::IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&tfull[as]);
                }
                if (t > 0) {
                    const int j = t - 1;
                    mbar_wait(&tfull[j & 1], (j >> 1) & 1, abort_flag, 200000000ull, false);
                }
            }
            __syncwarp();
        }
    } else {
        setmaxnreg_inc<232>();
        const int q = warp & 3, h = (warp - 4) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        int t = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
            const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
            const int as = t & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[as], (t >> 1) & 1, abort_flag))) {
                fused_ok = false;
                break;
            }
            tc_fence_after();
            const int grow = m_blk * BM + row;
            if constexpr (FUSE == kPlain) {
                __nv_bfloat16* dst = args.out + (int64_t)grow * args.ldo + n_blk * BN + CPT * h;
#pragma unroll
                for (int ch = 0; ch < CPT / 16; ++ch) {
                    float v[16];
                    tmem_ld16(lane_base + as * BN + CPT * h + 16 * ch, v);
                    tmem_wait_ld();
                    if (ch == CPT / 16 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[as]);
                    }
                    if (grow < args.M) {
                        uint32_t w[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                            w[i] = *reinterpret_cast<uint32_t*>(&b2);
                        }
                        uint4* d4 = reinterpret_cast<uint4*>(dst + 16 * ch);
                        d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                }
            } else {
                // push this warp's 32 x CPT piece of the tile to the owner, CC columns
                // at a time: registers -> shared (16-byte chunks XOR-swizzled by row)
                // -> whole row segments of 2*CC bytes to the owner's slot
                constexpr int CC = C::CC, LPR = CC * 2 / 16, RPI = 32 / LPR;
                const int owner = tile % F.world;
                uint8_t* dst_tile = F.P.buf[F.buffer][owner] + (int64_t)F.rank * F.slot_bytes +
                                    (int64_t)(tile / F.world) * C::TILE_BYTES;
                uint8_t* stg = push_smem + (warp - 4) * (32 * CC * 2);
#pragma unroll
                for (int ch = 0; ch < CPT / CC; ++ch) {
#pragma unroll
                    for (int p = 0; p < CC / 16; ++p) {
                        float v[16];
                        tmem_ld16(lane_base + as * BN + CPT * h + CC * ch + 16 * p, v);
                        tmem_wait_ld();
                        if (ch == CPT / CC - 1 && p == CC / 16 - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&tempty[as]);
                        }
#pragma unroll
                        for (int c2 = 0; c2 < 2; ++c2) {
                            const int c = 2 * p + c2;
                            float a8[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) a8[i] = v[8 * c2 + i];
                            *reinterpret_cast<uint4*>(stg + lane * (CC * 2) + ((c ^ (lane % LPR)) * 16)) =
                                ipc::pack8(a8);
                        }
                    }
                    __syncwarp();
#pragma unroll
                    for (int it2 = 0; it2 < LPR; ++it2) {
                        const int r = it2 * RPI + lane / LPR, c = lane % LPR;
                        if (m_blk * BM + q * 32 + r < args.M) {
                            const uint4 val = *reinterpret_cast<const uint4*>(stg + r * (CC * 2) + ((c ^ (r % LPR)) * 16));
                            *reinterpret_cast<uint4*>(dst_tile + (int64_t)(q * 32 + r) * (BN * 2) +
                                                      (CPT * h + CC * ch + 8 * c) * 2) = val;
                        }
                    }
                    __syncwarp();
                }
                // the whole tile is on its way: warp 4 publishes it to the owner
                if (!epi_sync(ebar, t & 1, abort_flag)) {
                    fused_ok = false;
                    break;
                }
                if (warp == 4 && lane == 0) {
                    __threadfence_system();
                    ipc::st_release_sys(&F.P.sig[owner]->push[blockIdx.x][F.rank], ipc::progress(epoch, t));
                }
            }
        }
        if constexpr (FUSE == kTwoShot) {
            const int et = threadIdx.x - 128;  // 0..255
            constexpr int PPR = BN / 8;          // 16-byte packs per tile row
            constexpr int PACKS = BM * PPR;
            int tcount = t;
            // reduce the tiles this rank owns, in list order
            int nsync = tcount;  // epi_sync phases used so far
            for (int j = 0, tile = blockIdx.x; fused_ok && tile < num_tiles; tile += gridDim.x, ++j) {
                if (tile % F.world != F.rank) continue;
                const int m_blk = tile / args.n_tiles;
                for (int src = 0; src < F.world && fused_ok; ++src)
                    fused_ok = warp_wait_epoch(&F.P.sig[F.rank]->push[blockIdx.x][src], ipc::progress(epoch, j));
                if (!fused_ok) break;
                const int64_t toff = (int64_t)(tile / F.world) * C::TILE_BYTES;
                const uint8_t* mine = F.P.buf[F.buffer][F.rank];
                for (int i = et; i < PACKS; i += 256) {
                    if (m_blk * BM + i / PPR >= args.M) continue;
                    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    for (int src = 0; src < F.world; ++src)
                        ipc::acc8(a, ipc::ld_cg(mine + (int64_t)src * F.slot_bytes + toff + (int64_t)i * 16));
                    *reinterpret_cast<uint4*>(const_cast<uint8_t*>(mine) + (int64_t)F.rank * F.slot_bytes + toff +
                                              (int64_t)i * 16) = ipc::pack8(a);
                }
                if (!epi_sync(ebar, nsync & 1, abort_flag)) {
                    fused_ok = false;
                    break;
                }
                ++nsync;
                if (warp == 4 && lane == 0) {
                    __threadfence_system();
                    ipc::st_release_sys(&F.P.sig[F.rank]->ready[blockIdx.x], ipc::progress(epoch, j));
                }
            }
            // gather every tile of the list from its owner
            for (int j = 0, tile = blockIdx.x; fused_ok && tile < num_tiles; tile += gridDim.x, ++j) {
                const int owner = tile % F.world;
                const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
                fused_ok = warp_wait_epoch(&F.P.sig[owner]->ready[blockIdx.x], ipc::progress(epoch, j));
                if (!fused_ok) break;
                const uint8_t* src = F.P.buf[F.buffer][owner] + (int64_t)owner * F.slot_bytes +
                                     (int64_t)(tile / F.world) * C::TILE_BYTES;
                constexpr int U = 8;
                for (int i0 = et; i0 < PACKS; i0 += U * 256) {
                    uint4 v[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int i = i0 + u * 256;
                        if (i < PACKS && m_blk * BM + i / PPR < args.M) v[u] = ipc::ld_cg(src + (int64_t)i * 16);
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int i = i0 + u * 256;
                        if (i < PACKS && m_blk * BM + i / PPR < args.M)
                            *reinterpret_cast<uint4*>(args.out + (int64_t)(m_blk * BM + i / PPR) * args.ldo +
                                                      n_blk * BN + (i % PPR) * 8) = v[u];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (FUSE != kPlain && F.end_barrier) {
        // captured call: every replay reuses the same staging buffer, so nobody
        // leaves before every peer is done reading this rank's slots
        const bool all_ok = __syncthreads_and(fused_ok ? 1 : 0) != 0;
        if (all_ok) ipc::block_barrier(F.P, F.rank, F.world, 2, epoch);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

template <int BN, int FUSE>
void launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, Args args, const FuseArgs& F, int dev,
                 cudaStream_t st) {
    args.n_tiles = args.N / BN;
    const int tiles = args.m_tiles * args.n_tiles;
    const int grid = std::min(tiles, ab::num_sms(dev));
    constexpr int smem = FUSE == kPlain ? GCfg<BN>::SMEM_BYTES : GCfg<BN>::SMEM_BYTES_FUSED;
    ab::set_max_smem_once((const void*)gemm_bf16_kernel<BN, FUSE>, smem, dev);
    gemm_bf16_kernel<BN, FUSE><<<grid, NUM_THREADS, smem, st>>>(tmA, tmB, args, F);
}

// ---------------------------------------------------------------------------
// Small-M kernel (swap-AB, split-K over a thread-block cluster).
//
// For few activation rows the weights are the stream that matters, so they take
// the 128-row MMA side: D^T[n, m] = W[n, :] . A[m, :] with M=128 weight rows and
// N=MT activation rows (MT in 32..256).  A tile of 128 weight rows is split along K
// over the S CTAs of a cluster (S <= 8) so that tiles x S fills the SMs.  Each CTA
// leaves its fp32 partial in its own shared memory, [MT][128] (activation row
// major), and after a cluster barrier CTA r sums rows [r*MT/S, (r+1)*MT/S) of all S
// partials through distributed shared memory, in rank order (deterministic), and
// stores them as bf16 (S need not divide MT: shares of ceil(MT/S) rows, the last one
// shorter).  One tile per CTA (not persistent).
// Fused: CTA b's rows go, as a [M, N] image in slot [this rank], to every rank
// (kOneShot) or to rank b % W (kTwoShot) instead of `out`; then the per-CTA
// cross-rank barriers of the allreduce (phase 0 after the push, phase 1 after the
// owner's reduce) order the sums.
template <int MT>
struct SCfg {
    static constexpr int W_TILE = 128 * BK * 2;
    static constexpr int X_TILE = MT * BK * 2;
    static constexpr int STAGE_BYTES = W_TILE + X_TILE;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
    static constexpr int P_BYTES = MT * 128 * 4;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
    static constexpr int CPT = MT / 2;  // accumulator columns per epilogue thread
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MT >> 3) << 17) |
                                      ((uint32_t)(128 >> 4) << 24);
    static_assert(P_BYTES <= STAGES * STAGE_BYTES, "partial tile reuses the operand ring");
    static_assert(CPT % 16 == 0, "epilogue reads 16-column groups");
};

struct SArgs {
    __nv_bfloat16* out;
    int64_t ldo;
    int M, N, num_kb, n_tiles, split;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f4(const float* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(sm100::smem_u32(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

template <int MT, int FUSE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_bf16_swab_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const SArgs args, const FuseArgs F) {
    using namespace sm100;
    using C = SCfg<MT>;
    constexpr int STAGES = C::STAGES, STAGE_BYTES = C::STAGE_BYTES, CPT = C::CPT;
    constexpr int TMEM_COLS = MT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tdone = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tdone + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* s_epoch = tmem_slot + 2;
    float* part = reinterpret_cast<float*>(smem);  // [MT][128] fp32, after the K loop

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = args.split;
    const int rank = (int)cluster_ctarank();
    const int tile = blockIdx.x / S;
    const int n_blk = tile % args.n_tiles, m_blk = tile / args.n_tiles;
    const int kb0 = (int)((int64_t)args.num_kb * rank / S), kb1 = (int)((int64_t)args.num_kb * (rank + 1) / S);
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tdone, 1);
        *abort_flag = 0;
        if (FUSE != kPlain) *s_epoch = ipc::next_epoch(F.P, F.rank);
        fence_mbar_init();
        prefetch_tensormap(&tmW);
        prefetch_tensormap(&tmX);
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t epoch = FUSE != kPlain ? *s_epoch : 0u;

    if (warp == 0) {
        int it = 0;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % STAGES;
            ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag));
            if (!ok) break;
            if (lane == 0) {
                mbar_expect_tx(&full[s], STAGE_BYTES);
                uint8_t* w = smem + s * STAGE_BYTES;
                tma_load_2d(w, &tmW, &full[s], kb * BK * 2, n_blk * 128);
                tma_load_2d(w + C::W_TILE, &tmX, &full[s], kb * BK * 2, m_blk * MT);
            }
            __syncwarp();
        }
        if (!ok) {
            for (int d = 0; d < STAGES && it - 1 - d >= 0; ++d) {
                const int j = it - 1 - d;
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1, abort_flag, 200000000ull, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = it % STAGES;
                if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint8_t* w = smem + s * STAGE_BYTES;
                const uint64_t wdesc = smem_desc_sw128(w);
                const uint64_t xdesc = smem_desc_sw128(w + C::W_TILE);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    mma_bf16(tmem_base, wdesc + 2 * kk, xdesc + 2 * kk, C::IDESC, (it > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            mma_commit(tdone);  // fires once every MMA above has finished
            (void)ok;
        }
        __syncwarp();
    } else if (warp >= 4) {
        // TMEM (lane = weight row n, column = activation row m) -> part[m][n]
        const int q = warp & 3, h = (warp - 4) >> 2;
        const int n = q * 32 + lane;
        const bool have = __all_sync(0xffffffffu, mbar_wait(tdone, 0, abort_flag));
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + CPT * h;
#pragma unroll
        for (int c = 0; c < CPT / 16; ++c) {
            float v[16];
            tmem_ld16(taddr + 16 * c, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) part[(CPT * h + 16 * c + j) * 128 + n] = (have && kb1 > kb0) ? v[j] : 0.f;
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // every partial of the cluster is in place
    // rows [r*MT/S, (r+1)*MT/S) of the tile, as 4-column groups; rows past M are
    // skipped.  Each thread first issues the loads of R groups from all S ranks,
    // then sums: the remote reads overlap instead of paying one latency each.
    constexpr int R = 4;
    // ceil: S need not divide MT (S = 3, 5, 6, 7 leave a shorter last share)
    const int rows_per = (MT + S - 1) / S, rbase = rank * rows_per;
    const int rows_live = max(0, min(min(rows_per, MT - rbase), args.M - m_blk * MT - rbase));
    const int groups = rows_live * 32;
    // fused: where this CTA's rows go, and the byte offset of group g's 4 columns
    const int owner = FUSE == kTwoShot ? (int)(blockIdx.x % F.world) : F.rank;
    auto img_off = [&](int g) -> int64_t {
        const int gm = m_blk * MT + rbase + g / 32;
        return ((int64_t)gm * args.N + n_blk * 128 + 4 * (g % 32)) * 2;
    };
    for (int g0 = threadIdx.x; g0 < groups; g0 += R * NUM_THREADS) {
        float4 v[R][8];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int g = g0 + j * NUM_THREADS;
            if (g < groups) {
                const float* src = part + (rbase + g / 32) * 128 + 4 * (g % 32);
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < S) v[j][r] = ld_dsmem_f4(src, (uint32_t)r);
            }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int g = g0 + j * NUM_THREADS;
            if (g < groups) {
                float4 acc = v[j][0];
#pragma unroll
                for (int r = 1; r < 8; ++r)
                    if (r < S) {  // rank order: identical bits for any thread layout
                        acc.x += v[j][r].x;
                        acc.y += v[j][r].y;
                        acc.z += v[j][r].z;
                        acc.w += v[j][r].w;
                    }
                const int gm = m_blk * MT + rbase + g / 32;
                __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
                uint2 pk = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
                if constexpr (FUSE == kPlain) {
                    *reinterpret_cast<uint2*>(args.out + (int64_t)gm * args.ldo + n_blk * 128 + 4 * (g % 32)) = pk;
                } else if constexpr (FUSE == kOneShot) {
                    const int64_t off = (int64_t)F.rank * F.slot_bytes + img_off(g);
                    for (int p = 0; p < F.world; ++p) *reinterpret_cast<uint2*>(F.P.buf[F.buffer][p] + off) = pk;
                } else {
                    *reinterpret_cast<uint2*>(F.P.buf[F.buffer][owner] + (int64_t)F.rank * F.slot_bytes +
                                              img_off(g)) = pk;
                }
            }
        }
    }
    cluster_sync();  // peers are done reading this CTA's partial
    if constexpr (FUSE != kPlain) {
        // phase 0: every rank's CTA b has pushed its rows
        bool ok = ipc::block_barrier(F.P, F.rank, F.world, 0, epoch);
        const uint8_t* mine = F.P.buf[F.buffer][F.rank];
        if (ok && (FUSE == kOneShot || owner == F.rank)) {
            // sum the W images of this CTA's rows in rank order
            for (int g = threadIdx.x; g < groups; g += NUM_THREADS) {
                const int64_t off = img_off(g);
                float a[4] = {0, 0, 0, 0};
                for (int src = 0; src < F.world; ++src) ipc::acc4(a, ipc::ld_cg8(mine + (int64_t)src * F.slot_bytes + off));
                const uint2 pk = ipc::pack4(a);
                if (FUSE == kOneShot) {
                    const int gm = m_blk * MT + rbase + g / 32;
                    *reinterpret_cast<uint2*>(args.out + (int64_t)gm * args.ldo + n_blk * 128 + 4 * (g % 32)) = pk;
                } else {
                    *reinterpret_cast<uint2*>(const_cast<uint8_t*>(mine) + (int64_t)F.rank * F.slot_bytes + off) = pk;
                }
            }
        }
        if (FUSE == kTwoShot) {
            // phase 1: the owner's sum is published; every rank copies it
            ok = ok && ipc::block_barrier(F.P, F.rank, F.world, 1, epoch);
            if (ok) {
                const uint8_t* src = F.P.buf[F.buffer][owner] + (int64_t)owner * F.slot_bytes;
                for (int g = threadIdx.x; g < groups; g += NUM_THREADS) {
                    const int gm = m_blk * MT + rbase + g / 32;
                    *reinterpret_cast<uint2*>(args.out + (int64_t)gm * args.ldo + n_blk * 128 + 4 * (g % 32)) =
                        ipc::ld_cg8(src + img_off(g));
                }
            }
        }
        if (ok && F.end_barrier) ipc::block_barrier(F.P, F.rank, F.world, 2, epoch);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Split of K over a cluster so that tiles x split covers the SMs once.
inline int pick_split(int tiles, int num_kb, int sms) {
    int s = sms / std::max(tiles, 1);
    s = std::min(s, 8);
    s = std::min(s, num_kb);
    return std::max(s, 1);
}

inline int swab_mt(int M) { return M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

// Grid of the swap-AB kernel (CTAs) for this problem.
inline int swab_grid(int M, int N, int num_kb, int sms, int* split_out = nullptr) {
    const int mt = swab_mt(M);
    const int tiles = (N / 128) * ((M + mt - 1) / mt);
    const int s = pick_split(tiles, num_kb, sms);
    if (split_out) *split_out = s;
    return tiles * s;
}

template <int MT, int FUSE>
void launch_swab(const CUtensorMap& tmW, const CUtensorMap& tmX, SArgs args, const FuseArgs& F, int dev,
                 cudaStream_t st) {
    const int tiles = args.n_tiles * ((args.M + MT - 1) / MT);
    args.split = pick_split(tiles, args.num_kb, ab::num_sms(dev));
    ab::set_max_smem_once((const void*)gemm_bf16_swab_kernel<MT, FUSE>, SCfg<MT>::SMEM_BYTES, dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * args.split);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SCfg<MT>::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = args.split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    AB_CUDA(cudaLaunchKernelEx(&cfg, gemm_bf16_swab_kernel<MT, FUSE>, tmW, tmX, args, F));
}

inline void make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    // bf16 [rows, cols] as a byte matrix of 2*cols bytes per row; box 64 elements x box_rows
    ab::make_tmap_2d_u8(map, base, rows, cols * 2, 128, box_rows, true);
}

// Tile width by problem size: enough tiles to cover the SMs when M is small.
inline int pick_bn(int M, int N, int sms) {
    const int m_tiles = (M + BM - 1) / BM;
    for (int bn : {256, 128, 64, 32})
        if (N % bn == 0 && m_tiles * (N / bn) >= sms) return bn;
    return N % 32 == 0 ? 32 : 256;
}

// Bytes of one source slot of the persistent two-shot GEMM + allreduce: the tiles
// one rank owns (every W-th), each a full 128 x BN bf16 tile.
inline int64_t twoshot_slot_bytes(int M, int N, int world, int sms, int* tiles_out = nullptr) {
    const int bn = pick_bn(M, N, sms);
    const int tiles = ((M + BM - 1) / BM) * (N / bn);
    if (tiles_out) *tiles_out = tiles;
    return (int64_t)((tiles + world - 1) / world) * BM * bn * 2;
}

// Launch of either kernel for A [M, K] x W [N, K]^T -> out (plain) or the fused
// allreduce of it.  Shapes are checked by the callers.
template <int FUSE>
void run(const aiter_tensor_t* a, const aiter_tensor_t* w, __nv_bfloat16* out, int64_t ldo, const FuseArgs& F,
         int dev, cudaStream_t st) {
    const int M = (int)a->shape[0], K = (int)a->shape[1], N = (int)w->shape[0];
    if (M <= kSwabMaxM && N % 128 == 0) {
        const int mt = swab_mt(M);
        CUtensorMap tmW, tmX;
        make_tmap_bf16(&tmW, w->ptr, N, K, 128);
        make_tmap_bf16(&tmX, a->ptr, M, K, mt);
        SArgs sa{out, ldo, M, N, K / BK, N / 128, 1};
        switch (mt) {
            case 32: launch_swab<32, FUSE>(tmW, tmX, sa, F, dev, st); break;
            case 64: launch_swab<64, FUSE>(tmW, tmX, sa, F, dev, st); break;
            case 128: launch_swab<128, FUSE>(tmW, tmX, sa, F, dev, st); break;
            default: launch_swab<256, FUSE>(tmW, tmX, sa, F, dev, st); break;
        }
        return;
    }
    if constexpr (FUSE == kOneShot) {
        ab::fail("the one-shot GEMM + allreduce needs M <= ", kSwabMaxM, " and N % 128 == 0");
    } else {
        const int bn = pick_bn(M, N, ab::num_sms(dev));
        CUtensorMap tmA, tmB;
        make_tmap_bf16(&tmA, a->ptr, M, K, 128);
        make_tmap_bf16(&tmB, w->ptr, N, K, bn < 128 ? bn : 128);
        Args args{out, ldo, M, N, K / BK, (M + BM - 1) / BM, 0};
        switch (bn) {
            case 256: launch_gemm<256, FUSE>(tmA, tmB, args, F, dev, st); break;
            case 128: launch_gemm<128, FUSE>(tmA, tmB, args, F, dev, st); break;
            case 64: launch_gemm<64, FUSE>(tmA, tmB, args, F, dev, st); break;
            default: launch_gemm<32, FUSE>(tmA, tmB, args, F, dev, st); break;
        }
    }
}

}  // namespace g16
}  // namespace
