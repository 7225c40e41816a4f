// bf16 GEMM y = A @ W^T on tcgen05 (kind::f16, fp32 accumulate in TMEM): the GEMM
// half of the tensor-parallel GEMM + allreduce (tgemm.mm / gemm_a16w16,
// aiter/tuned_gemm.py:224-308,506-529; weights [N, K], the F.linear convention).
//
// Persistent kernel, one CTA per SM, 384 threads:
//   warp 0     TMA producer: A box 128 x 64 (128 B rows), W box 128 x 64 twice,
//              128-byte swizzle, 4-stage ring of 48 KB;
//   warp 1     TMEM allocator + single-thread MMA issuer (M=128, N=256, K=16 x 4
//              per 64-wide K block), accumulating the whole K of a tile in one
//              TMEM slab; two slabs alternate between tiles so the epilogue of
//              tile t overlaps the MMAs of tile t+1;
//   warps 4-11 epilogue: TMEM -> registers -> bf16 -> global (rows >= M skipped).
// The output may be the staging buffer of the IPC allreduce (custom_ar_next_buffer),
// which then reduces it without an extra copy.
#include "sm100.cuh"

namespace {

constexpr int BM = 128, BK = 64;
constexpr int A_TILE = BM * BK * 2;
constexpr int NUM_THREADS = 384;
constexpr int kSwabMaxM = 512;  // up to this many rows: the swap-AB split-K kernel

// Tile width BN (32 .. 256): small M uses narrow tiles so that more SMs stream the
// weights; large M uses 256-wide tiles for operand reuse.
template <int BN>
struct GCfg {
    static constexpr int B_TILE = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_TILE + B_TILE;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
    static constexpr int CPT = BN / 2;            // columns per epilogue thread
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    // kind::f16 instruction descriptor: D f32, A/B bf16, both K-major
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
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

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args args) {
    using namespace sm100;
    using C = GCfg<BN>;
    constexpr int STAGES = C::STAGES, STAGE_BYTES = C::STAGE_BYTES, CPT = C::CPT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
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
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[as], (t >> 1) & 1, abort_flag))) break;
            tc_fence_after();
            const int grow = m_blk * BM + row;
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
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

template <int BN>
void launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, Args args, int dev, cudaStream_t st) {
    args.n_tiles = args.N / BN;
    const int tiles = args.m_tiles * args.n_tiles;
    const int grid = std::min(tiles, ab::num_sms(dev));
    ab::set_max_smem_once((const void*)gemm_bf16_kernel<BN>, GCfg<BN>::SMEM_BYTES, dev);
    gemm_bf16_kernel<BN><<<grid, NUM_THREADS, GCfg<BN>::SMEM_BYTES, st>>>(tmA, tmB, args);
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
// stores them as bf16.  One tile per CTA (not persistent).
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

template <int MT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_bf16_swab_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const SArgs args) {
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
        fence_mbar_init();
        prefetch_tensormap(&tmW);
        prefetch_tensormap(&tmX);
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

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
    const int rows_per = MT / S, rbase = rank * rows_per;
    const int rows_live = max(0, min(rows_per, args.M - m_blk * MT - rbase));
    const int groups = rows_live * 32;
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
                *reinterpret_cast<uint2*>(args.out + (int64_t)gm * args.ldo + n_blk * 128 + 4 * (g % 32)) = pk;
            }
        }
    }
    cluster_sync();  // peers are done reading this CTA's partial
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Split of K over a cluster so that tiles x split covers the SMs once.
int pick_split(int tiles, int num_kb, int sms) {
    int s = sms / std::max(tiles, 1);
    s = std::min(s, 8);
    s = std::min(s, num_kb);
    return std::max(s, 1);
}

template <int MT>
void launch_swab(const CUtensorMap& tmW, const CUtensorMap& tmX, SArgs args, int dev, cudaStream_t st) {
    const int tiles = args.n_tiles * ((args.M + MT - 1) / MT);
    args.split = pick_split(tiles, args.num_kb, ab::num_sms(dev));
    ab::set_max_smem_once((const void*)gemm_bf16_swab_kernel<MT>, SCfg<MT>::SMEM_BYTES, dev);
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
    AB_CUDA(cudaLaunchKernelEx(&cfg, gemm_bf16_swab_kernel<MT>, tmW, tmX, args));
}

void make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    // bf16 [rows, cols] as a byte matrix of 2*cols bytes per row; box 64 elements x box_rows
    ab::make_tmap_2d_u8(map, base, rows, cols * 2, 128, box_rows, true);
}

// Tile width by problem size: enough tiles to cover the SMs when M is small.
int pick_bn(int M, int N, int sms) {
    const int m_tiles = (M + BM - 1) / BM;
    for (int bn : {256, 128, 64, 32})
        if (N % bn == 0 && m_tiles * (N / bn) >= sms) return bn;
    return N % 32 == 0 ? 32 : 256;
}

}  // namespace

AB_ENTRY(gemm_a16w16,
         (aiter_tensor_t * a, aiter_tensor_t* w, aiter_tensor_t* out, void* stream), (a, w, out, stream)) {
    using namespace ab;
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
    AB_CHECK(out->ndim == 2 && out->strides[1] == 1, "out rows must be contiguous");
    const int M = (int)a->shape[0], K = (int)a->shape[1], N = (int)w->shape[0];
    AB_CHECK(w->shape[1] == K, "W must be [N, K] with the K of A");
    AB_CHECK(out->shape[0] == M && out->shape[1] == N, "out must be [M, N]");
    AB_CHECK(K % BK == 0 && N % 32 == 0, "need K % 64 == 0 and N % 32 == 0");
    AB_CHECK(out->strides[0] % 8 == 0 && ((uintptr_t)out->ptr & 15) == 0, "out rows must be 16-byte aligned");
    if (M == 0) return;
    DeviceGuard dg(a->device_id);
    const int dev = a->device_id;
    cudaStream_t st = as_stream(stream);
    if (M <= kSwabMaxM && N % 128 == 0) {
        const int mt = M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
        CUtensorMap tmW, tmX;
        make_tmap_bf16(&tmW, w->ptr, N, K, 128);
        make_tmap_bf16(&tmX, a->ptr, M, K, mt);
        SArgs sa{(__nv_bfloat16*)out->ptr, out->strides[0], M, N, K / BK, N / 128, 1};
        switch (mt) {
            case 32: launch_swab<32>(tmW, tmX, sa, dev, st); break;
            case 64: launch_swab<64>(tmW, tmX, sa, dev, st); break;
            case 128: launch_swab<128>(tmW, tmX, sa, dev, st); break;
            default: launch_swab<256>(tmW, tmX, sa, dev, st); break;
        }
        check_launch("gemm_a16w16");
        return;
    }
    const int bn = pick_bn(M, N, num_sms(dev));
    CUtensorMap tmA, tmB;
    make_tmap_bf16(&tmA, a->ptr, M, K, 128);
    make_tmap_bf16(&tmB, w->ptr, N, K, bn < 128 ? bn : 128);
    Args args{(__nv_bfloat16*)out->ptr, out->strides[0], M, N, K / BK, (M + BM - 1) / BM, 0};
    switch (bn) {
        case 256: launch_gemm<256>(tmA, tmB, args, dev, st); break;
        case 128: launch_gemm<128>(tmA, tmB, args, dev, st); break;
        case 64: launch_gemm<64>(tmA, tmB, args, dev, st); break;
        default: launch_gemm<32>(tmA, tmB, args, dev, st); break;
    }
    check_launch("gemm_a16w16");
}
