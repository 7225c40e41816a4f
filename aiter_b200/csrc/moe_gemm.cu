// FP8 block-scale grouped GEMMs of the fused MoE, written for sm_100a.
//
// Both stages run one persistent, warp-specialised kernel:
//   warp 0       TMA producer.  A is stored in sorted-row order (written by
//                moe_gather_quant_1x128 for stage 1 and by the stage-1 epilogue for
//                stage 2), so every operand tile is one plain 2-D TMA box: A =
//                128 sorted rows x 128 K, B = 2 x 128 weight rows x 128 K.
//                128-byte swizzle, 4-stage smem ring.
//   warp 1       TMEM allocator and single-thread tcgen05.mma issuer
//                (kind::f8f6f4, M=128, N=256, K=32 x 4 per 128-wide K block).
//   warps 4..11  epilogue.  Every 128-wide K block lands in one of two TMEM
//                accumulator slabs; the epilogue promotes it into fp32 registers
//                with the block scales, acc += slab * a_scale[row, kb] * w_scale[n, kb]
//                (the 1x128 / 128x128 scale contract of torch_moe_stage1/2,
//                aiter/fused_moe.py:1523-1536,1623-1634), while the MMA fills the
//                other slab.
// Stage 1 epilogue: act(gate) * up (gate = columns [0, I), up = [I, 2I) of w1,
// aiter/fused_moe.py:1578-1582), rounded to bf16, then 1x128 fp8 requant
// (amax / 448) -- the separate requant of aiter/fused_moe.py:1306-1314 fused in --
// written to the sorted row it was computed for.
// Scales of the sorted activations are stored transposed, [K/128][rows], so each
// epilogue warp reads its 32 rows' scales of one K block with one coalesced load.
// Stage 2 epilogue: multiply by the row's top-k weight and add into the bf16
// output row of its token with vector red.global.add (the output is zeroed by
// moe_sorting_fwd), i.e. the scatter-reduce over the k slots.
#include <cstdlib>

#include "sm100.cuh"

namespace {

constexpr int BM = 128, BK = 128;
constexpr int A_TILE = BM * BK;
constexpr int NUM_THREADS = 384;
constexpr int TMEM_COLS = 512;
constexpr int SRING = 8;            // block-scale ring depth (K blocks ahead)
constexpr int SRING_FLOATS = 132;   // 128 row scales + 2 column-block scales, padded

// Tile configuration by accumulator width BN.  TMEM (512 fp32 columns x 128 lanes)
// is split into 512/BN accumulator slabs: the MMA writes one slab per 128-wide K
// block while the epilogue promotes the previous ones.  The smem ring takes what
// the operand tiles leave of 192 KB.
//
// W4 (MXFP4 weights, kind::mxf8f6f4.block_scale): the weights' e8m0 scales live in
// TMEM next to the accumulators, so a tile's 256 columns are two N=128 MMAs, each
// into its own 128-column slab of a 3-deep ring (columns 0-383); columns 384-387
// hold the unit A scales and 392.. one 8-column buffer of B scales per smem stage
// (a buffer is rewritten only after the MMAs of its previous K block completed,
// which the stage's "empty" barrier already guarantees).  A smem stage carries the
// A box, the two B boxes (unpacked by the TMA to one byte per e2m1 value) and the
// two 512-byte scale chunks of the B boxes.
template <int BN_, bool W4 = false>
struct Cfg {
    static_assert(!W4 || BN_ == 256, "W4 tiles are 2 x 128 columns");
    static constexpr int SLAB_COLS = W4 ? 128 : BN_;
    static constexpr int SLABS = W4 ? 3 : TMEM_COLS / BN_;
    static constexpr int B_TILE = BN_ * BK;
    static constexpr int SF_BYTES = W4 ? 2 * 512 : 0;
    static constexpr int STAGE_BYTES = A_TILE + B_TILE + SF_BYTES;
    static constexpr int STAGES = (W4 ? 200 * 1024 : 192 * 1024) / STAGE_BYTES;
    // bytes the TMA and bulk copies deliver per stage (packed e2m1: half a byte per value)
    static constexpr uint32_t TX_BYTES = W4 ? A_TILE + B_TILE / 2 + SF_BYTES : STAGE_BYTES;
    static constexpr int CPT = BN_ / 2;  // accumulator columns per epilogue thread
    static constexpr uint32_t IDESC = W4 ? sm100::idesc_e4m3_e2m1_ue8m0(BM, 128) : sm100::idesc_e4m3_f32(BM, BN_);
    static constexpr uint32_t IDESC64 = sm100::idesc_e4m3_f32(64, BN_);  // half tiles
    static constexpr uint32_t SFA_COL = 384, SFB_COL = 392;              // W4 scale columns
    static constexpr int BAR_BYTES = 512;
    static constexpr int RED_BYTES = 2 * 256 * 4;                 // stage-1 row amax exchange
    static constexpr int SRING_BYTES = SRING * SRING_FLOATS * 4;  // block-scale ring
    static constexpr int OUT_BYTES = BM * 128;                    // stage-1 fp8 output tile
    static constexpr int ONES_BYTES = W4 ? 512 : 0;               // W4: chunk of unit A scales
    static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + OUT_BYTES + BAR_BYTES +
                                      RED_BYTES + SRING_BYTES + ONES_BYTES;
    static_assert(CPT % 64 == 0, "epilogue works in 64-column chunks");
    static_assert(2 * (STAGES + SLABS + SRING) * 8 + 2 * 8 + 8 <= BAR_BYTES, "barrier area");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    static_assert(!W4 || (SLABS * SLAB_COLS <= (int)SFA_COL && SFB_COL + 8 * STAGES <= (uint32_t)TMEM_COLS),
                  "TMEM map");
};

struct GemmArgs {
    const int* sorted_ids;
    const int* sorted_eids;
    const int* num_valid;
    const float* a_scale;   // [num_kb][rows_pad], sorted rows
    const float* b_scale;   // [E, N/128, num_kb]
    const uint8_t* b_sf;    // W4: e8m0 scale chunks [E, N/128, num_kb, 512]
    const float* sorted_w;  // stage 2
    void* out;              // stage 1: fp8 [rows_pad, I] sorted; stage 2: bf16 [M, D]
    float* out_scale;       // stage 1: [I/128][rows_pad]
    int M, N, n_tiles, num_kb, max_m_blocks, act, out_cols, E, rows_pad;
    int half_tiles;  // 1: blocks whose rows 64.. are all padding run as M=64 tiles
    int l2hint;      // stage 2: output rows reduced with an L2 evict_last policy
    int doweight;    // stage 1: multiply gate/up by the row's top-k weight (doweight_stage1)
    int inter_f16;   // stage 1: round the intermediate to fp16 (else bf16) before the requant
    int out_f16;     // stage 2: fp16 output (else bf16); sorted_w == nullptr: weight 1
    const float* bias;  // BIAS kernels: f32 [E, bias_ld] (stage 1: 2I gate|up, stage 2: D)
    int bias_ld;
};

// Half tile: sorted row 64 of the block is padding.  Within an expert's segment the
// real rows come first and padding fills the block, so rows 64..127 are then all
// padding and an M=64 MMA covers every real row.  The M=64 accumulator occupies the
// lower 16 lanes of each TMEM subpartition (rows 16q..16q+15 -> lanes 32q..32q+15),
// so the epilogue reads half the TMEM bytes of a full tile.
__device__ __forceinline__ bool half_block(const GemmArgs& a, int m_blk) {
    return a.half_tiles && (a.sorted_ids[m_blk * 128 + 64] & 0xFFFFFF) >= a.M;
}

// Activations in the reference's fp32 order (SiLU x / (1 + e^-x), GELU 0.5 x (1 +
// erf(x / sqrt 2)), Swiglu below) with CUDA's accurate expf / erff and a division
// within 2 ulps (__fdividef): the result is rounded to bf16 right after, and a
// last-bit difference from the reference moves that rounding only within a few fp32
// ulps of a bf16 rounding boundary.  The activation is a template parameter of the
// kernel, so each instance carries the code of one activation only (the unrolled
// tile epilogue is otherwise large enough to thrash the instruction cache).
template <int ACT>
__device__ __forceinline__ float act_fn(float g) {
    if constexpr (ACT == AITER_ACT_GELU) return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
    return __fdividef(g, 1.0f + expf(-g));
}

// Gated activation of a (gate, up) pair: act(gate) * up, or Swiglu
// (aiter/fused_moe.py:1473-1480): min(gate, 7) * sigmoid(1.702 min(gate, 7)) *
// (clamp(up, -7, 7) + 1), the sigmoid as 1 / (1 + e^-(1.702 g)).
template <int ACT>
__device__ __forceinline__ float act_pair(float g, float u) {
    if constexpr (ACT == AITER_ACT_SWIGLU) {
        g = fminf(g, 7.0f);
        u = fminf(fmaxf(u, -7.0f), 7.0f);
        const float sig = __fdividef(1.0f, 1.0f + expf(-1.702f * g));
        return g * sig * (u + 1.0f);
    } else {
        return act_fn<ACT>(g) * u;
    }
}

// fp8 e4m3 codes (RNE, saturating) of the fp32 quotients RN(x_i / s), i.e. of the
// reference's `(x / scale).to(fp8)`, in two steps.  fp8x4_bracket: q = x * RN(1/s) is
// within 2^-23 relative of x / s, so when q * (1 - 2^-20) and q * (1 + 2^-20) give the
// same fp8 codes, the exact quotient (and its fp32 rounding) lies between them and has
// those codes too; otherwise `exact` is raised and the caller recomputes its codes
// with fp8x4_ieee (IEEE division), which only a quotient within 2^-20 of an fp8
// rounding boundary needs.
__device__ __forceinline__ uint32_t fp8x4_bracket(float x0, float x1, float x2, float x3, float rs, bool& exact) {
    const float lo = 1.0f - 0x1p-20f, hi = 1.0f + 0x1p-20f;
    const float q0 = x0 * rs, q1 = x1 * rs, q2 = x2 * rs, q3 = x3 * rs;
    __nv_fp8x4_e4m3 pl(make_float4(q0 * lo, q1 * lo, q2 * lo, q3 * lo));
    __nv_fp8x4_e4m3 ph(make_float4(q0 * hi, q1 * hi, q2 * hi, q3 * hi));
    const uint32_t cl = *reinterpret_cast<uint32_t*>(&pl), ch = *reinterpret_cast<uint32_t*>(&ph);
    exact |= cl != ch;
    return cl;
}

__device__ __forceinline__ uint32_t fp8x4_ieee(float x0, float x1, float x2, float x3, float s) {
    __nv_fp8x4_e4m3 pe(make_float4(__fdiv_rn(x0, s), __fdiv_rn(x1, s), __fdiv_rn(x2, s), __fdiv_rn(x3, s)));
    return *reinterpret_cast<uint32_t*>(&pe);
}

// The stage-1 intermediate is rounded to the activation dtype (bf16 or fp16) before
// its fp8 requant, as the reference casts it (aiter/fused_moe.py:1585).
__device__ __forceinline__ float round_inter(float y, int f16) {
    return f16 ? __half2float(__float2half_rn(y)) : __bfloat162float(__float2bfloat16_rn(y));
}

// Barrier of the 8 epilogue warps: lane 0 of each warp arrives after the warp's
// shared-memory writes, then every lane waits (bounded) for the phase.
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) sm100::mbar_arrive(bar);
    return __all_sync(0xffffffffu, sm100::mbar_wait(bar, parity, abort_flag));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The same with an L2 policy for the output line (evict_last keeps the rows that
// further slots still add into resident while the weights stream through L2).
__device__ __forceinline__ void red_add_bf16x8_hint(__nv_bfloat16* dst, uint32_t a, uint32_t b, uint32_t c,
                                                    uint32_t d, uint64_t policy) {
    asm volatile("red.global.add.L2::cache_hint.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4}, %5;" ::"l"(dst), "r"(a),
                 "r"(b), "r"(c), "r"(d), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void red_add_bf16x8(__nv_bfloat16* dst, uint32_t a, uint32_t b, uint32_t c,
                                               uint32_t d) {
    asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void red_add_f16x8(__half* dst, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// out[off .. off+8) += a[0..8) * w, as bf16 (default) or fp16 vector atomics.
__device__ __forceinline__ void scatter_add8(void* out, int64_t off, const float* a, float w, int f16,
                                             uint64_t policy = 0) {
    if (policy != 0 && !f16) {
        red_add_bf16x8_hint(reinterpret_cast<__nv_bfloat16*>(out) + off, pack_bf16x2(a[0] * w, a[1] * w),
                            pack_bf16x2(a[2] * w, a[3] * w), pack_bf16x2(a[4] * w, a[5] * w),
                            pack_bf16x2(a[6] * w, a[7] * w), policy);
    } else if (f16) {
        red_add_f16x8(reinterpret_cast<__half*>(out) + off, pack_f16x2(a[0] * w, a[1] * w),
                      pack_f16x2(a[2] * w, a[3] * w), pack_f16x2(a[4] * w, a[5] * w), pack_f16x2(a[6] * w, a[7] * w));
    } else {
        red_add_bf16x8(reinterpret_cast<__nv_bfloat16*>(out) + off, pack_bf16x2(a[0] * w, a[1] * w),
                       pack_bf16x2(a[2] * w, a[3] * w), pack_bf16x2(a[4] * w, a[5] * w),
                       pack_bf16x2(a[6] * w, a[7] * w));
    }
}

// STAGE 1: B tile = 128 gate rows + 128 up rows of w1 (BN must be 256), epilogue
//          act(gate)*up -> 1x128 fp8 requant of the 128 outputs, TMA-stored.
// STAGE 2: B tile = BN consecutive rows of w2, epilogue weighted scatter-add.
// BIAS: the expert's f32 bias is added to the GEMM output before the activation
//       (stage 1, after the doweight multiply) or before the top-k weight (stage 2),
//       as torch_moe_stage1/2 add w1_bias / w2_bias (aiter/fused_moe.py:1572-1573,
//       1662-1663); the kernels without it are unchanged.
//
// Warp roles: 0 TMA producer, 1 TMEM owner + MMA issuer, 2 block-scale prefetcher
// (cp.async of a_scale[kb][tile rows] and the two w-scales of the tile's column
// blocks into an SRING-deep smem ring, so the epilogue never waits on a global
// load), 4..11 epilogue.
template <int STAGE, int BN_, bool BIAS, int ACT, bool W4>
__global__ void __launch_bounds__(NUM_THREADS, 1)
moe_gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmO, const GemmArgs args) {
    using namespace sm100;
    using C = Cfg<BN_, W4>;
    static_assert(STAGE == 2 || BN_ == 256, "stage 1 pairs 128 gate with 128 up columns");
    constexpr int STAGES = C::STAGES, SLABS = C::SLABS, CPT = C::CPT, STAGE_BYTES = C::STAGE_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* out_tile = smem + STAGES * STAGE_BYTES;  // 1024-aligned (swizzled TMA store source)
    uint64_t* full = reinterpret_cast<uint64_t*>(out_tile + C::OUT_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + SLABS;
    uint64_t* sfull = tempty + SLABS;
    uint64_t* sempty = sfull + SRING;
    uint64_t* ebar = sempty + SRING;  // [0] row amax exchange, [1] output tile complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(out_tile + C::OUT_BYTES + C::BAR_BYTES);
    float* sring = red + 2 * 256;
    uint8_t* ones = reinterpret_cast<uint8_t*>(sring + SRING * SRING_FLOATS);  // W4 only

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < SLABS; ++s) {
            mbar_init(&tfull[s], 1);
            // W4 stage 2: each 128-column slab is read by one epilogue warpgroup
            mbar_init(&tempty[s], W4 && STAGE == 2 ? 4 : 8);
        }
        for (int s = 0; s < SRING; ++s) {
            mbar_init(&sfull[s], 32);  // one cp.async arrival per prefetcher lane
            mbar_init(&sempty[s], 8);  // one arrival per epilogue warp
        }
        mbar_init(&ebar[0], 8);
        mbar_init(&ebar[1], 8);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (STAGE == 1) prefetch_tensormap(&tmO);
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m_blocks = min(args.num_valid[0] / BM, args.max_m_blocks);
    const int num_tiles = num_m_blocks * args.n_tiles;
    const int nblk128 = args.N / 128;

    if (warp < 4) {
    setmaxnreg_dec<40>();
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
            const int e = min(max(args.sorted_eids[m_blk], 0), args.E - 1);
            for (int kb = 0; kb < args.num_kb; ++kb, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag));
                if (!ok) break;
                if (lane == 0) {
                    mbar_expect_tx(&full[s], C::TX_BYTES);
                    uint8_t* a = smem + s * STAGE_BYTES;
                    uint8_t* b = a + A_TILE;
                    tma_load_2d(a, &tmA, &full[s], kb * BK, m_blk * BM);
                    if (STAGE == 1) {
                        tma_load_2d(b, &tmB, &full[s], kb * BK, e * args.N + n_blk * 128);                    // gate
                        tma_load_2d(b + 128 * BK, &tmB, &full[s], kb * BK, e * args.N + (args.N >> 1) + n_blk * 128);  // up
                    } else {
#pragma unroll
                        for (int j = 0; j < BN_ / 128; ++j)
                            tma_load_2d(b + j * 128 * BK, &tmB, &full[s], kb * BK, e * args.N + n_blk * BN_ + j * 128);
                    }
                    if constexpr (W4) {
                        // the e8m0 scale chunks of the two 128-row B boxes for this K block
                        const int nb0 = STAGE == 1 ? n_blk : 2 * n_blk;
                        const int nb1 = STAGE == 1 ? nblk128 / 2 + n_blk : 2 * n_blk + 1;
                        const uint8_t* sf = args.b_sf + ((int64_t)e * nblk128 * args.num_kb + kb) * 512;
                        bulk_load(b + C::B_TILE, sf + (int64_t)nb0 * args.num_kb * 512, 512, &full[s]);
                        bulk_load(b + C::B_TILE + 512, sf + (int64_t)nb1 * args.num_kb * 512, 512, &full[s]);
                    }
                }
                __syncwarp();
            }
        }
        // drain: wait for the loads of the last STAGES iterations (bounded)
        if (!ok) {
            for (int d = 0; d < STAGES && it - 1 - d >= 0; ++d) {
                const int j = it - 1 - d;
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1, abort_flag, 200000000ull, false);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if constexpr (W4) {
            // unit A scales (e8m0 127 = 2^0) for every row: one 512-byte chunk copied
            // into TMEM once; the A operand's fp32 1x128 scales are promoted in the
            // epilogue as in the FP8 kernel
            reinterpret_cast<uint4*>(ones)[lane] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tmem_cp_32x128b_x4(tmem_base + C::SFA_COL, smem_desc_noswz(ones, 128));
        }
        if (lane == 0 && W4) {
            // two N=128 MMAs per K block (gate / up, or the tile's column halves), each
            // into the next slab of the ring; the B scales of the K block are copied to
            // TMEM first (tcgen05.cp -> tcgen05.mma is ordered in issue order) into the
            // buffer of the smem stage: its last readers, the MMAs of K block it -
            // STAGES, completed before the producer could refill the stage
            int it = 0, j = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < args.num_kb && ok; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint8_t* a = smem + s * STAGE_BYTES;
                    const uint64_t adesc = smem_desc_sw128(a);
                    const uint32_t sfb = tmem_base + C::SFB_COL + 8 * s;
                    tmem_cp_32x128b_x4(sfb, smem_desc_noswz(a + A_TILE + C::B_TILE, 128));
                    tmem_cp_32x128b_x4(sfb + 4, smem_desc_noswz(a + A_TILE + C::B_TILE + 512, 128));
                    for (int c = 0; c < 2; ++c, ++j) {
                        const int as = j % SLABS;
                        if (!mbar_wait(&tempty[as], ((j / SLABS) & 1) ^ 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t bdesc = smem_desc_sw128(a + A_TILE + c * 128 * BK);
                        const uint32_t d = tmem_base + as * C::SLAB_COLS;
#pragma unroll
                        for (int kk = 0; kk < BK / 32; ++kk)
                            mma_mxf8f6f4_bs(d, adesc + 2 * kk, bdesc + 2 * kk, C::IDESC | (kk << 4) | (kk << 29),
                                            (tmem_base + C::SFA_COL) | ((uint32_t)kk << 30),
                                            (sfb + 4 * c) | ((uint32_t)kk << 30), kk > 0 ? 1u : 0u);
                        mma_commit(&tfull[as]);
                    }
                    mma_commit(&empty[s]);
                }
            }
            if (j > 0) {
                const int jl = j - 1;
                mbar_wait(&tfull[jl % SLABS], (jl / SLABS) & 1, abort_flag, 200000000ull, false);
            }
        } else if (lane == 0) {
            int it = 0, acc_it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const uint32_t idesc = half_block(args, tile / args.n_tiles) ? C::IDESC64 : C::IDESC;
                for (int kb = 0; kb < args.num_kb; ++kb, ++it, ++acc_it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    const int as = acc_it % SLABS;
                    const uint32_t aph = (acc_it / SLABS) & 1;
                    if (!mbar_wait(&tempty[as], aph ^ 1, abort_flag)) { ok = false; break; }
                    if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint8_t* a = smem + s * STAGE_BYTES;
                    const uint64_t adesc = smem_desc_sw128(a);
                    const uint64_t bdesc = smem_desc_sw128(a + A_TILE);
                    const uint32_t d = tmem_base + as * BN_;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk)
                        mma_f8f6f4(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
                    mma_commit(&empty[s]);
                    mma_commit(&tfull[as]);
                }
            }
            // make sure no MMA is still writing TMEM before teardown
            if (acc_it > 0) {
                const int j = acc_it - 1;
                mbar_wait(&tfull[j % SLABS], (j / SLABS) & 1, abort_flag, 200000000ull, false);
            }
        }
        __syncwarp();
    } else if (warp == 2) {
        // ------------------------------------------------------------ scale prefetcher
        // ring entry (tile, kb): [0,128) a_scale of the tile's rows, [128] and [129]
        // the w-scales of the two 128-column blocks the epilogue threads cover
        // (stage 1: gate block, up block; stage 2: columns [0,128) and [128,256)).
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
            const int e = min(max(args.sorted_eids[m_blk], 0), args.E - 1);
            const float* sbA = nullptr;
            const float* sbB = nullptr;
            if (W4) {
            } else if (STAGE == 1) {
                sbA = args.b_scale + ((int64_t)e * nblk128 + n_blk) * args.num_kb;
                sbB = args.b_scale + ((int64_t)e * nblk128 + (nblk128 >> 1) + n_blk) * args.num_kb;
            } else {
                sbA = args.b_scale + ((int64_t)e * nblk128 + n_blk * (BN_ / 128)) * args.num_kb;
                sbB = BN_ >= 256 ? sbA + args.num_kb : sbA;
            }
            const float* sa = args.a_scale + m_blk * BM + lane;
            for (int kb = 0; kb < args.num_kb; ++kb, ++it) {
                const int i = it % SRING;
                ok = __all_sync(0xffffffffu, mbar_wait(&sempty[i], ((it / SRING) & 1) ^ 1, abort_flag));
                if (!ok) break;
                float* dst = sring + i * SRING_FLOATS;
                const float* src = sa + (int64_t)kb * args.rows_pad;
#pragma unroll
                for (int j = 0; j < 4; ++j) cp_async4(dst + lane + 32 * j, src + 32 * j);
                if (lane == 0 && !W4) {  // W4: the weight scales are applied by the MMA
                    cp_async4(dst + 128, sbA + kb);
                    cp_async4(dst + 129, sbB + kb);
                }
                cp_async_mbar_arrive(&sfull[i]);
            }
        }
        cp_async_wait_all();
    }
    } else {
        setmaxnreg_inc<232>();
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3, h = (warp - 4) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        int acc_it = 0, tcount = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tcount) {
            const int m_blk = tile / args.n_tiles, n_blk = tile % args.n_tiles;
            // half tile: this thread holds row 16q + lane%16 and the column half lane/16
            // of its warp's columns (16x32bx2 loads); full tile: row 32q + lane
            const bool half = !W4 && half_block(args, m_blk);
            const int hh = lane >> 4;
            const int erow = half ? q * 16 + (lane & 15) : row;
            const int srow = m_blk * BM + erow;
            // needed only after the K loop: issued now, they land meanwhile
            const int sid = args.sorted_ids[srow];
            const float wrow = (STAGE == 2 || args.doweight) && args.sorted_w != nullptr ? args.sorted_w[srow] : 1.f;
            float acc[CPT];
            float v[64];
            for (int kb = 0; kb < args.num_kb; ++kb, ++acc_it) {
                const int si = acc_it % SRING;
                if (!__all_sync(0xffffffffu, mbar_wait(&sfull[si], (acc_it / SRING) & 1, abort_flag))) {
                    ok = false;
                    break;
                }
                const float* se = sring + si * SRING_FLOATS;
                const float sa = se[erow], sbA = se[128], sbB = se[129];
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[si]);
                const float s0 = W4 ? sa : sa * (STAGE == 2 && h * CPT >= 128 ? sbB : sbA);
                const float s1 = W4 ? sa : sa * sbB;
                if constexpr (W4) {
                    // stage 1: gate columns 64h.. of slab 2i, up columns 64h.. of slab
                    // 2i+1; stage 2: columns 0..127 of slab 2i+h
#pragma unroll
                    for (int ch = 0; ch < 2; ++ch) {
                        const int jj = 2 * acc_it + (STAGE == 1 ? ch : h);
                        const int as = jj % SLABS;
                        if (STAGE == 1 || ch == 0) {
                            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[as], (jj / SLABS) & 1, abort_flag))) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        const uint32_t t = lane_base + as * C::SLAB_COLS + (STAGE == 1 ? 64 * h : 64 * ch);
                        tmem_ld32(t, *reinterpret_cast<float(*)[32]>(&v[0]));
                        tmem_ld32(t + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
                        tmem_wait_ld();
                        if (STAGE == 1 || ch == 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&tempty[as]);
                        }
                        if (kb == 0) {
#pragma unroll
                            for (int q2 = 0; q2 < 64; ++q2) acc[64 * ch + q2] = v[q2] * sa;
                        } else {
                            const uint64_t sc2 = splat2(sa);
#pragma unroll
                            for (int q2 = 0; q2 < 64; q2 += 2) fma2(&acc[64 * ch + q2], &v[q2], sc2);
                        }
                    }
                    if (!ok) break;
                    continue;
                }
                const int as = acc_it % SLABS;
                const uint32_t aph = (acc_it / SLABS) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&tfull[as], aph, abort_flag))) { ok = false; break; }
                tc_fence_after();
                const uint32_t t = lane_base + as * BN_;
                if (half) {
                    // stage 1: gate columns 64h.. and up columns 128 + 64h..; stage 2:
                    // columns 128h.. and 128h + 64..; 32 of each per thread half
                    const uint32_t c0 = STAGE == 1 ? 64 * h : 128 * h;
                    const uint32_t c1 = STAGE == 1 ? 128 + 64 * h : 128 * h + 64;
                    tmem_ld16x32bx2_32(t + c0, &v[0]);
                    tmem_ld16x32bx2_32(t + c1, &v[32]);
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[as]);
                    const float sc1 = STAGE == 1 ? s1 : s0;
                    if (kb == 0) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            acc[j] = v[j] * s0;
                            acc[32 + j] = v[32 + j] * sc1;
                        }
                    } else {
                        const uint64_t a2 = splat2(s0), b2 = splat2(sc1);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            fma2(&acc[j], &v[j], a2);
                            fma2(&acc[32 + j], &v[32 + j], b2);
                        }
                    }
                    continue;
                }
                // this thread's CPT columns in 64-column chunks; the slab is released
                // as soon as the last chunk is in registers
#pragma unroll
                for (int ch = 0; ch < CPT / 64; ++ch) {
                    const uint32_t col = STAGE == 1 ? (ch == 0 ? 64 * h : 128 + 64 * h) : CPT * h + 64 * ch;
                    const float sc = (STAGE == 1 && ch == 1) ? s1 : s0;
                    tmem_ld32(t + col, *reinterpret_cast<float(*)[32]>(&v[0]));
                    tmem_ld32(t + col + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
                    tmem_wait_ld();
                    if (ch == CPT / 64 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[as]);
                    }
                    if (kb == 0) {
#pragma unroll
                        for (int j = 0; j < 64; ++j) acc[64 * ch + j] = v[j] * sc;
                    } else {
                        const uint64_t sc2 = splat2(sc);
#pragma unroll
                        for (int j = 0; j < 64; j += 2) fma2(&acc[64 * ch + j], &v[j], sc2);
                    }
                }
            }
            if (!ok) break;
            const int tok = sid & 0xFFFFFF;
            const bool valid = tok < args.M;
            // BIAS: this thread's bias columns (the expert's row of the bias matrix)
            const float* brow = nullptr;
            if constexpr (BIAS)
                brow = args.bias + (int64_t)min(max(args.sorted_eids[m_blk], 0), args.E - 1) * args.bias_ld;
            if (STAGE == 1 && half) {
                // 32 gate / up pairs -> 32 outputs: columns 64h + 32hh .. of the tile
                float amax = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float g = args.doweight ? acc[j] * wrow : acc[j];
                    float u = args.doweight ? acc[32 + j] * wrow : acc[32 + j];
                    if constexpr (BIAS) {
                        const int cg = n_blk * 128 + 64 * h + 32 * hh + j;
                        g += brow[cg];
                        u += brow[args.out_cols + cg];
                    }
                    const float yb = round_inter(act_pair<ACT>(g, u), args.inter_f16);
                    acc[j] = yb;
                    amax = fmaxf(amax, fabsf(yb));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 16));  // the row's other half
                float* rb = red + (tcount & 1) * 256;
                if (hh == 0) rb[h * 128 + erow] = amax;
                if (threadIdx.x == 128) bulk_wait_read0();
                if (!epi_sync(&ebar[0], tcount & 1, abort_flag)) break;
                amax = fmaxf(rb[erow], rb[128 + erow]);
                float scale = amax / 448.0f;
                if (scale == 0.f) scale = 1.0f;
                const float rs = __frcp_rn(scale);
                uint8_t* orow = out_tile + erow * 128;
                uint32_t w[8];
                bool exact = false;
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    w[g] = fp8x4_bracket(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3], rs, exact);
                if (exact) {
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        w[g] = fp8x4_ieee(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3], scale);
                }
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int chunk = (4 * h + 2 * hh + c) ^ (erow & 7);
                    *reinterpret_cast<uint4*>(orow + 16 * chunk) =
                        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                }
                if (h == 0 && hh == 0) args.out_scale[(int64_t)n_blk * args.rows_pad + srow] = scale;
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar[1]);
                if (warp == 4) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&ebar[1], tcount & 1, abort_flag))) break;
                    if (lane == 0) {
                        tma_store_2d(&tmO, out_tile, n_blk * 128, m_blk * BM);
                        bulk_commit();
                    }
                }
            } else if (STAGE == 2 && half) {
                if (valid) {
                    const int64_t base = (int64_t)tok * args.out_cols + n_blk * BN_ + 128 * h + 32 * hh;
                    if constexpr (BIAS) {
#pragma unroll
                        for (int r = 0; r < 2; ++r)
#pragma unroll
                            for (int j = 0; j < 32; ++j) acc[32 * r + j] += brow[n_blk * BN_ + 128 * h + 64 * r + 32 * hh + j];
                    }
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            scatter_add8(args.out, base + 64 * r + 8 * c, &acc[32 * r + 8 * c], wrow, args.out_f16);
                    }
                }
            } else if constexpr (STAGE == 1) {
                float amax = 0.f;
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    float g = args.doweight ? acc[j] * wrow : acc[j];
                    float u = args.doweight ? acc[64 + j] * wrow : acc[64 + j];
                    if constexpr (BIAS) {
                        const int cg = n_blk * 128 + 64 * h + j;
                        g += brow[cg];
                        u += brow[args.out_cols + cg];
                    }
                    const float yb = round_inter(act_pair<ACT>(g, u), args.inter_f16);
                    acc[j] = yb;
                    amax = fmaxf(amax, fabsf(yb));
                }
                float* rb = red + (tcount & 1) * 256;
                rb[h * 128 + row] = amax;
                // the previous tile's TMA store must have finished reading out_tile
                if (threadIdx.x == 128) bulk_wait_read0();
                // barriers among the epilogue warps are mbarriers with bounded waits:
                // a warp that gave up earlier never strands the others here
                if (!epi_sync(&ebar[0], tcount & 1, abort_flag)) break;
                amax = fmaxf(rb[row], rb[128 + row]);
                float scale = amax / 448.0f;
                if (scale == 0.f) scale = 1.0f;
                const float rs = __frcp_rn(scale);
                // row `row` of the 128x128-byte tile, 128-byte swizzle: 16-byte chunk c
                // of the row sits at chunk c ^ (row & 7).  The codes are those of
                // x / scale, as the reference's pertoken_quant divides.
                uint8_t* orow = out_tile + row * 128;
                uint32_t w[16];
                bool exact = false;
#pragma unroll
                for (int g = 0; g < 16; ++g)
                    w[g] = fp8x4_bracket(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3], rs, exact);
                if (exact) {
#pragma unroll
                    for (int g = 0; g < 16; ++g)
                        w[g] = fp8x4_ieee(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3], scale);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int chunk = (4 * h + c) ^ (row & 7);
                    *reinterpret_cast<uint4*>(orow + 16 * chunk) =
                        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                }
                if (h == 0) args.out_scale[(int64_t)n_blk * args.rows_pad + srow] = scale;
                fence_proxy_async_smem();
                // only the storing warp waits for the whole tile; the others move on
                __syncwarp();
                if (lane == 0) mbar_arrive(&ebar[1]);
                if (warp == 4) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&ebar[1], tcount & 1, abort_flag))) break;
                    if (lane == 0) {
                        tma_store_2d(&tmO, out_tile, n_blk * 128, m_blk * BM);
                        bulk_commit();
                    }
                }
            } else {
                if (valid) {
                    const int64_t base = (int64_t)tok * args.out_cols + n_blk * BN_ + CPT * h;
                    if constexpr (BIAS) {
#pragma unroll
                        for (int j = 0; j < CPT; ++j) acc[j] += brow[n_blk * BN_ + CPT * h + j];
                    }
                    const uint64_t pol = args.l2hint ? l2_policy_evict_last() : 0;
#pragma unroll
                    for (int c = 0; c < CPT / 8; ++c)
                        scatter_add8(args.out, base + 8 * c, &acc[8 * c], wrow, args.out_f16, pol);
                }
            }
        }
        if (STAGE == 1 && threadIdx.x == 128) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
    static EncodeFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        AB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) ab::fail("cuTensorMapEncodeTiled not available");
        fn = reinterpret_cast<EncodeFn>(p);
    }
    return fn;
}

}  // namespace

namespace ab {
void make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                     uint32_t box_rows, bool swizzle128) {
    AB_CHECK(((uintptr_t)base & 15) == 0, "TMA base address must be 16-byte aligned");
    AB_CHECK(cols % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
    // Encoded maps depend only on these values: a small per-thread cache saves the
    // driver call for operands seen again (weights, reused activation buffers).
    struct Entry {
        const void* base;
        uint64_t rows, cols;
        uint32_t box_cols, box_rows;
        bool swz, used;
        CUtensorMap map;
    };
    constexpr int kEntries = 32;
    thread_local Entry cache[kEntries] = {};
    thread_local int next = 0;
    for (Entry& e : cache)
        if (e.used && e.base == base && e.rows == rows && e.cols == cols && e.box_cols == box_cols &&
            e.box_rows == box_rows && e.swz == swizzle128) {
            *map = e.map;
            return;
        }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail("cuTensorMapEncodeTiled failed with code ", (int)r);
    Entry& e = cache[next];
    next = (next + 1) % kEntries;
    e = Entry{base, rows, cols, box_cols, box_rows, swizzle128, true, *map};
}

void make_tmap_2d_e2m1(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k, uint32_t box_rows) {
    // 16U4_ALIGN16B: every 16 packed values (8 bytes) land in 16 bytes of shared
    // memory, so a 128-value box row fills one 128-byte swizzle row like an fp8 row.
    AB_CHECK(((uintptr_t)base & 31) == 0, "e2m1 TMA base address must be 32-byte aligned");
    AB_CHECK(k % 128 == 0, "e2m1 K must be a multiple of 128");
    cuuint64_t dims[2] = {k, rows};
    cuuint64_t strides[1] = {k / 2};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), dims, strides,
                              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail("cuTensorMapEncodeTiled (e2m1) failed with code ", (int)r);
}
}  // namespace ab

namespace {

struct Sorted {
    int rows_pad;       // sorted_token_ids length (max_num_tokens_padded)
    int max_m_blocks;
};

Sorted check_sorting(aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids,
                     aiter_tensor_t* num_valid_ids, int64_t block_m) {
    using namespace ab;
    need(sorted_token_ids, "sorted_token_ids");
    need(sorted_expert_ids, "sorted_expert_ids");
    need(num_valid_ids, "num_valid_ids");
    need_dtype(sorted_token_ids, AITER_DTYPE_i32, "sorted_token_ids");
    need_dtype(sorted_expert_ids, AITER_DTYPE_i32, "sorted_expert_ids");
    need_dtype(num_valid_ids, AITER_DTYPE_i32, "num_valid_ids");
    AB_CHECK(block_m == BM, "block_m must be ", BM, " for the tcgen05 grouped GEMM, got ", block_m);
    Sorted c{};
    c.rows_pad = (int)sorted_token_ids->numel_;
    c.max_m_blocks = (int)std::min<int64_t>((int64_t)sorted_token_ids->numel_ / BM, (int64_t)sorted_expert_ids->numel_);
    return c;
}

// Sorted-row operand: [rows_pad, K] fp8 with scales [K/128, rows_pad] f32.
void check_sorted_operand(aiter_tensor_t* a, aiter_tensor_t* sc, int rows_pad, const char* an, const char* sn) {
    using namespace ab;
    need(a, an);
    need(sc, sn);
    need_dtype(a, AITER_DTYPE_fp8, an);
    need_dtype(sc, AITER_DTYPE_fp32, sn);
    need_contig(a, an);
    need_contig(sc, sn);
    need_ndim(a, 2, an);
    AB_CHECK(a->shape[0] == rows_pad, an, " must have one row per sorted slot (", rows_pad, ")");
    AB_CHECK(a->shape[1] % 128 == 0, an, " K must be a multiple of 128");
    AB_CHECK((int64_t)sc->numel_ == (a->shape[1] / 128) * (int64_t)rows_pad, sn, " must be [K/128, rows]");
}

// M=64 tiles for blocks whose rows 64.. are padding (half_block): on by default
// (config 1 on a B200: step 1.152 -> 1.121 ms, stage 1 0.728 -> 0.704 ms);
// AITER_B200_MOE_HALF_TILES=0 runs every block as a full 128-row tile.
int half_tiles_enabled() {
    static const int on = [] {
        const char* e = std::getenv("AITER_B200_MOE_HALF_TILES");
        return e != nullptr && e[0] == '0' ? 0 : 1;
    }();
    return on;
}

template <int STAGE, int BN_, bool BIAS, int ACT, bool W4>
void launch_k(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO, const GemmArgs& a, int grid,
              int dev, cudaStream_t st) {
    constexpr int smem = Cfg<BN_, W4>::SMEM_BYTES;
    ab::set_max_smem_once((const void*)moe_gemm_fp8_kernel<STAGE, BN_, BIAS, ACT, W4>, smem, dev);
    moe_gemm_fp8_kernel<STAGE, BN_, BIAS, ACT, W4><<<grid, NUM_THREADS, smem, st>>>(tmA, tmB, tmO, a);
}

// Stage 1 instantiates one kernel per activation (the stage-2 kernel has none).
template <int STAGE, int BN_, bool BIAS, bool W4>
void launch_act(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO, const GemmArgs& a, int grid,
                int dev, cudaStream_t st) {
    if constexpr (STAGE == 2) {
        launch_k<STAGE, BN_, BIAS, AITER_ACT_SILU, W4>(tmA, tmB, tmO, a, grid, dev, st);
    } else if (a.act == AITER_ACT_GELU) {
        launch_k<STAGE, BN_, BIAS, AITER_ACT_GELU, W4>(tmA, tmB, tmO, a, grid, dev, st);
    } else if (a.act == AITER_ACT_SWIGLU) {
        launch_k<STAGE, BN_, BIAS, AITER_ACT_SWIGLU, W4>(tmA, tmB, tmO, a, grid, dev, st);
    } else {
        launch_k<STAGE, BN_, BIAS, AITER_ACT_SILU, W4>(tmA, tmB, tmO, a, grid, dev, st);
    }
}

template <int STAGE, int BN_, bool W4>
void launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO, GemmArgs a, int dev,
            cudaStream_t st) {
    a.half_tiles = W4 ? 0 : half_tiles_enabled();
    // Stage 2 reduces every output row k times while the weights stream through L2;
    // evict_last on the reductions keeps the rows resident between their slots
    // (config 1, B200: DRAM writes 159 -> 73 MB per launch, 0.335 -> 0.333 ms; also
    // loading the weights evict_first cut the writes to 35 MB but raised the weight
    // re-reads from 0.97 to 1.52 GB and gained no time).
    a.l2hint = STAGE == 2 ? 1 : 0;
    a.n_tiles = STAGE == 1 ? a.n_tiles : a.N / BN_;
    const int tiles = a.max_m_blocks * a.n_tiles;
    if (tiles == 0) return;
    const int grid = std::min(tiles, ab::num_sms(dev));
    if (a.bias)
        launch_act<STAGE, BN_, true, W4>(tmA, tmB, tmO, a, grid, dev, st);
    else
        launch_act<STAGE, BN_, false, W4>(tmA, tmB, tmO, a, grid, dev, st);
    ab::check_launch(W4 ? (STAGE == 1 ? "moe_stage1_a8w4" : "moe_stage2_a8w4")
                        : (STAGE == 1 ? "moe_stage1_fp8_blockscale" : "moe_stage2_fp8_blockscale"));
}

// MXFP4 weights [E, N, K/2] (e2m1 pairs) with their e8m0 scales arranged in chunks
// [E, N/128, K/128, 512] (mxfp4_moe_weight_scale_chunks).
void check_w4(aiter_tensor_t* w, aiter_tensor_t* sf, int E, int N, int K, const char* wn, const char* sn) {
    using namespace ab;
    AB_CHECK(w->dtype_ == AITER_DTYPE_fp4x2 || w->dtype_ == AITER_DTYPE_u8 || w->dtype_ == AITER_DTYPE_i8, wn,
             " must be fp4x2 (MXFP4, or its uint8 view)");
    AB_CHECK(sf->dtype_ == AITER_DTYPE_fp8_e8m0 || sf->dtype_ == AITER_DTYPE_u8, sn,
             " must be e8m0 scale chunks (or their uint8 view)");
    need_contig(w, wn);
    need_contig(sf, sn);
    AB_CHECK(w->ndim == 3 && w->shape[0] == E && w->shape[1] == N && w->shape[2] * 2 == K, wn, " must be [E, ", N,
             ", ", K / 2, "] packed e2m1");
    AB_CHECK((int64_t)sf->numel_ == (int64_t)E * (N / 128) * (K / 128) * 512, sn,
             " must hold the scale chunks [E, N/128, K/128, 512] (mxfp4_moe_weight_scale_chunks)");
    AB_CHECK(((uintptr_t)w->ptr & 31) == 0 && ((uintptr_t)sf->ptr & 15) == 0, wn, " / ", sn, " misaligned");
}

}  // namespace

namespace {
// Stage 1 with its options: sorted_weights given = doweight_stage1 (gate and up
// multiplied by the row's top-k weight before the activation); inter_dtype = the
// dtype the intermediate is rounded to before its fp8 requant (bf16 or fp16).
void run_stage1(aiter_tensor_t* a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1, aiter_tensor_t* w1_scale,
                aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m,
                int64_t activation, aiter_tensor_t* sorted_weights, int64_t inter_dtype, aiter_tensor_t* bias,
                void* stream, bool w4 = false) {
    using namespace ab;
    Sorted c = check_sorting(sorted_token_ids, sorted_expert_ids, num_valid_ids, block_m);
    check_sorted_operand(a1, a1_scale, c.rows_pad, "a1", "a1_scale");
    need(w1, "w1");
    need(w1_scale, "w1_scale");
    need_ndim(w1, 3, "w1");
    AB_CHECK(activation == AITER_ACT_SILU || activation == AITER_ACT_GELU || activation == AITER_ACT_SWIGLU,
             "activation must be Silu, Gelu or Swiglu");
    AB_CHECK(inter_dtype == AITER_DTYPE_bf16 || inter_dtype == AITER_DTYPE_fp16, "inter_dtype must be bf16 or fp16");
    const int D = (int)a1->shape[1];
    const int E = (int)w1->shape[0], N = (int)w1->shape[1];
    AB_CHECK(N % 256 == 0, "2 * inter_dim must be a multiple of 256");
    if (w4) {
        check_w4(w1, w1_scale, E, N, D, "w1", "w1_scale");
    } else {
        need_dtype(w1, AITER_DTYPE_fp8, "w1");
        need_dtype(w1_scale, AITER_DTYPE_fp32, "w1_scale");
        need_contig(w1, "w1");
        need_contig(w1_scale, "w1_scale");
        AB_CHECK(w1->shape[2] == D, "w1 K dim must equal the activation width");
        AB_CHECK((int64_t)w1_scale->numel_ == (int64_t)E * (N / 128) * (D / 128),
                 "w1_scale must be [E, 2I/128, D/128]");
    }
    const int I = N / 2;
    check_sorted_operand(out, out_scale, c.rows_pad, "out", "out_scale");
    AB_CHECK(out->shape[1] == I, "out must be [rows, inter_dim]");
    AB_CHECK(num_tokens >= 0 && num_tokens < (1 << 24), "bad num_tokens");
    if (num_tokens == 0) return;
    GemmArgs a{};
    a.sorted_ids = (const int*)sorted_token_ids->ptr;
    a.sorted_eids = (const int*)sorted_expert_ids->ptr;
    a.num_valid = (const int*)num_valid_ids->ptr;
    a.a_scale = (const float*)a1_scale->ptr;
    if (w4)
        a.b_sf = (const uint8_t*)w1_scale->ptr;
    else
        a.b_scale = (const float*)w1_scale->ptr;
    a.out = out->ptr;
    a.out_scale = (float*)out_scale->ptr;
    a.M = (int)num_tokens;
    a.N = N;
    a.n_tiles = I / 128;
    a.num_kb = D / 128;
    a.max_m_blocks = c.max_m_blocks;
    a.act = (int)activation;
    a.out_cols = I;
    a.E = E;
    a.rows_pad = c.rows_pad;
    if (sorted_weights) {
        need_dtype(sorted_weights, AITER_DTYPE_fp32, "sorted_weights");
        AB_CHECK(!sorted_weights || (int64_t)sorted_weights->numel_ >= c.rows_pad, "sorted_weights too small");
        a.sorted_w = (const float*)sorted_weights->ptr;
        a.doweight = 1;
    }
    a.inter_f16 = inter_dtype == AITER_DTYPE_fp16 ? 1 : 0;
    if (bias) {
        need_dtype(bias, AITER_DTYPE_fp32, "bias");
        need_contig(bias, "bias");
        AB_CHECK((int64_t)bias->numel_ == (int64_t)E * N, "bias must be [E, 2 * inter_dim] f32");
        a.bias = (const float*)bias->ptr;
        a.bias_ld = N;
    }
    DeviceGuard dg(a1->device_id);
    CUtensorMap tmA, tmB, tmO;
    make_tmap_2d_u8(&tmA, a1->ptr, (uint64_t)c.rows_pad, D, 128, 128, true);
    if (w4)
        make_tmap_2d_e2m1(&tmB, w1->ptr, (uint64_t)E * N, D, 128);
    else
        make_tmap_2d_u8(&tmB, w1->ptr, (uint64_t)E * N, D, 128, 128, true);
    // output tiles: 128 sorted rows x 128 fp8 columns
    make_tmap_2d_u8(&tmO, out->ptr, (uint64_t)c.rows_pad, I, 128, 128, true);
    if (w4)
        launch<1, 256, true>(tmA, tmB, tmO, a, a1->device_id, as_stream(stream));
    else
        launch<1, 256, false>(tmA, tmB, tmO, a, a1->device_id, as_stream(stream));
}
}  // namespace

AB_ENTRY(moe_stage1_fp8_blockscale,
         (aiter_tensor_t * a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1, aiter_tensor_t* w1_scale,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m, int64_t activation,
          void* stream),
         (a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale, num_tokens,
          block_m, activation, stream)) {
    run_stage1(a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale,
               num_tokens, block_m, activation, nullptr, AITER_DTYPE_bf16, nullptr, stream);
}

AB_ENTRY(moe_stage1_fp8_blockscale_ex,
         (aiter_tensor_t * a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1, aiter_tensor_t* w1_scale,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m, int64_t activation,
          aiter_tensor_t* sorted_weights, int64_t inter_dtype, void* stream),
         (a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale, num_tokens,
          block_m, activation, sorted_weights, inter_dtype, stream)) {
    run_stage1(a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale,
               num_tokens, block_m, activation, sorted_weights, inter_dtype, nullptr, stream);
}

// The same with the expert bias of the gate/up GEMM (the exp_bias of
// moe_cktile2stages_gemm1, aiter/ops/moe_op.py:344-403): f32 [E, 2 * inter_dim].
AB_ENTRY(moe_stage1_fp8_blockscale_bias,
         (aiter_tensor_t * a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1, aiter_tensor_t* w1_scale,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m, int64_t activation,
          aiter_tensor_t* sorted_weights, int64_t inter_dtype, aiter_tensor_t* bias, void* stream),
         (a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale, num_tokens,
          block_m, activation, sorted_weights, inter_dtype, bias, stream)) {
    run_stage1(a1, a1_scale, w1, w1_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale,
               num_tokens, block_m, activation, sorted_weights, inter_dtype, bias, stream);
}

namespace {
void run_stage2(aiter_tensor_t* a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2, aiter_tensor_t* w2_scale,
                aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m, aiter_tensor_t* bias,
                void* stream, bool w4 = false) {
    using namespace ab;
    Sorted c = check_sorting(sorted_token_ids, sorted_expert_ids, num_valid_ids, block_m);
    check_sorted_operand(a2, a2_scale, c.rows_pad, "a2", "a2_scale");
    need(w2, "w2");
    need(w2_scale, "w2_scale");
    need(out, "out");
    AB_CHECK(out->dtype_ == AITER_DTYPE_bf16 || out->dtype_ == AITER_DTYPE_fp16, "out must be bf16 or fp16");
    if (sorted_weights) need_dtype(sorted_weights, AITER_DTYPE_fp32, "sorted_weights");
    need_contig(out, "out");
    need_ndim(w2, 3, "w2");
    need_ndim(out, 2, "out");
    AB_CHECK(!sorted_weights || (int64_t)sorted_weights->numel_ >= c.rows_pad, "sorted_weights too small");
    const int I = (int)a2->shape[1];
    const int E = (int)w2->shape[0], D = (int)w2->shape[1];
    const int M = (int)out->shape[0];
    AB_CHECK(out->shape[1] == D, "out must be [M, D]");
    AB_CHECK(D % 256 == 0, "model_dim must be a multiple of 256");
    if (w4) {
        check_w4(w2, w2_scale, E, D, I, "w2", "w2_scale");
    } else {
        need_dtype(w2, AITER_DTYPE_fp8, "w2");
        need_dtype(w2_scale, AITER_DTYPE_fp32, "w2_scale");
        for (auto* t : {w2, w2_scale}) need_contig(t, "operand");
        AB_CHECK(w2->shape[2] == I, "w2 must be [E, D, I]");
        AB_CHECK((int64_t)w2_scale->numel_ == (int64_t)E * (D / 128) * (I / 128),
                 "w2_scale must be [E, D/128, I/128]");
    }
    AB_CHECK(((uintptr_t)out->ptr & 15) == 0, "out must be 16-byte aligned");
    if (M == 0) return;
    GemmArgs a{};
    a.sorted_ids = (const int*)sorted_token_ids->ptr;
    a.sorted_eids = (const int*)sorted_expert_ids->ptr;
    a.num_valid = (const int*)num_valid_ids->ptr;
    a.a_scale = (const float*)a2_scale->ptr;
    if (w4)
        a.b_sf = (const uint8_t*)w2_scale->ptr;
    else
        a.b_scale = (const float*)w2_scale->ptr;
    a.sorted_w = sorted_weights ? (const float*)sorted_weights->ptr : nullptr;  // none: weight 1
    a.out_f16 = out->dtype_ == AITER_DTYPE_fp16 ? 1 : 0;
    a.out = out->ptr;
    a.M = M;
    a.N = D;
    a.num_kb = I / 128;
    a.max_m_blocks = c.max_m_blocks;
    a.out_cols = D;
    a.E = E;
    a.rows_pad = c.rows_pad;
    if (bias) {
        need_dtype(bias, AITER_DTYPE_fp32, "bias");
        need_contig(bias, "bias");
        AB_CHECK((int64_t)bias->numel_ == (int64_t)E * D, "bias must be [E, model_dim] f32");
        a.bias = (const float*)bias->ptr;
        a.bias_ld = D;
    }
    DeviceGuard dg(a2->device_id);
    CUtensorMap tmA, tmB;
    make_tmap_2d_u8(&tmA, a2->ptr, (uint64_t)c.rows_pad, I, 128, 128, true);
    if (w4) {
        make_tmap_2d_e2m1(&tmB, w2->ptr, (uint64_t)E * D, I, 128);
        launch<2, 256, true>(tmA, tmB, tmA, a, a2->device_id, as_stream(stream));
    } else {
        make_tmap_2d_u8(&tmB, w2->ptr, (uint64_t)E * D, I, 128, 128, true);
        launch<2, 256, false>(tmA, tmB, tmA, a, a2->device_id, as_stream(stream));
    }
}
}  // namespace

AB_ENTRY(moe_stage2_fp8_blockscale,
         (aiter_tensor_t * a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2, aiter_tensor_t* w2_scale,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m, void* stream),
         (a2, a2_scale, w2, w2_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights, out,
          block_m, stream)) {
    run_stage2(a2, a2_scale, w2, w2_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights, out,
               block_m, nullptr, stream);
}

// The same with the expert bias of the down GEMM (the exp_bias of
// moe_cktile2stages_gemm2, aiter/ops/moe_op.py:406-465): f32 [E, model_dim], added
// before the top-k weight.
AB_ENTRY(moe_stage2_fp8_blockscale_bias,
         (aiter_tensor_t * a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2, aiter_tensor_t* w2_scale,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m, aiter_tensor_t* bias, void* stream),
         (a2, a2_scale, w2, w2_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights, out,
          block_m, bias, stream)) {
    run_stage2(a2, a2_scale, w2, w2_scale, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights, out,
               block_m, bias, stream);
}

// A8W4 grouped GEMMs (the MXFP4 path of moe_cktile2stages_gemm1 / gemm2,
// aiter/ops/moe_op.py:343-465): fp8 1x128 sorted activations x MXFP4 weights kept at
// 4 bits in HBM, their e8m0 scales (arranged by mxfp4_moe_weight_scale_chunks)
// applied by tcgen05.mma.kind::mxf8f6f4.block_scale, the activation scales promoted
// per 128-wide K block as in the FP8 kernels.  Same options as the _bias entries.
AB_ENTRY(moe_stage1_a8w4,
         (aiter_tensor_t * a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1, aiter_tensor_t* w1_scale_chunks,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m, int64_t activation,
          aiter_tensor_t* sorted_weights, int64_t inter_dtype, aiter_tensor_t* bias, void* stream),
         (a1, a1_scale, w1, w1_scale_chunks, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale,
          num_tokens, block_m, activation, sorted_weights, inter_dtype, bias, stream)) {
    run_stage1(a1, a1_scale, w1, w1_scale_chunks, sorted_token_ids, sorted_expert_ids, num_valid_ids, out, out_scale,
               num_tokens, block_m, activation, sorted_weights, inter_dtype, bias, stream, true);
}

AB_ENTRY(moe_stage2_a8w4,
         (aiter_tensor_t * a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2, aiter_tensor_t* w2_scale_chunks,
          aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
          aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m, aiter_tensor_t* bias, void* stream),
         (a2, a2_scale, w2, w2_scale_chunks, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights, out,
          block_m, bias, stream)) {
    run_stage2(a2, a2_scale, w2, w2_scale_chunks, sorted_token_ids, sorted_expert_ids, num_valid_ids, sorted_weights,
               out, block_m, bias, stream, true);
}

// Error word of every mbarrier wait outside the allreduce context: this unit's
// (the grouped GEMMs) folded with the bf16 GEMM unit's.
extern "C" int aiter_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, sm100::g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        int z = 0;
        cudaMemcpyToSymbol(sm100::g_device_error, &z, sizeof(int));
    }
    const int g = ab::gemm_bf16_device_error(clear);
    if (g < 0) return -1;
    return v ? v : g;
}
