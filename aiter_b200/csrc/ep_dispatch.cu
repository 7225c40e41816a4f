// Expert-parallel dispatch / combine over CUDA IPC peer memory (NVLink 5 /
// NVSwitch): the token all-to-all around an EP fused MoE.  Replaces the MoRI
// EpDispatchCombineOp the reference drives (aiter/dist/device_communicators/
// all2all.py:21-98; op_tests/multigpu_tests/test_dispatch_combine.py:76-171), for
// the intra-node case.
//
// Rank r owns experts [r*El, (r+1)*El).  dispatch(tokens, weights, scales, ids):
// every token goes once to every rank that owns one of its top-k experts, with its
// scales, ids and weights; rank d receives the tokens of source 0, then source 1,
// ..., each source's in token order (deterministic), plus the count.  The EP MoE
// then runs on the received rows with the rank's expert mask (masked experts
// contribute nothing).  combine(out): every received row's output goes back to
// its source; the source sums, per token, the rows of the ranks it went to, in
// rank order, in fp32, rounded once.
//
// Per rank, one cudaMalloc'd region (IPC-shared):
//   [ EpSignal | route scratch (own) | receive arrays (peers write) | combine slots ]
// Kernels, per call:
//   route   (1 CTA):  destination mask and per-destination position of every
//                     token; the count row goes to every rank (flag cnt_flag);
//                     waits for every rank's row; base offsets and the received
//                     count follow from the count matrix.
//   scatter (grid):   warp per token, pushes its row to each destination; the last
//                     CTA raises disp_done on every rank and waits for every source.
//   push    (grid):   warp per received row, pushes the output row to its source's
//                     slot [own rank][token]; the last CTA raises comb_done on every
//                     rank and waits for every destination.
//   reduce  (grid):   per token, sum of the slots of its destinations in rank order.
// Flags carry the call's epoch (a per-rank counter in device memory, the same on
// every rank because every rank makes the same calls) and are compared with a
// wrap-safe >=; every wait gives up after 2 s and sets the error word.
// Reuse across calls needs dispatch and combine to alternate: a source rewrites a
// destination's receive arrays (dispatch n+1) only after the destination's count row
// of call n+1 arrived, which the destination sends after its combine of call n,
// i.e. after its MoE of call n read the arrays; a destination rewrites a source's
// combine slots (combine n+1) only after the source's count row of call n+1.
#include <mutex>
#include <vector>

#include "ipc.cuh"

namespace {

constexpr int kW = ipc::kMaxRanks;
constexpr size_t kEpSignalPad = 64 * 1024;
constexpr int kRouteThreads = 1024;
constexpr int kThreads = 256;

struct EpSignal {
    uint32_t cnt[kW][kW];      // [source][destination] token counts of the current call
    uint32_t cnt_flag[kW];     // epoch of the count row of each source
    uint32_t disp_done[kW];    // epoch: source finished pushing its rows here
    uint32_t comb_done[kW];    // epoch: destination finished pushing its outputs here
    uint32_t epoch;            // own call counter
    uint32_t cur;              // epoch of the current call
    int32_t recv_num;          // rows received by the current call (num_local_tokens)
    int32_t ntok;              // own tokens of the current call
    uint32_t arrive_disp;      // CTAs of scatter done (last-CTA detection)
    uint32_t arrive_comb;      // CTAs of push done
    int32_t base[kW];          // own first row in each destination's arrays
};
static_assert(sizeof(EpSignal) <= kEpSignalPad, "signal block exceeds its pad");

struct EpDims {
    int world, experts_per_rank, topk, hidden;
    int tok_bytes;    // bytes of one token row (hidden * element size), multiple of 16
    int scale_dim;    // f32 scales per token (0 = none)
    int max_tokens;   // per source
    int comb_esize;   // 2 (bf16 / fp16 outputs)
};

struct EpPeers {
    EpSignal* sig[kW];
    uint8_t* tok[kW];      // [world * max_tokens][tok_bytes]
    float* scale[kW];      // [world * max_tokens][scale_dim]
    int32_t* ids[kW];      // [world * max_tokens][topk]
    float* w[kW];          // [world * max_tokens][topk]
    int32_t* src[kW];      // [world * max_tokens]: source << 24 | token
    uint8_t* comb[kW];     // [world][max_tokens][hidden] outputs pushed back
    uint8_t* mask[kW];     // own route scratch: [max_tokens] destination bitmask
    int32_t* pos[kW];      // own route scratch: [max_tokens][kW] position in each destination
};

__device__ __forceinline__ uint32_t ld_acq(const void* p) { return ipc::ld_acquire_sys((const uint32_t*)p); }

__device__ __forceinline__ uint32_t ld_cg32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Count of CTAs that finished, then (last CTA only) flags on every rank and the
// wait for every rank's.  Returns false when a wait timed out.
__device__ __forceinline__ bool last_cta_exchange(const EpPeers& P, int rank, int world, uint32_t* arrive,
                                                  int which, uint32_t epoch) {
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(arrive, 1u);
        s_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return true;
    bool ok = true;
    if ((int)threadIdx.x < world) {
        __threadfence_system();
        EpSignal* peer = P.sig[threadIdx.x];
        ipc::st_release_sys(which == 0 ? &peer->disp_done[rank] : &peer->comb_done[rank], epoch);
        EpSignal* me = P.sig[rank];
        ok = ipc::wait_epoch(which == 0 ? &me->disp_done[threadIdx.x] : &me->comb_done[threadIdx.x], epoch);
    }
    if (threadIdx.x == 0) *arrive = 0;  // every CTA has arrived: ready for the next call
    return __syncthreads_and(ok ? 1 : 0) != 0;
}

// rank_arg < 0: emulated ranks on one GPU (cooperative launch, rank = blockIdx.y).
__global__ void __launch_bounds__(kRouteThreads)
ep_route_kernel(EpPeers P, EpDims dims, int rank_arg, const int32_t* __restrict__ ids, int T, int64_t ids_stride) {
    const int rank = rank_arg >= 0 ? rank_arg : (int)blockIdx.y;
    if (rank_arg < 0) ids += rank * ids_stride;
    EpSignal* me = P.sig[rank];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int W = dims.world, K = dims.topk, El = dims.experts_per_rank;
    __shared__ uint32_t s_epoch;
    __shared__ int s_warp[32][kW];
    __shared__ int s_run[kW];
    if (tid == 0) {
        const uint32_t e = me->epoch + 1;
        me->epoch = e;
        me->cur = e;
        me->ntok = T;
        s_epoch = e;
    }
    if (tid < kW) s_run[tid] = 0;
    __syncthreads();
    const uint32_t epoch = s_epoch;
    uint8_t* mask_out = P.mask[rank];
    int32_t* pos_out = P.pos[rank];
    for (int c0 = 0; c0 < T; c0 += kRouteThreads) {
        const int t = c0 + tid;
        uint32_t m = 0;
        if (t < T) {
            for (int j = 0; j < K; ++j) {
                const int e = ids[(int64_t)t * K + j];
                if (e >= 0 && e < El * W) m |= 1u << (e / El);
            }
            mask_out[t] = (uint8_t)m;
        }
        int lpos[kW];
#pragma unroll
        for (int d = 0; d < kW; ++d) {
            const uint32_t bal = __ballot_sync(0xffffffffu, (m >> d) & 1u);
            lpos[d] = __popc(bal & ((1u << lane) - 1u));
            if (lane == 0) s_warp[warp][d] = __popc(bal);
        }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int d = 0; d < kW; ++d) {
                const int v = s_warp[lane][d];
                int incl = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int u = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += u;
                }
                const int run = s_run[d];
                s_warp[lane][d] = run + incl - v;
                __syncwarp();
                if (lane == 31) s_run[d] = run + incl;
                __syncwarp();
            }
        }
        __syncthreads();
        if (t < T) {
#pragma unroll
            for (int d = 0; d < kW; ++d)
                pos_out[(int64_t)t * kW + d] = ((m >> d) & 1u) ? s_warp[warp][d] + lpos[d] : -1;
        }
        __syncthreads();
    }
    // every rank gets this rank's count row
    bool ok = true;
    if (tid < W) {
        EpSignal* peer = P.sig[tid];
        for (int d = 0; d < W; ++d) peer->cnt[rank][d] = (uint32_t)s_run[d];
        __threadfence_system();
        ipc::st_release_sys(&peer->cnt_flag[rank], epoch);
        ok = ipc::wait_epoch(&me->cnt_flag[tid], epoch);
    }
    if (__syncthreads_and(ok ? 1 : 0) == 0) {
        if (tid == 0) me->recv_num = 0;
        return;
    }
    if (tid < W) {
        int b = 0;
        for (int s = 0; s < rank; ++s) b += (int)ld_acq(&me->cnt[s][tid]);
        me->base[tid] = b;
    }
    if (tid == 0) {
        int n = 0;
        for (int s = 0; s < W; ++s) n += (int)ld_acq(&me->cnt[s][rank]);
        me->recv_num = n;
        me->arrive_disp = 0;
        me->arrive_comb = 0;
    }
}

// Warp per token: push the token to every destination in its mask.
__global__ void __launch_bounds__(kThreads)
ep_scatter_kernel(EpPeers P, EpDims dims, int rank_arg, const uint8_t* __restrict__ tokens,
                  const float* __restrict__ scales, const int32_t* __restrict__ ids, const float* __restrict__ wts,
                  int64_t tok_stride, int64_t meta_stride) {
    const int rank = rank_arg >= 0 ? rank_arg : (int)blockIdx.y;
    if (rank_arg < 0) {
        tokens += rank * tok_stride * dims.tok_bytes;
        if (scales) scales += rank * tok_stride * dims.scale_dim;
        ids += rank * meta_stride;
        wts += rank * meta_stride;
    }
    EpSignal* me = P.sig[rank];
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * kThreads) >> 5;
    const uint32_t epoch = ld_cg32(&me->cur);
    const int T = (int)ld_cg32(&me->ntok);
    const int W = dims.world, K = dims.topk, SD = dims.scale_dim;
    const int n16 = dims.tok_bytes / 16;
    const uint8_t* mask = P.mask[rank];
    const int32_t* pos = P.pos[rank];
    for (int t = gwarp; t < T; t += nwarps) {
        const uint32_t m = mask[t];
        const uint4* srow = reinterpret_cast<const uint4*>(tokens + (int64_t)t * dims.tok_bytes);
        for (int d = 0; d < W; ++d) {
            if (!((m >> d) & 1u)) continue;
            const int64_t i = (int64_t)ld_cg32(&me->base[d]) + pos[(int64_t)t * kW + d];
            uint4* drow = reinterpret_cast<uint4*>(P.tok[d] + i * dims.tok_bytes);
            for (int c = lane; c < n16; c += 32) drow[c] = __ldg(srow + c);
            for (int c = lane; c < SD; c += 32) P.scale[d][i * SD + c] = __ldg(scales + (int64_t)t * SD + c);
            if (lane < K) {
                P.ids[d][i * K + lane] = __ldg(ids + (int64_t)t * K + lane);
                P.w[d][i * K + lane] = __ldg(wts + (int64_t)t * K + lane);
            }
            if (lane == 0) P.src[d][i] = (rank << 24) | t;
        }
    }
    last_cta_exchange(P, rank, W, &me->arrive_disp, 0, epoch);
}

// Warp per received row: push its output row to the source's slot [own rank][token].
__global__ void __launch_bounds__(kThreads)
ep_push_kernel(EpPeers P, EpDims dims, int rank_arg, const uint8_t* __restrict__ out, int64_t out_row_bytes,
               int64_t out_stride_rows) {
    const int rank = rank_arg >= 0 ? rank_arg : (int)blockIdx.y;
    if (rank_arg < 0) out += rank * out_stride_rows * out_row_bytes;
    EpSignal* me = P.sig[rank];
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * kThreads) >> 5;
    const uint32_t epoch = ld_cg32(&me->cur);
    const int recv = (int)ld_cg32(&me->recv_num);
    const int row_bytes = dims.hidden * dims.comb_esize;
    const int n16 = row_bytes / 16;
    for (int i = gwarp; i < recv; i += nwarps) {
        const uint32_t tag = ld_cg32(&P.src[rank][i]);
        const int s = (int)(tag >> 24), t = (int)(tag & 0xFFFFFF);
        const uint4* srow = reinterpret_cast<const uint4*>(out + (int64_t)i * out_row_bytes);
        uint4* drow = reinterpret_cast<uint4*>(P.comb[s] + ((int64_t)rank * dims.max_tokens + t) * row_bytes);
        for (int c = lane; c < n16; c += 32) drow[c] = srow[c];
    }
    last_cta_exchange(P, rank, dims.world, &me->arrive_comb, 1, epoch);
}

template <typename T>
struct Pk;
template <>
struct Pk<__nv_bfloat16> {
    __device__ static float2 f2(uint32_t v) { return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v)); }
    __device__ static uint32_t p2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <>
struct Pk<__half> {
    __device__ static float2 f2(uint32_t v) { return __half22float2(*reinterpret_cast<__half2*>(&v)); }
    __device__ static uint32_t p2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// out[t] = sum over the token's destinations d (rank order) of slot [d][t], fp32.
template <typename T>
__global__ void __launch_bounds__(kThreads)
ep_reduce_kernel(EpPeers P, EpDims dims, int rank_arg, uint8_t* __restrict__ y, int64_t y_row_bytes,
                 int64_t y_stride_rows) {
    const int rank = rank_arg >= 0 ? rank_arg : (int)blockIdx.y;
    if (rank_arg < 0) y += rank * y_stride_rows * y_row_bytes;
    EpSignal* me = P.sig[rank];
    const int ntok = (int)ld_cg32(&me->ntok);
    const int W = dims.world;
    const int row_bytes = dims.hidden * 2;
    const int n16 = row_bytes / 16;
    const uint8_t* mask = P.mask[rank];
    const uint8_t* comb = P.comb[rank];
    const int64_t total = (int64_t)ntok * n16;
    for (int64_t q = (int64_t)blockIdx.x * kThreads + threadIdx.x; q < total; q += (int64_t)gridDim.x * kThreads) {
        const int t = (int)(q / n16), c = (int)(q % n16);
        const uint32_t m = mask[t];
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int d = 0; d < W; ++d) {
            if (!((m >> d) & 1u)) continue;
            const uint4 v = ipc::ld_cg(comb + ((int64_t)d * dims.max_tokens + t) * row_bytes + (int64_t)c * 16);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = Pk<T>::f2(u[j]);
                a[2 * j] += f.x;
                a[2 * j + 1] += f.y;
            }
        }
        uint4 o;
        o.x = Pk<T>::p2(a[0], a[1]);
        o.y = Pk<T>::p2(a[2], a[3]);
        o.z = Pk<T>::p2(a[4], a[5]);
        o.w = Pk<T>::p2(a[6], a[7]);
        reinterpret_cast<uint4*>(y + (int64_t)t * y_row_bytes)[c] = o;
    }
}

struct EpCtx {
    int rank = 0, device = -1;
    EpDims dims{};
    int tok_dtype = 0, comb_dtype = AITER_DTYPE_bf16;
    size_t off_mask = 0, off_pos = 0, off_tok = 0, off_scale = 0, off_ids = 0, off_w = 0, off_src = 0, off_comb = 0;
    size_t total = 0;
    uint8_t* base = nullptr;
    std::vector<void*> opened;
    EpPeers peers{};
    bool ready = false;
    int last_tokens = -1;   // tokens of the last dispatch (combine's output rows)
    bool dispatched = false;
};

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

void layout(EpCtx* c) {
    const EpDims& d = c->dims;
    const size_t cap = (size_t)d.world * d.max_tokens;
    size_t o = kEpSignalPad;
    c->off_mask = o;
    o += up256((size_t)d.max_tokens);
    c->off_pos = o;
    o += up256((size_t)d.max_tokens * kW * 4);
    c->off_tok = o;
    o += up256(cap * d.tok_bytes);
    c->off_scale = o;
    o += up256(cap * d.scale_dim * 4);
    c->off_ids = o;
    o += up256(cap * d.topk * 4);
    c->off_w = o;
    o += up256(cap * d.topk * 4);
    c->off_src = o;
    o += up256(cap * 4);
    c->off_comb = o;
    o += up256(cap * (size_t)d.hidden * d.comb_esize);
    c->total = o;
}

void map_rank(EpCtx* c, int p, uint8_t* b) {
    c->peers.sig[p] = reinterpret_cast<EpSignal*>(b);
    c->peers.mask[p] = b + c->off_mask;
    c->peers.pos[p] = reinterpret_cast<int32_t*>(b + c->off_pos);
    c->peers.tok[p] = b + c->off_tok;
    c->peers.scale[p] = reinterpret_cast<float*>(b + c->off_scale);
    c->peers.ids[p] = reinterpret_cast<int32_t*>(b + c->off_ids);
    c->peers.w[p] = reinterpret_cast<float*>(b + c->off_w);
    c->peers.src[p] = reinterpret_cast<int32_t*>(b + c->off_src);
    c->peers.comb[p] = b + c->off_comb;
}

EpCtx* as_ep(int64_t h) {
    EpCtx* c = reinterpret_cast<EpCtx*>(h);
    AB_CHECK(c != nullptr, "null EP dispatch/combine context");
    return c;
}

void check_dims(const EpDims& d) {
    AB_CHECK(d.world >= 2 && d.world <= kW, "world size must be in [2, ", kW, "]");
    AB_CHECK(d.experts_per_rank > 0 && d.topk > 0 && d.topk <= 32, "need experts_per_rank > 0 and 0 < topk <= 32");
    AB_CHECK(d.hidden > 0 && d.tok_bytes % 16 == 0, "token rows must be a multiple of 16 bytes");
    AB_CHECK((d.hidden * d.comb_esize) % 16 == 0, "output rows must be a multiple of 16 bytes");
    AB_CHECK(d.scale_dim >= 0 && d.max_tokens > 0 && d.max_tokens < (1 << 24), "bad scale_dim / max_tokens");
}

int scatter_grid(int device, int rows) {
    const int warps = kThreads / 32;
    return std::max(1, std::min((rows + warps - 1) / warps, 2 * ab::num_sms(device)));
}

}  // namespace

// ep_init: this rank's region for `world` ranks, tokens of `hidden` elements of
// token_dtype (fp8, bf16 or fp16) with `scale_dim` f32 scales each, up to
// max_tokens per rank, experts_per_rank experts per rank, topk experts per token;
// outputs of comb_dtype (bf16 or fp16).  Writes the 64-byte cudaIpcMemHandle.
AB_ENTRY(ep_init,
         (int64_t rank, int64_t world, int64_t hidden, int64_t token_dtype, int64_t scale_dim, int64_t max_tokens,
          int64_t experts_per_rank, int64_t topk, int64_t comb_dtype, int64_t device, int64_t* ctx_out,
          void* handle_out),
         (rank, world, hidden, token_dtype, scale_dim, max_tokens, experts_per_rank, topk, comb_dtype, device, ctx_out,
          handle_out)) {
    using namespace ab;
    AB_CHECK(rank >= 0 && rank < world, "bad rank");
    AB_CHECK(ctx_out && handle_out, "null output pointers");
    AB_CHECK(token_dtype == AITER_DTYPE_fp8 || token_dtype == AITER_DTYPE_bf16 || token_dtype == AITER_DTYPE_fp16,
             "tokens must be fp8, bf16 or fp16");
    AB_CHECK(comb_dtype == AITER_DTYPE_bf16 || comb_dtype == AITER_DTYPE_fp16, "outputs must be bf16 or fp16");
    EpDims d{};
    d.world = (int)world;
    d.experts_per_rank = (int)experts_per_rank;
    d.topk = (int)topk;
    d.hidden = (int)hidden;
    d.tok_bytes = (int)(hidden * (int64_t)elem_size((int)token_dtype));
    d.scale_dim = (int)scale_dim;
    d.max_tokens = (int)max_tokens;
    d.comb_esize = 2;
    check_dims(d);
    DeviceGuard dg((int)device);
    EpCtx* c = new EpCtx();
    c->rank = (int)rank;
    c->device = (int)device;
    c->dims = d;
    c->tok_dtype = (int)token_dtype;
    c->comb_dtype = (int)comb_dtype;
    layout(c);
    cudaError_t e = cudaMalloc(&c->base, c->total);
    if (e != cudaSuccess) {
        delete c;
        fail("cudaMalloc of the EP region failed: ", cudaGetErrorString(e));
    }
    e = cudaMemset(c->base, 0, kEpSignalPad);
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

AB_ENTRY(ep_open_handles, (int64_t ctx, const void* handles), (ctx, handles)) {
    using namespace ab;
    EpCtx* c = as_ep(ctx);
    AB_CHECK(!c->ready, "handles already opened");
    AB_CHECK(handles != nullptr, "null handles");
    DeviceGuard dg(c->device);
    const cudaIpcMemHandle_t* hs = reinterpret_cast<const cudaIpcMemHandle_t*>(handles);
    for (int p = 0; p < c->dims.world; ++p) {
        uint8_t* b = c->base;
        if (p != c->rank) {
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
        map_rank(c, p, b);
    }
    c->ready = true;
}

// Device pointers of this rank's receive arrays: [tokens, scales, ids, weights,
// recv_num (i32 scalar), source tags], and the capacity in rows.
AB_ENTRY(ep_buffers, (int64_t ctx, int64_t* ptrs_out, int64_t* rows_out), (ctx, ptrs_out, rows_out)) {
    EpCtx* c = as_ep(ctx);
    AB_CHECK(ptrs_out && rows_out, "null output pointers");
    uint8_t* b = c->base;
    ptrs_out[0] = reinterpret_cast<int64_t>(b + c->off_tok);
    ptrs_out[1] = reinterpret_cast<int64_t>(b + c->off_scale);
    ptrs_out[2] = reinterpret_cast<int64_t>(b + c->off_ids);
    ptrs_out[3] = reinterpret_cast<int64_t>(b + c->off_w);
    ptrs_out[4] = reinterpret_cast<int64_t>(&reinterpret_cast<EpSignal*>(b)->recv_num);
    ptrs_out[5] = reinterpret_cast<int64_t>(b + c->off_src);
    *rows_out = (int64_t)c->dims.world * c->dims.max_tokens;
}

// dispatch: tokens [T, hidden] (the init dtype), weights [T, topk] f32, scales
// [T, scale_dim] f32 (NULL when scale_dim is 0), ids [T, topk] i32 global expert
// ids (ids outside [0, world * experts_per_rank) go nowhere).  T <= max_tokens.
AB_ENTRY(ep_dispatch,
         (int64_t ctx, aiter_tensor_t* tokens, aiter_tensor_t* weights, aiter_tensor_t* scales, aiter_tensor_t* ids,
          void* stream),
         (ctx, tokens, weights, scales, ids, stream)) {
    using namespace ab;
    EpCtx* c = as_ep(ctx);
    AB_CHECK(c->ready, "ep_open_handles has not been called");
    AB_CHECK(!c->dispatched, "dispatch called twice without a combine in between");
    const EpDims& d = c->dims;
    need(tokens, "tokens");
    need(weights, "weights");
    need(ids, "ids");
    need_dtype(tokens, c->tok_dtype, "tokens");
    need_dtype(weights, AITER_DTYPE_fp32, "weights");
    need_dtype(ids, AITER_DTYPE_i32, "ids");
    for (const aiter_tensor_t* t : {tokens, weights, ids}) need_contig(t, "operand");
    const int64_t T = tokens->ndim == 2 ? tokens->shape[0] : -1;
    AB_CHECK(T >= 0 && tokens->shape[1] == d.hidden, "tokens must be [T, hidden]");
    AB_CHECK(T <= d.max_tokens, "T = ", T, " exceeds max_tokens ", d.max_tokens);
    AB_CHECK((int64_t)weights->numel_ == T * d.topk && (int64_t)ids->numel_ == T * d.topk,
             "weights and ids must be [T, topk]");
    if (d.scale_dim > 0) {
        need(scales, "scales");
        need_dtype(scales, AITER_DTYPE_fp32, "scales");
        need_contig(scales, "scales");
        AB_CHECK((int64_t)scales->numel_ == T * d.scale_dim, "scales must be [T, scale_dim]");
    }
    AB_CHECK(((uintptr_t)tokens->ptr & 15) == 0, "tokens must be 16-byte aligned");
    AB_CHECK(tokens->device_id == c->device, "tensor on a different device than the communicator");
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    ep_route_kernel<<<1, kRouteThreads, 0, st>>>(c->peers, d, c->rank, (const int32_t*)ids->ptr, (int)T, 0);
    check_launch("ep_dispatch (route)");
    ep_scatter_kernel<<<scatter_grid(c->device, (int)T), kThreads, 0, st>>>(
        c->peers, d, c->rank, (const uint8_t*)tokens->ptr, d.scale_dim > 0 ? (const float*)scales->ptr : nullptr,
        (const int32_t*)ids->ptr, (const float*)weights->ptr, 0, 0);
    check_launch("ep_dispatch (scatter)");
    c->last_tokens = (int)T;
    c->dispatched = true;
}

// combine: out [rows, hidden] (comb dtype; row i = the output of received row i,
// rows >= the received count) -> y [T, hidden] for the T tokens of the last dispatch.
AB_ENTRY(ep_combine, (int64_t ctx, aiter_tensor_t* out, aiter_tensor_t* y, void* stream), (ctx, out, y, stream)) {
    using namespace ab;
    EpCtx* c = as_ep(ctx);
    AB_CHECK(c->ready, "ep_open_handles has not been called");
    AB_CHECK(c->dispatched, "combine called without a dispatch");
    const EpDims& d = c->dims;
    need(out, "out");
    need(y, "y");
    need_dtype(out, c->comb_dtype, "out");
    need_dtype(y, c->comb_dtype, "y");
    AB_CHECK(out->ndim == 2 && out->shape[1] == d.hidden && out->strides[1] == 1, "out must be [rows, hidden]");
    // the received count lives on the device: out must cover the full capacity
    AB_CHECK(out->shape[0] >= (int64_t)d.world * d.max_tokens, "out must have world * max_tokens = ",
             (int64_t)d.world * d.max_tokens, " rows (the dispatch capacity)");
    need_contig(y, "y");
    AB_CHECK(y->ndim == 2 && y->shape[0] == c->last_tokens && y->shape[1] == d.hidden,
             "y must be [tokens of the last dispatch, hidden]");
    AB_CHECK((out->strides[0] * 2) % 16 == 0 && ((uintptr_t)out->ptr & 15) == 0 && ((uintptr_t)y->ptr & 15) == 0,
             "rows must be 16-byte aligned");
    AB_CHECK(out->device_id == c->device && y->device_id == c->device,
             "tensor on a different device than the communicator");
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    // received rows are only known on the device: size the grid for the capacity
    // (warps stride over rows)
    const int cap_rows = d.world * d.max_tokens;
    ep_push_kernel<<<scatter_grid(c->device, cap_rows), kThreads, 0, st>>>(
        c->peers, d, c->rank, (const uint8_t*)out->ptr, out->strides[0] * 2, 0);
    check_launch("ep_combine (push)");
    const int64_t n16 = (int64_t)c->last_tokens * d.hidden * 2 / 16;
    const int rgrid = (int)std::max<int64_t>(1, std::min<int64_t>((n16 + kThreads - 1) / kThreads,
                                                                  4 * ab::num_sms(c->device)));
    if (c->comb_dtype == AITER_DTYPE_bf16)
        ep_reduce_kernel<__nv_bfloat16><<<rgrid, kThreads, 0, st>>>(c->peers, d, c->rank, (uint8_t*)y->ptr,
                                                                    (int64_t)d.hidden * 2, 0);
    else
        ep_reduce_kernel<__half><<<rgrid, kThreads, 0, st>>>(c->peers, d, c->rank, (uint8_t*)y->ptr,
                                                             (int64_t)d.hidden * 2, 0);
    check_launch("ep_combine (reduce)");
    c->dispatched = false;
}

// ---- emulated ranks on one GPU (test hook, no reference counterpart) --------
// ep_emu_init allocates `world` regions on one device; ep_emu_dispatch takes
// tokens [world, T, hidden], weights / ids [world, T, topk], scales [world, T,
// scale_dim] and runs every rank's route and scatter as CTA rows of one
// cooperative launch each (the ranks wait on one another inside a launch);
// ep_emu_buffers gives rank r's receive arrays; ep_emu_combine takes out [world,
// world * max_tokens, hidden] and writes y [world, T, hidden].  Synchronous.
AB_ENTRY(ep_emu_init,
         (int64_t world, int64_t hidden, int64_t token_dtype, int64_t scale_dim, int64_t max_tokens,
          int64_t experts_per_rank, int64_t topk, int64_t comb_dtype, int64_t device, int64_t* ctx_out),
         (world, hidden, token_dtype, scale_dim, max_tokens, experts_per_rank, topk, comb_dtype, device, ctx_out)) {
    using namespace ab;
    AB_CHECK(ctx_out, "null output pointer");
    AB_CHECK(token_dtype == AITER_DTYPE_fp8 || token_dtype == AITER_DTYPE_bf16 || token_dtype == AITER_DTYPE_fp16,
             "tokens must be fp8, bf16 or fp16");
    AB_CHECK(comb_dtype == AITER_DTYPE_bf16 || comb_dtype == AITER_DTYPE_fp16, "outputs must be bf16 or fp16");
    EpDims d{};
    d.world = (int)world;
    d.experts_per_rank = (int)experts_per_rank;
    d.topk = (int)topk;
    d.hidden = (int)hidden;
    d.tok_bytes = (int)(hidden * (int64_t)elem_size((int)token_dtype));
    d.scale_dim = (int)scale_dim;
    d.max_tokens = (int)max_tokens;
    d.comb_esize = 2;
    check_dims(d);
    DeviceGuard dg((int)device);
    EpCtx* c = new EpCtx();
    c->rank = -1;
    c->device = (int)device;
    c->dims = d;
    c->tok_dtype = (int)token_dtype;
    c->comb_dtype = (int)comb_dtype;
    layout(c);
    cudaError_t e = cudaMalloc(&c->base, c->total * (size_t)world);
    if (e != cudaSuccess) {
        delete c;
        fail("cudaMalloc of the emulated EP regions failed: ", cudaGetErrorString(e));
    }
    e = cudaMemset(c->base, 0, c->total * (size_t)world);
    if (e != cudaSuccess) {
        cudaFree(c->base);
        delete c;
        fail("cudaMemset failed: ", cudaGetErrorString(e));
    }
    for (int p = 0; p < world; ++p) map_rank(c, p, c->base + c->total * p);
    c->ready = true;
    *ctx_out = reinterpret_cast<int64_t>(c);
}

AB_ENTRY(ep_emu_buffers, (int64_t ctx, int64_t rank, int64_t* ptrs_out, int64_t* rows_out),
         (ctx, rank, ptrs_out, rows_out)) {
    EpCtx* c = as_ep(ctx);
    AB_CHECK(c->rank < 0, "not an emulated context");
    AB_CHECK(rank >= 0 && rank < c->dims.world && ptrs_out && rows_out, "bad arguments");
    uint8_t* b = c->base + c->total * rank;
    ptrs_out[0] = reinterpret_cast<int64_t>(b + c->off_tok);
    ptrs_out[1] = reinterpret_cast<int64_t>(b + c->off_scale);
    ptrs_out[2] = reinterpret_cast<int64_t>(b + c->off_ids);
    ptrs_out[3] = reinterpret_cast<int64_t>(b + c->off_w);
    ptrs_out[4] = reinterpret_cast<int64_t>(&reinterpret_cast<EpSignal*>(b)->recv_num);
    ptrs_out[5] = reinterpret_cast<int64_t>(b + c->off_src);
    *rows_out = (int64_t)c->dims.world * c->dims.max_tokens;
}

namespace {
int coop_grid(const void* k, int threads, int device, int world, int want) {
    int occ = 0;
    AB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, threads, 0));
    const int cap = std::max(1, occ * ab::num_sms(device) / world);
    return std::max(1, std::min(want, cap));
}
}  // namespace

AB_ENTRY(ep_emu_dispatch,
         (int64_t ctx, aiter_tensor_t* tokens, aiter_tensor_t* weights, aiter_tensor_t* scales, aiter_tensor_t* ids,
          void* stream),
         (ctx, tokens, weights, scales, ids, stream)) {
    using namespace ab;
    EpCtx* c = as_ep(ctx);
    AB_CHECK(c->rank < 0, "not an emulated context");
    const EpDims& d = c->dims;
    for (const aiter_tensor_t* t : {tokens, weights, ids}) {
        need(t, "operand");
        need_contig(t, "operand");
    }
    need_dtype(tokens, c->tok_dtype, "tokens");
    need_dtype(weights, AITER_DTYPE_fp32, "weights");
    need_dtype(ids, AITER_DTYPE_i32, "ids");
    AB_CHECK(tokens->ndim == 3 && tokens->shape[0] == d.world && tokens->shape[2] == d.hidden,
             "tokens must be [world, T, hidden]");
    const int64_t T = tokens->shape[1];
    AB_CHECK(T <= d.max_tokens, "T exceeds max_tokens");
    AB_CHECK((int64_t)ids->numel_ == d.world * T * d.topk && (int64_t)weights->numel_ == d.world * T * d.topk,
             "ids and weights must be [world, T, topk]");
    const float* sp = nullptr;
    if (d.scale_dim > 0) {
        need(scales, "scales");
        need_dtype(scales, AITER_DTYPE_fp32, "scales");
        need_contig(scales, "scales");
        AB_CHECK((int64_t)scales->numel_ == d.world * T * d.scale_dim, "scales must be [world, T, scale_dim]");
        sp = (const float*)scales->ptr;
    }
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    EpPeers peers = c->peers;
    EpDims dims = d;
    int rank = -1, Ti = (int)T;
    const int32_t* idp = (const int32_t*)ids->ptr;
    int64_t ids_stride = T * d.topk;
    void* rargs[] = {&peers, &dims, &rank, &idp, &Ti, &ids_stride};
    AB_CUDA(cudaLaunchCooperativeKernel((const void*)ep_route_kernel, dim3(1, d.world), dim3(kRouteThreads), rargs,
                                        0, st));
    const uint8_t* tp = (const uint8_t*)tokens->ptr;
    const float* wp = (const float*)weights->ptr;
    int64_t tok_stride = T, meta_stride = T * d.topk;
    const int g = coop_grid((const void*)ep_scatter_kernel, kThreads, c->device, d.world,
                            std::max<int>(1, (int)((T + 7) / 8)));
    void* sargs[] = {&peers, &dims, &rank, &tp, &sp, &idp, &wp, &tok_stride, &meta_stride};
    AB_CUDA(cudaLaunchCooperativeKernel((const void*)ep_scatter_kernel, dim3(g, d.world), dim3(kThreads), sargs, 0,
                                        st));
    AB_CUDA(cudaStreamSynchronize(st));
    c->last_tokens = (int)T;
    c->dispatched = true;
}

AB_ENTRY(ep_emu_combine, (int64_t ctx, aiter_tensor_t* out, aiter_tensor_t* y, void* stream), (ctx, out, y, stream)) {
    using namespace ab;
    EpCtx* c = as_ep(ctx);
    AB_CHECK(c->rank < 0, "not an emulated context");
    AB_CHECK(c->dispatched, "combine called without a dispatch");
    const EpDims& d = c->dims;
    need(out, "out");
    need(y, "y");
    need_dtype(out, c->comb_dtype, "out");
    need_dtype(y, c->comb_dtype, "y");
    need_contig(out, "out");
    need_contig(y, "y");
    const int64_t cap = (int64_t)d.world * d.max_tokens;
    AB_CHECK(out->ndim == 3 && out->shape[0] == d.world && out->shape[1] == cap && out->shape[2] == d.hidden,
             "out must be [world, world * max_tokens, hidden]");
    AB_CHECK(y->ndim == 3 && y->shape[0] == d.world && y->shape[1] == c->last_tokens && y->shape[2] == d.hidden,
             "y must be [world, T, hidden]");
    DeviceGuard dg(c->device);
    cudaStream_t st = as_stream(stream);
    EpPeers peers = c->peers;
    EpDims dims = d;
    int rank = -1;
    const uint8_t* op = (const uint8_t*)out->ptr;
    int64_t row_bytes = (int64_t)d.hidden * 2, out_stride = cap;
    const int g = coop_grid((const void*)ep_push_kernel, kThreads, c->device, d.world, (int)((cap + 7) / 8));
    void* pargs[] = {&peers, &dims, &rank, &op, &row_bytes, &out_stride};
    AB_CUDA(cudaLaunchCooperativeKernel((const void*)ep_push_kernel, dim3(g, d.world), dim3(kThreads), pargs, 0, st));
    const int64_t n16 = (int64_t)c->last_tokens * d.hidden * 2 / 16;
    const int rg = (int)std::max<int64_t>(1, std::min<int64_t>((n16 + kThreads - 1) / kThreads, 256));
    const int64_t y_stride = c->last_tokens;
    if (c->comb_dtype == AITER_DTYPE_bf16)
        ep_reduce_kernel<__nv_bfloat16><<<dim3(rg, d.world), kThreads, 0, st>>>(peers, d, -1, (uint8_t*)y->ptr,
                                                                                row_bytes, y_stride);
    else
        ep_reduce_kernel<__half><<<dim3(rg, d.world), kThreads, 0, st>>>(peers, d, -1, (uint8_t*)y->ptr, row_bytes,
                                                                         y_stride);
    check_launch("ep_emu_combine (reduce)");
    AB_CUDA(cudaStreamSynchronize(st));
    c->dispatched = false;
}

AB_ENTRY(ep_destroy, (int64_t ctx), (ctx)) {
    EpCtx* c = as_ep(ctx);
    {
        ab::DeviceGuard dg(c->device);
        cudaDeviceSynchronize();
        for (void* o : c->opened) cudaIpcCloseMemHandle(o);
        if (c->base) cudaFree(c->base);
    }
    delete c;
}

// Error word of the EP kernels' peer waits (1 = a peer did not arrive within 2 s).
extern "C" int ep_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, ipc::g_ar_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        int z = 0;
        cudaMemcpyToSymbol(ipc::g_ar_error, &z, sizeof(int));
    }
    return v;
}
