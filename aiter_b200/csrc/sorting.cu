// moe_sorting: expert-major, block-padded permutation of the (token, slot) pairs.
//
// Output contract (bit-exact with moe_sorting_native, op_tests/test_moe_sorting.py:15-70,
// and the layout of csrc/include/moe_sorting_opus.h:274-322):
//   * experts in ascending id; an expert with no tokens takes no block;
//   * inside an expert, entries in ascending (token, slot) order;
//   * entry = token | slot << 24, padding = tokens_dim | topk << 24 with weight 0;
//   * sorted_expert_ids[b] = expert (its local id under local_expert_mask);
//   * num_valid_ids = {padded total, tokens}; moe_buf[:tokens] zeroed.
//
// B200 design: the (token, slot) list is cut into chunks of <= 1024 entries in
// row-major order.  Ranks inside a chunk come from warp match masks
// (__match_any_sync + popc of the lower lanes) and a per-expert exclusive scan
// over the 32 warps, so the scatter is stable without atomics.
//   * one-shot (small inputs): one CTA counts, scans and scatters chunk by chunk;
//   * multi-CTA: kernel 1 writes per-chunk expert histograms to the workspace,
//     kernel 2 has every chunk-CTA rebuild the expert bases from the histograms and
//     scatter its chunk.  Extra CTAs of the first kernel zero moe_buf meanwhile.
#include <cuda.h>  // CUcontext / CUresult types only: no driver library is linked

#include <mutex>

#include "common.cuh"

// Size of the library-owned sorting scratch of moe_sorting_fwd_static_scratch.
constexpr int kSortScratchInts = 262144;  // 1 MiB

namespace {

constexpr int kThreads = 1024;
constexpr int kChunk = 1024;  // entries per chunk (one per thread)

struct SortArgs {
    const int* topk_ids;
    const float* topk_w;
    const int* expert_mask;   // may be null
    const int* local_tokens;  // may be null
    int* sorted_ids;
    float* sorted_w;
    int* sorted_eids;
    int* num_valid;
    int M, topk, E, B;
    int tpc;  // tokens per chunk
    int nchunks;
    uint8_t* moe_buf;
    int64_t moe_row_bytes;
    int* counts;  // workspace [nchunks][E]
    int* inv;     // optional [M * topk]: sorted row of (token, slot), -1 if not routed here
};

__device__ __forceinline__ int num_tokens(const SortArgs& a) {
    return a.local_tokens ? min(max(a.local_tokens[0], 0), a.M) : a.M;
}

__device__ __forceinline__ bool expert_on(const SortArgs& a, int e) {
    return e >= 0 && e < a.E && (a.expert_mask == nullptr || a.expert_mask[e] != 0);
}

// Zero moe_buf[:tokens] with 16-byte stores, grid-stride over `nblk` CTAs.
__device__ void zero_moe_buf(const SortArgs& a, int blk, int nblk) {
    if (!a.moe_buf) return;
    const int64_t bytes = (int64_t)num_tokens(a) * a.moe_row_bytes;
    const int64_t n16 = bytes / 16;
    uint4* p = reinterpret_cast<uint4*>(a.moe_buf);
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int64_t i = (int64_t)blk * blockDim.x + threadIdx.x; i < n16; i += (int64_t)nblk * blockDim.x)
        p[i] = z;
    if (blk == 0)
        for (int64_t i = n16 * 16 + threadIdx.x; i < bytes; i += blockDim.x) a.moe_buf[i] = 0;
}

// Expert bases from totals: padded sizes, exclusive scan, local ids; CTA `writer`
// also emits sorted_expert_ids, the padding entries and num_valid_ids.
// smem: tot[E] (in: totals), base[E] (out), scratch[kThreads]
__device__ void build_bases(const SortArgs& a, const int* tot, int* base, int* scratch, bool writer) {
    const int tid = threadIdx.x;
    // per-thread serial scan over a contiguous slice of experts, then block scan
    const int per = (a.E + kThreads - 1) / kThreads;
    const int e0 = tid * per, e1 = min(e0 + per, a.E);
    int run = 0, lrun = 0;
    for (int e = e0; e < e1; ++e) {
        bool on = expert_on(a, e);
        int padded = on ? (tot[e] + a.B - 1) / a.B * a.B : 0;
        run += padded;
        lrun += on ? 1 : 0;
    }
    // inclusive scan of (run, lrun) across threads, packed in two passes
    scratch[tid] = run;
    __syncthreads();
    for (int o = 1; o < kThreads; o <<= 1) {
        int v = tid >= o ? scratch[tid - o] : 0;
        __syncthreads();
        scratch[tid] += v;
        __syncthreads();
    }
    int excl = scratch[tid] - run;
    const int total = scratch[kThreads - 1];
    __syncthreads();
    scratch[tid] = lrun;
    __syncthreads();
    for (int o = 1; o < kThreads; o <<= 1) {
        int v = tid >= o ? scratch[tid - o] : 0;
        __syncthreads();
        scratch[tid] += v;
        __syncthreads();
    }
    int lexcl = scratch[tid] - lrun;
    const int tokens = num_tokens(a);
    const int pad_id = (a.topk << 24) | a.M;
    for (int e = e0; e < e1; ++e) {
        bool on = expert_on(a, e);
        int cnt = on ? tot[e] : 0;
        int padded = on ? (cnt + a.B - 1) / a.B * a.B : 0;
        base[e] = excl;
        if (writer && padded > 0) {
            for (int b = excl / a.B; b < (excl + padded) / a.B; ++b) a.sorted_eids[b] = lexcl;
            for (int i = excl + cnt; i < excl + padded; ++i) {
                a.sorted_ids[i] = pad_id;
                a.sorted_w[i] = 0.f;
            }
        }
        excl += padded;
        lexcl += on ? 1 : 0;
    }
    if (writer && tid == 0) {
        a.num_valid[0] = total;
        a.num_valid[1] = tokens;
    }
    __syncthreads();
}

// Stable scatter of one chunk.  off[e] = first slot of expert e for this chunk.
// wcnt: smem [32][E] scratch; ctot (smem [E], may be null) receives the chunk's
// per-expert counts.
__device__ void scatter_chunk(const SortArgs& a, int chunk, const int* off, int* wcnt, int* ctot) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tokens = num_tokens(a);
    for (int i = tid; i < 32 * a.E; i += kThreads) wcnt[i] = 0;
    __syncthreads();
    const int t0 = chunk * a.tpc;
    const int n_ent = max(0, min(a.tpc, tokens - t0)) * a.topk;   // routed entries
    const int n_all = max(0, min(a.tpc, a.M - t0)) * a.topk;      // rows of the inverse map
    int e = -1, t = 0, s = 0;
    if (tid < n_all) {
        t = t0 + tid / a.topk;
        s = tid % a.topk;
    }
    if (tid < n_ent) {
        e = a.topk_ids[(int64_t)t * a.topk + s];
        if (!expert_on(a, e)) e = -1;
    }
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(grp & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp * a.E + e] = __popc(grp);
    __syncthreads();
    // exclusive scan over the 32 warps, per expert
    for (int x = tid; x < a.E; x += kThreads) {
        int run = 0;
        for (int w = 0; w < 32; ++w) {
            int c = wcnt[w * a.E + x];
            wcnt[w * a.E + x] = run;
            run += c;
        }
        if (ctot) ctot[x] = run;
    }
    __syncthreads();
    if (e >= 0) {
        const int pos = off[e] + wcnt[warp * a.E + e] + rank;
        a.sorted_ids[pos] = t | (s << 24);
        a.sorted_w[pos] = a.topk_w[(int64_t)t * a.topk + s];
        if (a.inv) a.inv[(int64_t)t * a.topk + s] = pos;
    } else if (a.inv && tid < n_all) {
        a.inv[(int64_t)t * a.topk + s] = -1;
    }
    __syncthreads();
}

// One-shot: a single CTA sorts everything; CTAs > 0 zero moe_buf.
__global__ void __launch_bounds__(kThreads) sort_oneshot_kernel(SortArgs a) {
    extern __shared__ int smem[];
    if (blockIdx.x > 0) {
        zero_moe_buf(a, blockIdx.x - 1, gridDim.x - 1);
        return;
    }
    int* tot = smem;                 // [E]
    int* base = tot + a.E;           // [E]
    int* wcnt = base + a.E;          // [32][E]
    int* scratch = wcnt + 32 * a.E;  // [kThreads]
    const int tid = threadIdx.x;
    const int tokens = num_tokens(a);
    for (int e = tid; e < a.E; e += kThreads) tot[e] = 0;
    __syncthreads();
    const int n_all = tokens * a.topk;
    for (int i = tid; i < n_all; i += kThreads) {
        int e = a.topk_ids[i];
        if (expert_on(a, e)) atomicAdd(&tot[e], 1);
    }
    __syncthreads();
    build_bases(a, tot, base, scratch, true);
    // base[e] advances chunk by chunk; tot is reused for the chunk counts
    const int rows_done = a.inv ? a.M : tokens;
    for (int c = 0; c * a.tpc < rows_done; ++c) {
        scatter_chunk(a, c, base, wcnt, tot);
        for (int e = tid; e < a.E; e += kThreads) base[e] += tot[e];
        __syncthreads();
    }
}

// Multi-CTA phase 1: per-chunk histograms; CTAs past nchunks zero moe_buf.
__global__ void __launch_bounds__(kThreads) sort_count_kernel(SortArgs a) {
    extern __shared__ int smem[];
    if ((int)blockIdx.x >= a.nchunks) {
        zero_moe_buf(a, blockIdx.x - a.nchunks, gridDim.x - a.nchunks);
        return;
    }
    const int c = blockIdx.x, tid = threadIdx.x;
    int* h = smem;
    for (int e = tid; e < a.E; e += kThreads) h[e] = 0;
    __syncthreads();
    const int tokens = num_tokens(a);
    const int t0 = c * a.tpc;
    const int n_ent = max(0, min(a.tpc, tokens - t0)) * a.topk;
    if (tid < n_ent) {
        int e = a.topk_ids[(int64_t)t0 * a.topk + tid];
        if (expert_on(a, e)) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = tid; e < a.E; e += kThreads) a.counts[(int64_t)c * a.E + e] = h[e];
}

// Multi-CTA phase 2: every chunk-CTA rebuilds the bases and scatters its chunk.
__global__ void __launch_bounds__(kThreads) sort_scatter_kernel(SortArgs a) {
    extern __shared__ int smem[];
    int* tot = smem;
    int* base = tot + a.E;
    int* wcnt = base + a.E;
    int* scratch = wcnt + 32 * a.E;
    const int c = blockIdx.x, tid = threadIdx.x;
    for (int e = tid; e < a.E; e += kThreads) {
        int t = 0;
        for (int q = 0; q < a.nchunks; ++q) t += a.counts[(int64_t)q * a.E + e];
        tot[e] = t;
    }
    __syncthreads();
    build_bases(a, tot, base, scratch, c == 0);
    for (int e = tid; e < a.E; e += kThreads) {
        int p = 0;
        for (int q = 0; q < c; ++q) p += a.counts[(int64_t)q * a.E + e];
        base[e] += p;
    }
    __syncthreads();
    scatter_chunk(a, c, base, wcnt, nullptr);
}

size_t smem_bytes(int E) { return (size_t)(2 * E + 32 * E + kThreads) * sizeof(int); }

int tokens_per_chunk(int topk) { return topk >= kChunk ? 1 : kChunk / topk; }

bool use_oneshot(int64_t M, int64_t topk, int64_t policy) {
    if (policy == 1) return true;
    if (policy == 2) return false;
    return M * topk <= 4 * kChunk;
}

}  // namespace

extern "C" int64_t moe_sorting_get_workspace_size(int64_t num_tokens, int64_t num_experts,
                                                  int64_t topk, int64_t dispatch_policy) {
    if (num_tokens <= 0 || topk <= 0 || num_experts <= 0) return 0;
    if (use_oneshot(num_tokens, topk, dispatch_policy)) return 0;
    int64_t tpc = tokens_per_chunk((int)topk);
    int64_t nchunks = (num_tokens + tpc - 1) / tpc;
    return nchunks * num_experts * (int64_t)sizeof(int);
}

AB_ENTRY(moe_sorting_fwd,
         (aiter_tensor_t * topk_ids, aiter_tensor_t* topk_weights, aiter_tensor_t* sorted_token_ids,
          aiter_tensor_t* sorted_weights, aiter_tensor_t* sorted_expert_ids,
          aiter_tensor_t* num_valid_ids, aiter_tensor_t* moe_buf, int64_t num_experts,
          int64_t unit_size, aiter_tensor_t* local_expert_mask, aiter_tensor_t* num_local_tokens,
          int64_t dispatch_policy, aiter_tensor_t* workspace, aiter_tensor_t* token_sorted_pos,
          void* stream),
         (topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids,
          num_valid_ids, moe_buf, num_experts, unit_size, local_expert_mask, num_local_tokens,
          dispatch_policy, workspace, token_sorted_pos, stream)) {
    using namespace ab;
    need(topk_ids, "topk_ids");
    need(topk_weights, "topk_weights");
    need(sorted_token_ids, "sorted_token_ids");
    need(sorted_weights, "sorted_weights");
    need(sorted_expert_ids, "sorted_expert_ids");
    need(num_valid_ids, "num_valid_ids");
    need_dtype(topk_ids, AITER_DTYPE_i32, "topk_ids");
    need_dtype(topk_weights, AITER_DTYPE_fp32, "topk_weights");  // moe_sorting_kernels.cu:23-25
    need_dtype(sorted_token_ids, AITER_DTYPE_i32, "sorted_token_ids");
    need_dtype(sorted_weights, AITER_DTYPE_fp32, "sorted_weights");
    need_dtype(sorted_expert_ids, AITER_DTYPE_i32, "sorted_expert_ids");
    need_dtype(num_valid_ids, AITER_DTYPE_i32, "num_valid_ids");
    need_ndim(topk_ids, 2, "topk_ids");
    need_contig(topk_ids, "topk_ids");
    need_contig(topk_weights, "topk_weights");
    AB_CHECK(topk_weights->shape[0] == topk_ids->shape[0] && topk_weights->shape[1] == topk_ids->shape[1],
             "topk_weights must match topk_ids");
    const int64_t M = topk_ids->shape[0], K = topk_ids->shape[1];
    AB_CHECK(M < (1 << 24), "at most 2^24-1 tokens");
    AB_CHECK(K >= 1 && K < 256, "topk must be in [1, 255]");
    AB_CHECK(num_experts >= 1 && num_experts <= 1024, "num_experts must be in [1, 1024]");
    AB_CHECK(unit_size >= 1 && unit_size <= 1024, "bad unit_size ", unit_size);
    const int64_t max_pad = M * K + num_experts * unit_size - K;
    const int64_t max_blk = (max_pad + unit_size - 1) / unit_size;
    AB_CHECK((int64_t)sorted_token_ids->numel_ >= max_pad, "sorted_token_ids needs ", max_pad, " elements");
    AB_CHECK((int64_t)sorted_weights->numel_ >= max_pad, "sorted_weights needs ", max_pad, " elements");
    AB_CHECK((int64_t)sorted_expert_ids->numel_ >= max_blk, "sorted_expert_ids needs ", max_blk, " elements");
    AB_CHECK(num_valid_ids->numel_ >= 2, "num_valid_ids needs 2 elements");
    if (local_expert_mask) {
        need_dtype(local_expert_mask, AITER_DTYPE_i32, "local_expert_mask");
        AB_CHECK((int64_t)local_expert_mask->numel_ >= num_experts, "local_expert_mask too small");
    }
    if (num_local_tokens) need_dtype(num_local_tokens, AITER_DTYPE_i32, "num_local_tokens");
    if (token_sorted_pos) {
        need_dtype(token_sorted_pos, AITER_DTYPE_i32, "token_sorted_pos");
        AB_CHECK((int64_t)token_sorted_pos->numel_ >= M * K, "token_sorted_pos needs M*topk elements");
    }

    SortArgs a{};
    a.topk_ids = (const int*)topk_ids->ptr;
    a.topk_w = (const float*)topk_weights->ptr;
    a.expert_mask = local_expert_mask ? (const int*)local_expert_mask->ptr : nullptr;
    a.local_tokens = num_local_tokens ? (const int*)num_local_tokens->ptr : nullptr;
    a.sorted_ids = (int*)sorted_token_ids->ptr;
    a.sorted_w = (float*)sorted_weights->ptr;
    a.sorted_eids = (int*)sorted_expert_ids->ptr;
    a.num_valid = (int*)num_valid_ids->ptr;
    a.M = (int)M;
    a.topk = (int)K;
    a.E = (int)num_experts;
    a.B = (int)unit_size;
    a.tpc = tokens_per_chunk((int)K);
    a.nchunks = (int)((M + a.tpc - 1) / a.tpc);
    a.inv = token_sorted_pos ? (int*)token_sorted_pos->ptr : nullptr;
    int64_t moe_bytes = 0;
    if (moe_buf && moe_buf->numel_ > 0) {
        need_contig(moe_buf, "moe_buf");
        AB_CHECK(moe_buf->shape[0] >= M, "moe_buf needs at least M rows");
        a.moe_buf = (uint8_t*)moe_buf->ptr;
        a.moe_row_bytes = (int64_t)(moe_buf->numel_ / moe_buf->shape[0]) * (int64_t)elem_size(moe_buf->dtype_);
        AB_CHECK(((uintptr_t)a.moe_buf & 15) == 0, "moe_buf must be 16-byte aligned");
        moe_bytes = M * a.moe_row_bytes;
    }
    DeviceGuard dg(topk_ids->device_id);
    const int dev = topk_ids->device_id;
    const size_t smem = smem_bytes(a.E);
    AB_CHECK(smem <= 227 * 1024, "too many experts for the sorting kernel");
    const int zero_ctas = moe_bytes > 0
        ? (int)std::min<int64_t>((moe_bytes + kThreads * 16 * 4 - 1) / (kThreads * 16 * 4), 2 * num_sms(dev))
        : 0;
    cudaStream_t st = as_stream(stream);
    if (M == 0) {
        // nothing routed: num_valid = {0, 0}
        AB_CUDA(cudaMemsetAsync(a.num_valid, 0, 2 * sizeof(int), st));
        return;
    }
    if (use_oneshot(M, K, dispatch_policy)) {
        ab::set_max_smem_once((const void*)sort_oneshot_kernel, (int)smem, dev);
        sort_oneshot_kernel<<<1 + zero_ctas, kThreads, smem, st>>>(a);
        check_launch("moe_sorting_fwd(one-shot)");
        return;
    }
    const int64_t ws_need = moe_sorting_get_workspace_size(M, num_experts, K, dispatch_policy);
    AB_CHECK(workspace && workspace->ptr && (int64_t)(workspace->numel_ * elem_size(workspace->dtype_)) >= ws_need,
             "workspace of at least ", ws_need, " bytes required (moe_sorting_get_workspace_size)");
    a.counts = (int*)workspace->ptr;
    ab::set_max_smem_once((const void*)sort_count_kernel, (int)smem, dev);
    ab::set_max_smem_once((const void*)sort_scatter_kernel, (int)smem, dev);
    sort_count_kernel<<<a.nchunks + zero_ctas, kThreads, a.E * sizeof(int), st>>>(a);
    check_launch("moe_sorting_fwd(count)");
    sort_scatter_kernel<<<a.nchunks, kThreads, smem, st>>>(a);
    check_launch("moe_sorting_fwd(scatter)");
}

// ---------------------------------------------------------------------------
// moe_sorting_fwd for callers that cannot allocate device memory.
//
// Some callers of this library must not call cudaMalloc (or any allocator) once
// they are running: a serving engine that carved all free HBM into its KV-cache
// pool at start-up and treats any later allocation as a fault, or a plain C host
// program that links this library without a device allocator of its own.  For
// them the sorting histograms (the only scratch the multi-CTA sort needs) live in
// this fixed device array of 1 MiB.  CUDA loads a library's device code lazily (by
// default since CUDA 12.2), so the array is placed on a GPU when this file's code
// is first used there -- by the first call of the entry point below on that
// device, whatever its size -- and stays until the process exits.  That first call
// therefore needs the memory to be free: make it at start-up, before the caller
// takes the free HBM, and before any stream capture.
//
// In host code `g_sort_scratch` is only a stand-in symbol, not a device address:
// its address on the current device comes from cudaGetSymbolAddress, looked up on
// the device's first call and cached per device (runtime device ids 0..63)
// together with the CUDA context it belongs to; a call under another context (the
// device was reset) looks it up again.
//
// Every call uses the same array, which keeps whatever the last call wrote.  The
// count kernel overwrites every histogram entry a call reads, so nothing has to
// be cleared first.  Two calls whose kernels overlap on the GPU (different streams
// without ordering between them) race on the array; order them on one stream.
static __device__ __align__(256) int g_sort_scratch[kSortScratchInts];

namespace {

struct ScratchSlot {
    CUcontext ctx;
    int* ptr;
};
std::mutex g_scratch_mu;
ScratchSlot g_scratch_dev[64] = {};

// The current driver context, through the runtime's driver entry-point lookup (the
// library links only the CUDA runtime); null if the lookup is unavailable.
CUcontext current_context() {
    using GetCtx = CUresult (*)(CUcontext*);
    static const GetCtx fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (GetCtx) nullptr;
        return reinterpret_cast<GetCtx>(f);
    }();
    CUcontext c = nullptr;
    if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
    return c;
}

int* sort_scratch_on_current_device() {
    int dev = -1;
    AB_CUDA(cudaGetDevice(&dev));
    AB_CHECK(dev >= 0 && dev < 64, "unsupported device id ", dev);
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    ScratchSlot& slot = g_scratch_dev[dev];
    if (!slot.ptr || slot.ctx != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_sort_scratch);
        if (e != cudaSuccess || p == nullptr)
            ab::fail("cudaGetSymbolAddress(g_sort_scratch) failed: ", cudaGetErrorString(e));
        slot.ptr = static_cast<int*>(p);
        slot.ctx = ctx;
    }
    return slot.ptr;
}

}  // namespace

AB_ENTRY(moe_sorting_fwd_static_scratch,
         (aiter_tensor_t * topk_ids, aiter_tensor_t* topk_weights, aiter_tensor_t* sorted_token_ids,
          aiter_tensor_t* sorted_weights, aiter_tensor_t* sorted_expert_ids,
          aiter_tensor_t* num_valid_ids, aiter_tensor_t* moe_buf, int64_t num_experts,
          int64_t unit_size, aiter_tensor_t* local_expert_mask, aiter_tensor_t* num_local_tokens,
          int64_t dispatch_policy, aiter_tensor_t* token_sorted_pos, void* stream),
         (topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids,
          num_valid_ids, moe_buf, num_experts, unit_size, local_expert_mask, num_local_tokens,
          dispatch_policy, token_sorted_pos, stream)) {
    using namespace ab;
    need(topk_ids, "topk_ids");
    need_ndim(topk_ids, 2, "topk_ids");
    const int64_t need_bytes = moe_sorting_get_workspace_size(topk_ids->shape[0], num_experts,
                                                              topk_ids->shape[1], dispatch_policy);
    const int64_t have = (int64_t)sizeof(int) * kSortScratchInts;
    AB_CHECK(need_bytes <= have, "this sort needs ", need_bytes, " bytes of scratch but the built-in array holds ",
             have, " (", kSortScratchInts, " ints >= ceil(tokens / floor(1024 / topk)) * experts); use "
             "moe_sorting_fwd with a workspace for larger inputs");
    aiter_tensor_t ws{};
    aiter_tensor_t* wsp = nullptr;
    int* scratch = nullptr;
    {
        // every call, even one small enough for the one-CTA sort, places the array on
        // the device and caches its address, so a small call at start-up prepares
        // the device for the larger calls that follow
        DeviceGuard dg(topk_ids->device_id);
        scratch = sort_scratch_on_current_device();
    }
    if (need_bytes > 0) {
        ws.ptr = scratch;
        ws.numel_ = (size_t)have;
        ws.ndim = 1;
        ws.shape[0] = have;
        ws.strides[0] = 1;
        ws.dtype_ = AITER_DTYPE_u8;
        ws.device_id = topk_ids->device_id;
        wsp = &ws;
    }
    moe_sorting_fwd_impl(topk_ids, topk_weights, sorted_token_ids, sorted_weights, sorted_expert_ids,
                         num_valid_ids, moe_buf, num_experts, unit_size, local_expert_mask, num_local_tokens,
                         dispatch_policy, wsp, token_sorted_pos, stream);
}
