// Quick allreduce over CUDA IPC peer memory: the B200 replacement of the
// reference's QuickReduce (aiter/dist/device_communicators/quick_all_reduce.py,
// csrc/kernels/quick_all_reduce.cu:11-103, csrc/include/quick_all_reduce.cuh:581-991),
// a two-shot allreduce whose NVLink traffic is quantised to FP8, INT6 or INT4
// with one scale pair per 64 elements (or left at full precision, level FP).
//
// Every rank owns one cudaMalloc'd region, exported with cudaIpcGetMemHandle:
//   [ QrSignal (flags written by peers, own tile counters) | region 0 | region 1 ]
// A message is cut into tiles of 16384 elements; tile t has a slot per source
// rank in both regions (slot bytes depend on the level).  Per tile, CTA b:
//   1. loads the tile (8 atom rows of 2048 elements), encodes the rows owned by
//      rank r (rows r*8/W .. (r+1)*8/W - 1) and stores them into r's region 0,
//      slot [t][own rank]: every byte crosses NVLink as a store;
//   2. raises flag[0][b][own rank] on every owner and waits for its own
//      flag[0][b][s] of every source s;
//   3. as owner, decodes its rows from every source slot and sums them in rank
//      order 0..W-1 (one T rounding per add), encodes the sum once and stores it
//      into every rank's region 1, slot [t][own rank];
//   4. raises flag[1][b][own rank] everywhere, waits for every owner, decodes all
//      rows from its own region 1 and writes the output.
// Every rank decodes the same codes, so all ranks return identical bits.
//
// Flags carry per-CTA tile epochs: CTA b numbers its tiles from its own
// counter[b] (only CTA b of this rank touches it; launches are stream-ordered),
// so every rank, making the same calls with the same grids, counts the same
// epochs per CTA index, in eager calls and graph replays alike.  Flags are
// compared with a wrap-safe >=.  Reusing the regions across calls needs no extra
// barrier: a rank starts call n+1 only after its call n has read every owner's
// region-1 sums for every tile, which each owner wrote after finishing its region-0
// reads of call n; and an owner writes region 1 of call n+1 only after every
// source's region-0 flag of call n+1, which a source raises only after finishing
// call n (including its region-1 reads).
// Every wait gives up after 2 s, sets the device error word (qr_device_error) and
// ends the kernel; the communicator is unusable afterwards.
#include <mutex>
#include <vector>

#include "ipc.cuh"
#include "quick_reduce.cuh"

namespace {

using namespace qr;

constexpr int kQrMaxBlocks = 1024;
constexpr size_t kQrSignalPad = 128 * 1024;
constexpr int64_t kQrDefaultMax = (int64_t)1 << 31;  // qr_max_size(): 2 GiB

struct QrSignal {
    uint32_t flag[2][kQrMaxBlocks][ipc::kMaxRanks];  // [phase][CTA][source rank]
    uint32_t counter[kQrMaxBlocks];                  // tiles done per CTA index (own)
};
static_assert(sizeof(QrSignal) <= kQrSignalPad, "signal block exceeds its pad");

struct QrPeers {
    QrSignal* sig[ipc::kMaxRanks];
    uint8_t* region[2][ipc::kMaxRanks];
};

__device__ __forceinline__ uint32_t ld_cg32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_cg16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Encode this thread's 8 values; the scale pair comes from the 8-lane group.
template <typename T, int L>
__device__ __forceinline__ Enc encode_atom(const float (&x)[8]) {
    if constexpr (L == kFP) {
        Enc e{};
        e.code = pack_t<T>(x);
        return e;
    } else {
        Stats s = local_stats<L>(x);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            Stats q;
            q.a_e = __shfl_xor_sync(0xffffffffu, s.a_e, o);
            q.a_o = __shfl_xor_sync(0xffffffffu, s.a_o, o);
            if constexpr (L != kFP8) {
                q.b_e = __shfl_xor_sync(0xffffffffu, s.b_e, o);
                q.b_o = __shfl_xor_sync(0xffffffffu, s.b_o, o);
            } else {
                q.b_e = q.b_o = 0.0f;
            }
            s = merge_stats<L>(s, q);
        }
        float de, dd;
        group_scales<T, L>(s, de, dd);
        return encode_with<T, L>(x, de, dd);
    }
}

template <int L>
__device__ __forceinline__ void store_enc(uint8_t* row, const Enc& e, int tid) {
    if constexpr (L == kFP) {
        reinterpret_cast<uint4*>(row)[tid] = e.code;
    } else {
        if constexpr (L == kFP8)
            reinterpret_cast<uint2*>(row)[tid] = make_uint2(e.code.x, e.code.y);
        else
            reinterpret_cast<uint32_t*>(row)[tid] = e.code.x;
        if constexpr (L == kINT6)
            reinterpret_cast<uint16_t*>(row + RowLayout<kINT6>::kHiOff)[tid] = (uint16_t)e.code.y;
        if ((tid & 7) == 0) reinterpret_cast<uint32_t*>(row + RowLayout<L>::kScaleOff)[tid >> 3] = e.scale;
    }
}

// Rows in the regions are written by peers: read them past L1.
template <int L>
__device__ __forceinline__ Enc load_enc(const uint8_t* row, int tid) {
    Enc e{};
    if constexpr (L == kFP) {
        e.code = ipc::ld_cg(row + (size_t)tid * 16);
    } else {
        if constexpr (L == kFP8) {
            const uint2 v = ipc::ld_cg8(row + (size_t)tid * 8);
            e.code.x = v.x;
            e.code.y = v.y;
        } else {
            e.code.x = ld_cg32(row + (size_t)tid * 4);
        }
        if constexpr (L == kINT6) e.code.y = ld_cg16(row + RowLayout<kINT6>::kHiOff + (size_t)tid * 2);
        e.scale = ld_cg32(row + RowLayout<L>::kScaleOff + (size_t)(tid >> 3) * 4);
    }
    return e;
}

// Raise this CTA's flag `phase` on every rank, then wait for every rank's.
__device__ __forceinline__ bool exchange(const QrPeers& P, int rank, int world, int phase, uint32_t epoch) {
    __syncthreads();
    bool ok = true;
    if ((int)threadIdx.x < world) {
        __threadfence_system();
        ipc::st_release_sys(&P.sig[threadIdx.x]->flag[phase][blockIdx.x][rank], epoch);
        ok = ipc::wait_epoch(&P.sig[rank]->flag[phase][blockIdx.x][threadIdx.x], epoch);
    }
    return __syncthreads_and(ok ? 1 : 0) != 0;
}

// IO: tensor element type; T: arithmetic type (IO, or fp16 for bf16 with cast_bf2half).
// rank < 0 emulates all W ranks in one cooperative launch on one GPU (test hook):
// rank = blockIdx.y, whose input and output sit io_stride packs apart.
template <typename IO, typename T, int L, int W>
__global__ void __launch_bounds__(kThreads)
qr_twoshot_kernel(QrPeers P, int rank_arg, const uint4* __restrict__ in, uint4* __restrict__ out, int64_t n16,
                  int ntiles, int64_t io_stride) {
    constexpr int RA = kAtoms / W;  // atom rows per owner per tile
    constexpr int64_t ROW = RowLayout<L>::kRowBytes;
    constexpr int64_t SLOT = RA * ROW;
    constexpr int64_t TILE = SLOT * W;
    const int tid = threadIdx.x;
    const int rank = rank_arg >= 0 ? rank_arg : (int)blockIdx.y;
    if (rank_arg < 0) {
        in += rank * io_stride;
        out += rank * io_stride;
    }
    __shared__ uint32_t s_epoch;
    if (tid == 0) s_epoch = P.sig[rank]->counter[blockIdx.x];
    __syncthreads();
    uint32_t epoch = s_epoch;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        ++epoch;
        const int64_t p0 = (int64_t)tile * (kTileElems / 8);
        const int64_t toff = (int64_t)tile * TILE;
        uint4 a[kAtoms];
#pragma unroll
        for (int i = 0; i < kAtoms; ++i) {
            const int64_t p = p0 + (int64_t)i * kThreads + tid;
            a[i] = p < n16 ? in[p] : make_uint4(0u, 0u, 0u, 0u);  // a partial tile reads zeros
        }
#pragma unroll
        for (int r = 0; r < W; ++r) {
            uint8_t* dst = P.region[0][r] + toff + rank * SLOT;
#pragma unroll
            for (int k = 0; k < RA; ++k) {
                float x[8];
                unpack_t<IO>(a[r * RA + k], x);
                if constexpr (!std::is_same<IO, T>::value) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) x[j] = Arith<T>::round(x[j]);
                }
                store_enc<L>(dst + k * ROW, encode_atom<T, L>(x), tid);
            }
        }
        if (!exchange(P, rank, W, 0, epoch)) break;
        float acc[RA][8];
#pragma unroll
        for (int k = 0; k < RA; ++k)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[k][j] = 0.0f;
        const uint8_t* mine0 = P.region[0][rank] + toff;
#pragma unroll
        for (int s = 0; s < W; ++s) {
#pragma unroll
            for (int k = 0; k < RA; ++k) {
                float v[8];
                decode<T, L>(load_enc<L>(mine0 + s * SLOT + k * ROW, tid), v);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[k][j] = Arith<T>::round(acc[k][j] + v[j]);
            }
        }
#pragma unroll
        for (int k = 0; k < RA; ++k) {
            const Enc e = encode_atom<T, L>(acc[k]);
#pragma unroll
            for (int r = 0; r < W; ++r) store_enc<L>(P.region[1][r] + toff + rank * SLOT + k * ROW, e, tid);
        }
        if (!exchange(P, rank, W, 1, epoch)) break;
        const uint8_t* mine1 = P.region[1][rank] + toff;
#pragma unroll
        for (int s = 0; s < W; ++s) {
#pragma unroll
            for (int k = 0; k < RA; ++k) {
                float v[8];
                decode<T, L>(load_enc<L>(mine1 + s * SLOT + k * ROW, tid), v);
                const int64_t p = p0 + (int64_t)(s * RA + k) * kThreads + tid;
                if (p < n16) out[p] = pack_t<IO>(v);
            }
        }
    }
    if (tid == 0) P.sig[rank]->counter[blockIdx.x] = epoch;
}

struct QrCtx {
    int rank = 0, world = 0, device = -1;
    int64_t region_bytes = 0;  // per region: the registered size rounded up to whole tiles
    uint8_t* base = nullptr;
    std::vector<void*> opened;
    QrPeers peers{};
    bool ready = false;
};

QrCtx* as_qr(int64_t h) {
    QrCtx* c = reinterpret_cast<QrCtx*>(h);
    AB_CHECK(c != nullptr, "null quick allreduce context");
    return c;
}

template <typename IO, typename T, int L, int W>
void launch_qr(QrCtx* c, const void* in, void* out, int64_t n16, int ntiles, cudaStream_t st) {
    auto k = qr_twoshot_kernel<IO, T, L, W>;
    int occ = 0;
    AB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, 0));
    occ = std::max(1, std::min(occ, 4));
    const int sms = ab::num_sms(c->device);
    if (c->rank >= 0) {
        // every CTA resident at once: CTA b of each rank waits only on CTA b of its peers
        const int grid = std::max(1, std::min(ntiles, std::min(kQrMaxBlocks, occ * sms)));
        k<<<grid, kThreads, 0, st>>>(c->peers, c->rank, (const uint4*)in, (uint4*)out, n16, ntiles, (int64_t)0);
        return;
    }
    // emulated ranks: W x grid CTAs, all co-resident (cooperative launch)
    const int grid = std::max(1, std::min(ntiles, std::min(kQrMaxBlocks, occ * sms / W)));
    QrPeers peers = c->peers;
    int rank = -1;
    const uint4* pin = (const uint4*)in;
    uint4* pout = (uint4*)out;
    int64_t stride = n16;
    void* args[] = {&peers, &rank, &pin, &pout, &n16, &ntiles, &stride};
    AB_CUDA(cudaLaunchCooperativeKernel((const void*)k, dim3(grid, W), dim3(kThreads), args, 0, st));
}

template <typename IO, typename T, int L>
void launch_w(QrCtx* c, const void* in, void* out, int64_t n16, int ntiles, cudaStream_t st) {
    switch (c->world) {
        case 2: launch_qr<IO, T, L, 2>(c, in, out, n16, ntiles, st); break;
        case 4: launch_qr<IO, T, L, 4>(c, in, out, n16, ntiles, st); break;
        default: launch_qr<IO, T, L, 8>(c, in, out, n16, ntiles, st); break;
    }
}

template <typename IO, typename T>
void launch_level(QrCtx* c, int level, const void* in, void* out, int64_t n16, int ntiles, cudaStream_t st) {
    switch (level) {
        case kFP8: launch_w<IO, T, kFP8>(c, in, out, n16, ntiles, st); break;
        case kINT6: launch_w<IO, T, kINT6>(c, in, out, n16, ntiles, st); break;
        case kINT4: launch_w<IO, T, kINT4>(c, in, out, n16, ntiles, st); break;
        default: launch_w<IO, T, kFP>(c, in, out, n16, ntiles, st); break;  // as the reference's dispatch
    }
}

}  // namespace

// init_custom_qr (csrc/kernels/quick_all_reduce.cu:11-26): world sizes 2, 4 and 8;
// qr_max_size <= 0 takes the default of qr_max_size().  Allocates this rank's IPC
// region (signals + 2 regions of the size rounded up to 32 KB tiles) and writes its
// 64-byte cudaIpcMemHandle to handle_out (qr_get_handle).
AB_ENTRY(init_custom_qr,
         (int64_t rank, int64_t world, int64_t qr_max_size, int64_t device, int64_t* ctx_out, void* handle_out),
         (rank, world, qr_max_size, device, ctx_out, handle_out)) {
    using namespace ab;
    AB_CHECK(world <= 8, "world size > 8 is not supported");
    AB_CHECK(world != 6, "world size == 6 is not supported");
    AB_CHECK(world % 2 == 0 && world >= 2, "Odd num gpus is not supported for now");
    AB_CHECK(rank >= 0 && rank < world, "invalid rank passed in");
    AB_CHECK(ctx_out && handle_out, "null output pointers");
    const int64_t max_bytes = qr_max_size > 0 ? qr_max_size : kQrDefaultMax;
    DeviceGuard dg((int)device);
    QrCtx* c = new QrCtx();
    c->rank = (int)rank;
    c->world = (int)world;
    c->device = (int)device;
    c->region_bytes = (max_bytes + kTileBytes - 1) / kTileBytes * kTileBytes;
    const size_t total = kQrSignalPad + 2 * (size_t)c->region_bytes;
    cudaError_t e = cudaMalloc(&c->base, total);
    if (e != cudaSuccess) {
        delete c;
        fail("cudaMalloc of the quick allreduce region failed: ", cudaGetErrorString(e));
    }
    e = cudaMemset(c->base, 0, kQrSignalPad);
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

// qr_open_handles (csrc/kernels/quick_all_reduce.cu:44-58): `handles` holds every
// rank's 64-byte handle in rank order.
AB_ENTRY(qr_open_handles, (int64_t ctx, const void* handles), (ctx, handles)) {
    using namespace ab;
    QrCtx* c = as_qr(ctx);
    AB_CHECK(!c->ready, "handles already opened");
    AB_CHECK(handles != nullptr, "null handles");
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
        c->peers.sig[p] = reinterpret_cast<QrSignal*>(b);
        c->peers.region[0][p] = b + kQrSignalPad;
        c->peers.region[1][p] = b + kQrSignalPad + c->region_bytes;
    }
    c->ready = true;
}

// qr_all_reduce (csrc/kernels/quick_all_reduce.cu:62-93): out = sum over ranks of
// inp, fp16 or bf16, through the codec of `quant_level` (0 FP, 1 FP8, 2 INT6,
// 3 INT4; any other value runs FP, as the reference's dispatch does).  bf16 with
// cast_bf2half computes in fp16.  inp and out may not alias.
AB_ENTRY(qr_all_reduce,
         (int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t quant_level, int64_t cast_bf2half,
          void* stream),
         (ctx, inp, out, quant_level, cast_bf2half, stream)) {
    using namespace ab;
    QrCtx* c = as_qr(ctx);
    AB_CHECK(c->ready, "qr_open_handles has not been called");
    need(inp, "inp");
    need(out, "out");
    AB_CHECK(inp->dtype_ == out->dtype_, "inp and out dtypes differ");
    AB_CHECK(inp->numel_ == out->numel_, "inp and out sizes differ");
    AB_CHECK(inp->dtype_ == AITER_DTYPE_fp16 || inp->dtype_ == AITER_DTYPE_bf16,
             "quick allreduce only supports float16 and bfloat16");
    need_contig(inp, "inp");
    need_contig(out, "out");
    const int64_t bytes = (int64_t)inp->numel_ * 2;
    AB_CHECK(bytes % 16 == 0, "quick allreduce size must be a multiple of 16 bytes");
    AB_CHECK(bytes <= c->region_bytes, "quick allreduce of ", bytes, " bytes exceeds the registered ",
             c->region_bytes);
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    AB_CHECK(inp->device_id == c->device && out->device_id == c->device,
             "tensor on a different device than the communicator");
    if (bytes == 0) return;
    const char* lo = (const char*)inp->ptr;
    const char* hi = (const char*)out->ptr;
    AB_CHECK(lo + bytes <= hi || hi + bytes <= lo, "inp and out must not overlap");
    DeviceGuard dg(c->device);
    const int64_t n16 = bytes / 16;
    const int64_t ntiles64 = (bytes + kTileBytes - 1) / kTileBytes;
    AB_CHECK(ntiles64 <= INT32_MAX, "message too large");
    const int ntiles = (int)ntiles64;
    const int level = (int)quant_level;
    cudaStream_t st = as_stream(stream);
    if (inp->dtype_ == AITER_DTYPE_fp16)
        launch_level<__half, __half>(c, level, inp->ptr, out->ptr, n16, ntiles, st);
    else if (cast_bf2half)
        launch_level<__nv_bfloat16, __half>(c, level, inp->ptr, out->ptr, n16, ntiles, st);
    else
        launch_level<__nv_bfloat16, __nv_bfloat16>(c, level, inp->ptr, out->ptr, n16, ntiles, st);
    check_launch("qr_all_reduce");
}

// Test hook with no reference counterpart: the quick allreduce of `world` ranks
// emulated on one GPU in one cooperative launch (CTA row y plays rank y), with
// private regions.  inp and out are [world, N]; row r of out receives rank r's
// result.  Synchronous: allocates, runs, waits and frees.
AB_ENTRY(qr_all_reduce_emulated,
         (int64_t world, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t quant_level, int64_t cast_bf2half,
          void* stream),
         (world, inp, out, quant_level, cast_bf2half, stream)) {
    using namespace ab;
    AB_CHECK(world == 2 || world == 4 || world == 8, "world size must be 2, 4 or 8");
    need(inp, "inp");
    need(out, "out");
    AB_CHECK(inp->dtype_ == out->dtype_ && inp->numel_ == out->numel_, "inp and out must match");
    AB_CHECK(inp->dtype_ == AITER_DTYPE_fp16 || inp->dtype_ == AITER_DTYPE_bf16,
             "quick allreduce only supports float16 and bfloat16");
    need_contig(inp, "inp");
    need_contig(out, "out");
    AB_CHECK(inp->ndim == 2 && inp->shape[0] == world, "inp must be [world, N]");
    const int64_t bytes = inp->shape[1] * 2;
    AB_CHECK(bytes % 16 == 0, "N * 2 must be a multiple of 16 bytes");
    AB_CHECK(((uintptr_t)inp->ptr & 15) == 0 && ((uintptr_t)out->ptr & 15) == 0, "buffers must be 16-byte aligned");
    if (bytes == 0) return;
    DeviceGuard dg(inp->device_id);
    QrCtx c;
    c.rank = -1;
    c.world = (int)world;
    c.device = inp->device_id;
    c.region_bytes = (bytes + kTileBytes - 1) / kTileBytes * kTileBytes;
    const size_t per = kQrSignalPad + 2 * (size_t)c.region_bytes;
    AB_CUDA(cudaMalloc(&c.base, per * (size_t)world));
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemsetAsync(c.base, 0, per * (size_t)world, st);
    for (int p = 0; p < world; ++p) {
        uint8_t* b = c.base + per * p;
        c.peers.sig[p] = reinterpret_cast<QrSignal*>(b);
        c.peers.region[0][p] = b + kQrSignalPad;
        c.peers.region[1][p] = b + kQrSignalPad + c.region_bytes;
    }
    const int64_t n16 = bytes / 16;
    const int ntiles = (int)((bytes + kTileBytes - 1) / kTileBytes);
    std::string err;
    if (e == cudaSuccess) {
        try {
            if (inp->dtype_ == AITER_DTYPE_fp16)
                launch_level<__half, __half>(&c, (int)quant_level, inp->ptr, out->ptr, n16, ntiles, st);
            else if (cast_bf2half)
                launch_level<__nv_bfloat16, __half>(&c, (int)quant_level, inp->ptr, out->ptr, n16, ntiles, st);
            else
                launch_level<__nv_bfloat16, __nv_bfloat16>(&c, (int)quant_level, inp->ptr, out->ptr, n16, ntiles,
                                                           st);
        } catch (const std::exception& ex) {
            err = ex.what();
        }
        e = cudaStreamSynchronize(st);
    }
    cudaFree(c.base);
    if (!err.empty()) fail(err);
    if (e != cudaSuccess) fail("qr_all_reduce_emulated: ", cudaGetErrorString(e));
}

AB_ENTRY(qr_destroy, (int64_t ctx), (ctx)) {
    QrCtx* c = as_qr(ctx);
    {
        ab::DeviceGuard dg(c->device);
        cudaDeviceSynchronize();
        for (void* o : c->opened) cudaIpcCloseMemHandle(o);
        if (c->base) cudaFree(c->base);
    }
    delete c;
}

// qr_max_size (csrc/kernels/quick_all_reduce.cu:95-98): the default registered size.
extern "C" int64_t qr_max_size() { return kQrDefaultMax; }

// Error word of the quick allreduce's peer waits (1 = a peer did not arrive in time).
extern "C" int qr_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, ipc::g_ar_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        int z = 0;
        cudaMemcpyToSymbol(ipc::g_ar_error, &z, sizeof(int));
    }
    return v;
}
