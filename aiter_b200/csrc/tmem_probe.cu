// Diagnostic: TMEM -> register read throughput per SM (`tcgen05.ld`), the resource the
// grouped GEMM's exact per-128-K block-scale promotion consumes (every K block's fp32
// accumulator slab is read once by the epilogue warps).  One CTA per SM (forced by its
// shared-memory request), 512 TMEM columns allocated, each warp reading its own
// subpartition's lanes over its share of the columns `iters` times.  Every loop is
// bounded and the only synchronisation is __syncthreads, so the kernel cannot wait on
// anything outside itself.  Not on the MoE path; `bench.py --mode tmem_ld` runs it.
#include "common.cuh"
#include "sm100.cuh"

namespace {

using namespace sm100;

// 16 TMEM lanes x 256 bits x 4 (16 lanes x 32 columns): 16 registers per thread
__device__ __forceinline__ void ld16x256b_x4(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr));
}

// 32 TMEM lanes x 64 consecutive columns: 64 registers per thread
__device__ __forceinline__ void ld32x32b_x64(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
        "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63"
        "}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
}

constexpr int kCols = 512;
constexpr int kSmemBytes = 200 * 1024;  // > half of the SM's shared memory: one CTA per SM

// SHAPE 0: 32x32b loads of X columns (16 or 32), one wait per load; SHAPE 1: two 32x32b.x32
// loads (64 columns) per wait; SHAPE 2: 16x32bx2.x32 (16 lanes, 64 columns) per wait;
// SHAPE 3: 16x256b.x4 at lane offsets 0 and 16 (32 lanes, 32 columns) per wait;
// SHAPE 4: the promotion epilogue's pattern, 32x32b.x32 then 32 FMAs into 128 accumulators;
// SHAPE 5: one 32x32b.x64 load (64 columns) per wait.
template <int NW, int SHAPE, int X>
__global__ void __launch_bounds__(NW * 32, 1) tmem_ld_kernel(int iters, long long* cycles, float* sink) {
    __shared__ uint32_t slot;
    const int warp = threadIdx.x >> 5;
    if (warp == 0) tmem_alloc(&slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t base = slot + ((uint32_t)((warp & 3) * 32) << 16);
    constexpr int kGroups = NW / 4;  // warps sharing a subpartition split the columns
    constexpr int kPer = kCols / kGroups;
    const int c_begin = (warp >> 2) * kPer;
    float acc[SHAPE == 4 ? 128 : 1];
#pragma unroll
    for (int i = 0; i < (SHAPE == 4 ? 128 : 1); ++i) acc[i] = 0.f;
    float v[SHAPE == 5 ? X : 64];
    const float s = 1.0f + threadIdx.x * 1e-7f;
    __syncthreads();
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
        if constexpr (SHAPE == 4) {
            for (int c0 = c_begin; c0 < c_begin + kPer; c0 += 128) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    tmem_ld32(base + c0 + 32 * q, *reinterpret_cast<float(*)[32]>(v));
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) acc[q * 32 + j] = fmaf(v[j], s, acc[q * 32 + j]);
                }
            }
        } else {
            constexpr int kStep = (SHAPE == 0 || SHAPE == 5) ? X : (SHAPE == 3 ? 32 : 64);
            for (int c = c_begin; c < c_begin + kPer; c += kStep) {
                if constexpr (SHAPE == 0) {
                    if constexpr (X == 16)
                        tmem_ld16(base + c, v);
                    else
                        tmem_ld32(base + c, *reinterpret_cast<float(*)[32]>(v));
                } else if constexpr (SHAPE == 1) {
                    tmem_ld32(base + c, *reinterpret_cast<float(*)[32]>(v));
                    tmem_ld32(base + c + 32, *reinterpret_cast<float(*)[32]>(v + 32));
                } else if constexpr (SHAPE == 2) {
                    tmem_ld16x32bx2_32(base + c, v);
                } else if constexpr (SHAPE == 5) {
                    ld32x32b_x64(base + c, v);
                } else {
                    ld16x256b_x4(base + c, v);
                    ld16x256b_x4(base + (16u << 16) + c, v + 16);
                }
                tmem_wait_ld();
                acc[0] += v[0] + v[kStep == 16 ? 15 : (SHAPE == 5 ? X - 1 : 31)];
            }
        }
    }
    __syncthreads();
    const long long t1 = clock64();
    if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < (SHAPE == 4 ? 128 : 1); ++i) total += acc[i];
    sink[blockIdx.x * blockDim.x + threadIdx.x] = total;
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(slot, kCols);
}

struct Variant {
    int warps, shape, x, lanes;  // lanes of each subpartition read (32, or 16 for SHAPE 2)
    void (*kernel)(int, long long*, float*);
};

const Variant kVariants[] = {
    {4, 0, 16, 32, tmem_ld_kernel<4, 0, 16>},   {4, 0, 32, 32, tmem_ld_kernel<4, 0, 32>},
    {8, 0, 16, 32, tmem_ld_kernel<8, 0, 16>},   {8, 0, 32, 32, tmem_ld_kernel<8, 0, 32>},
    {16, 0, 32, 32, tmem_ld_kernel<16, 0, 32>}, {4, 1, 64, 32, tmem_ld_kernel<4, 1, 64>},
    {8, 1, 64, 32, tmem_ld_kernel<8, 1, 64>},   {4, 2, 64, 16, tmem_ld_kernel<4, 2, 64>},
    {8, 2, 64, 16, tmem_ld_kernel<8, 2, 64>},   {4, 3, 32, 32, tmem_ld_kernel<4, 3, 32>},
    {8, 3, 32, 32, tmem_ld_kernel<8, 3, 32>},   {8, 4, 32, 32, tmem_ld_kernel<8, 4, 32>},
    {4, 5, 64, 32, tmem_ld_kernel<4, 5, 64>},   {8, 5, 64, 32, tmem_ld_kernel<8, 5, 64>},
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);

}  // namespace

extern "C" int tmem_ld_probe_variants(void) { return kNumVariants; }

// Describes variant `v`: warps per CTA, load shape (0..5 as above), columns per load, lanes
// of a subpartition read.  Returns -1 for an unknown variant.
extern "C" int tmem_ld_probe_info(int64_t v, int64_t* out4) {
    if (v < 0 || v >= kNumVariants || out4 == nullptr) return -1;
    out4[0] = kVariants[v].warps;
    out4[1] = kVariants[v].shape;
    out4[2] = kVariants[v].x;
    out4[3] = kVariants[v].lanes;
    return 0;
}

// Launches variant `v` on every SM: cycles (int64 [>= SMs]) gets each CTA's clock64 span,
// sink (fp32 [>= SMs * warps * 32]) the values read (kept live).  Bytes read per SM =
// iters * lanes * 4 subpartitions * 512 columns * 4 B.
AB_ENTRY(tmem_ld_probe, (int64_t v, int64_t iters, aiter_tensor_t* cycles, aiter_tensor_t* sink, void* stream),
         (v, iters, cycles, sink, stream)) {
    AB_CHECK(v >= 0 && v < kNumVariants, "unknown variant ", v);
    AB_CHECK(iters >= 1 && iters <= 1000000, "iters out of range: ", iters);
    ab::need(cycles, "cycles");
    ab::need(sink, "sink");
    ab::need_dtype(cycles, AITER_DTYPE_i64, "cycles");
    ab::need_dtype(sink, AITER_DTYPE_fp32, "sink");
    ab::DeviceGuard g(cycles->device_id);
    int dev = 0, sms = 0;
    AB_CUDA(cudaGetDevice(&dev));
    AB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const Variant& var = kVariants[v];
    AB_CHECK((int64_t)cycles->numel_ >= sms, "cycles needs >= ", sms, " elements");
    AB_CHECK((int64_t)sink->numel_ >= (int64_t)sms * var.warps * 32, "sink needs >= ", sms * var.warps * 32,
             " elements");
    AB_CUDA(cudaFuncSetAttribute(var.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    var.kernel<<<sms, var.warps * 32, kSmemBytes, ab::as_stream(stream)>>>(
        (int)iters, static_cast<long long*>(cycles->ptr), static_cast<float*>(sink->ptr));
    ab::check_launch("tmem_ld_probe");
}
