// Shared host/device helpers for the aiter_b200 C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include <sstream>
#include <stdexcept>
#include <string>

#include "../../include/aiter_b200.h"

namespace ab {

// ----------------------------------------------------------------- error bridge
// Status + thread-local message, the convention of the reference's ctypes ABI
// (csrc/include/aiter_ctypes_error.h:56-130): the entry returns 0 or -1 and the
// message is read with aiter_get_last_error().
std::string& last_error();

template <typename... Args>
[[noreturn]] inline void fail(Args&&... args) {
    std::ostringstream os;
    (os << ... << args);
    throw std::runtime_error(os.str());
}

#define AB_CHECK(cond, ...)                                                      \
    do {                                                                         \
        if (!(cond)) ::ab::fail(__func__, ": ", __VA_ARGS__);                    \
    } while (0)

#define AB_CUDA(call)                                                            \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess)                                                   \
            ::ab::fail(__func__, ": ", #call, " -> ", cudaGetErrorString(e_));   \
    } while (0)

template <typename F>
inline int safe_call(F&& f) {
    last_error().clear();
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        last_error() = e.what();
        return -1;
    } catch (...) {
        last_error() = "unknown C++ exception";
        return -1;
    }
}

// Defines `extern "C" int name DECL` that runs `name_impl CALL` under safe_call.
#define AB_ENTRY(name, DECL, CALL)                                               \
    static void name##_impl DECL;                                                \
    extern "C" int name DECL {                                                   \
        return ::ab::safe_call([&]() { name##_impl CALL; });                     \
    }                                                                            \
    static void name##_impl DECL

inline void check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) fail(what, ": kernel launch failed: ", cudaGetErrorString(e));
}

// Selects the tensor's device for the scope of an entry point.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        AB_CUDA(cudaGetDevice(&prev));
        if (dev >= 0 && dev != prev) AB_CUDA(cudaSetDevice(dev));
        else prev = -1;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// ----------------------------------------------------------------- tensors
inline size_t elem_size(int dt) {
    switch (dt) {
        case AITER_DTYPE_fp8: case AITER_DTYPE_fp8_e8m0: case AITER_DTYPE_i4x2:
        case AITER_DTYPE_fp4x2: case AITER_DTYPE_i8: case AITER_DTYPE_u8: return 1;
        case AITER_DTYPE_fp16: case AITER_DTYPE_bf16: case AITER_DTYPE_i16: return 2;
        case AITER_DTYPE_fp32: case AITER_DTYPE_u32: case AITER_DTYPE_i32: return 4;
        case AITER_DTYPE_i64: case AITER_DTYPE_u64: return 8;
        default: return 0;
    }
}

inline const char* dtype_name(int dt) {
    static const char* n[] = {"fp8", "fp8_e8m0", "fp16", "bf16", "fp32", "i4x2", "fp4x2",
                              "u32", "i32", "i16", "i8", "u8", "i64", "u64"};
    return (dt >= 0 && dt < 14) ? n[dt] : "unknown";
}

inline bool is_contiguous(const aiter_tensor_t* t) {
    if (t->numel_ == 0) return true;
    int64_t expect = 1;
    for (int d = t->ndim - 1; d >= 0; --d) {
        if (t->shape[d] != 1 && t->strides[d] != expect) return false;
        expect *= t->shape[d];
    }
    return true;
}

inline const aiter_tensor_t* need(const aiter_tensor_t* t, const char* name) {
    if (!t) fail(name, " must not be None");
    if (t->numel_ > 0 && !t->ptr) fail(name, " has a null data pointer");
    return t;
}

inline void need_dtype(const aiter_tensor_t* t, int dt, const char* name) {
    if (t->dtype_ != dt)
        fail(name, " must be ", dtype_name(dt), ", got ", dtype_name(t->dtype_));
}

inline void need_contig(const aiter_tensor_t* t, const char* name) {
    if (!is_contiguous(t)) fail(name, " must be contiguous");
}

inline void need_ndim(const aiter_tensor_t* t, int nd, const char* name) {
    if (t->ndim != nd) fail(name, " must have ", nd, " dims, got ", t->ndim);
}

inline int64_t rows_of(const aiter_tensor_t* t) {
    int64_t r = 1;
    for (int d = 0; d + 1 < t->ndim; ++d) r *= t->shape[d];
    return r;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms(int dev);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) costs a driver call; entry points
// call this instead, which raises the limit only when a launch needs more than any
// earlier one on that device.
void set_max_smem_once(const void* kernel, int bytes, int dev);

// Error word of the mbarrier waits in the bf16 GEMM unit (0 = none, -1 = read failed).
int gemm_bf16_device_error(int clear);

}  // namespace ab

// ----------------------------------------------------------------- device side
namespace abd {

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

// Nanosecond global timer, used to bound every device-side wait.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace abd
