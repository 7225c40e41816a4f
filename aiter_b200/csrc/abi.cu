// Error bridge and small host utilities of the C ABI
// (csrc/include/aiter_ctypes_error.h:56-67 in the reference).
#include <mutex>
#include <vector>
#include "common.cuh"

namespace ab {

std::string& last_error() {
    static thread_local std::string msg;
    return msg;
}

int num_sms(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) fail("bad device id ", dev);
    if (!cache[dev]) {
        int v = 0;
        AB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
        cache[dev] = v;
    }
    return cache[dev];
}

void set_max_smem_once(const void* kernel, int bytes, int dev) {
    struct Done {
        const void* kernel;
        int bytes, dev;
    };
    static std::mutex mu;
    static std::vector<Done> done;
    std::lock_guard<std::mutex> g(mu);
    // the attribute is an upper bound: keep the largest size set per kernel and device
    for (Done& d : done)
        if (d.kernel == kernel && d.dev == dev) {
            if (bytes > d.bytes) {
                AB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
                d.bytes = bytes;
            }
            return;
        }
    AB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.push_back({kernel, bytes, dev});
}

}  // namespace ab

extern "C" int aiter_ctypes_abi_version(void) { return 2; }

extern "C" const char* aiter_get_last_error(void) {
    const std::string& m = ab::last_error();
    return m.empty() ? nullptr : m.c_str();
}

extern "C" void aiter_clear_last_error(void) { ab::last_error().clear(); }
