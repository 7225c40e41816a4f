// Error bridge and small host utilities of the C ABI
// (csrc/include/aiter_ctypes_error.h:56-67 in the reference).
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

}  // namespace ab

extern "C" int aiter_ctypes_abi_version(void) { return 2; }

extern "C" const char* aiter_get_last_error(void) {
    const std::string& m = ab::last_error();
    return m.empty() ? nullptr : m.c_str();
}

extern "C" void aiter_clear_last_error(void) { ab::last_error().clear(); }
