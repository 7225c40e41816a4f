// gemm_a16w16: bf16 y = A @ W^T (tgemm.mm / gemm_a16w16, aiter/tuned_gemm.py:224-308,
// 506-529) on the tcgen05 kernels of gemm_bf16.cuh, plain mode.  The output may be
// the staging buffer of the IPC allreduce (custom_ar_next_buffer), which then
// reduces it without an extra copy.
#include "gemm_bf16.cuh"

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
    AB_CHECK(K % g16::BK == 0 && N % 32 == 0, "need K % 64 == 0 and N % 32 == 0");
    AB_CHECK(out->strides[0] % 8 == 0 && ((uintptr_t)out->ptr & 15) == 0, "out rows must be 16-byte aligned");
    if (M == 0) return;
    DeviceGuard dg(a->device_id);
    g16::run<g16::kPlain>(a, w, (__nv_bfloat16*)out->ptr, out->strides[0], g16::FuseArgs{}, a->device_id,
                          as_stream(stream));
    check_launch("gemm_a16w16");
}

// Error word of the mbarrier waits in this unit's kernels (sm100.cuh keeps one per
// unit); aiter_device_error() folds it in.
namespace ab {
int gemm_bf16_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, sm100::g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(sm100::g_device_error, &z, sizeof(int));
    }
    return v;
}
}  // namespace ab
