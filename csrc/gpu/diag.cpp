// Diagnostic entry points into the executor's copy core, callable through the C ABI (tests
// and benchmarks pass torch tensors' device pointers and a CUDA stream).
#include "gpu/executor.hpp"
#include "ugdr/api.hpp"

#include <cuda_runtime_api.h>

#include <cerrno>

extern "C" {

// One warp copies n bytes (alignment-matrix tests).  Returns a cudaError_t value.
int ugdr_x_copy_core_test(void *dst, const void *src, uint64_t n, void *stream) noexcept {
    return ugdr::gpu::launch_copy_test(dst, src, n, static_cast<cudaStream_t>(stream));
}

// Time `iters` whole-grid copies of n bytes with CUDA events on `stream`; writes the mean
// milliseconds per copy.  Returns a cudaError_t value.
int ugdr_x_grid_copy_bench(void *dst, const void *src, uint64_t n, int ctas, int iters, void *stream,
                           float *ms_per_copy) noexcept {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dst == nullptr || src == nullptr) return int(cudaErrorInvalidValue);
    if (ctas <= 0) {  // one CTA per SM
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&ctas, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || ctas <= 0)
            return int(cudaErrorInvalidValue);
    }
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    int rc = ugdr::gpu::launch_grid_copy(dst, src, n, ctas, s);  // warm-up
    cudaEventRecord(a, s);
    for (int i = 0; i < iters && rc == 0; ++i) rc = ugdr::gpu::launch_grid_copy(dst, src, n, ctas, s);
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    if (ms_per_copy) *ms_per_copy = iters > 0 ? ms / iters : 0.f;
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return rc != 0 ? rc : int(cudaGetLastError());
}

}  // extern "C"
