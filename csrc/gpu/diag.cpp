// Diagnostic entry points into the executor's copy core, callable through the C ABI (tests
// and benchmarks pass torch tensors' device pointers and a CUDA stream).
#include "gpu/executor.hpp"
#include "ugdr/api.hpp"

#include <cuda_runtime_api.h>

#include <cerrno>
#include <cstring>

namespace {

// Fills `out` for one kernel: resources from cudaFuncGetAttributes, residency from the
// occupancy calculator at the kernel's launch block size.
template <typename Ref> int fill_kernel_attr(const Ref &k, ugdr_x_kernel_attr *out) {
    cudaFuncAttributes a{};
    if (cudaError_t e = cudaFuncGetAttributes(&a, k.fn); e != cudaSuccess) {
        (void)cudaGetLastError();
        return int(e);
    }
    int blocks = 0;
    if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k.fn, k.threads, 0); e != cudaSuccess) {
        (void)cudaGetLastError();
        return int(e);
    }
    std::memset(out, 0, sizeof(*out));
    std::strncpy(out->name, k.name, sizeof(out->name) - 1);
    out->threads_per_block = k.threads;
    out->registers_per_thread = a.numRegs;
    out->local_bytes_per_thread = int(a.localSizeBytes);
    out->static_smem_bytes = int(a.sharedSizeBytes);
    out->max_threads_per_block = a.maxThreadsPerBlock;
    out->blocks_per_sm = blocks;
    return 0;
}

}  // namespace

extern "C" {

int ugdr_x_kernel_attributes(int index, ugdr_x_kernel_attr *out) noexcept {
    const ugdr::gpu::KernelRef *refs = nullptr;
    const int n = ugdr::gpu::executor_kernels(&refs);
    if (out == nullptr || index < 0) return int(cudaErrorInvalidValue);
    if (index == n) return fill_kernel_attr(ugdr::gpu::bulk_copy_kernel_ref(), out);
    if (index > n) return -1;
    return fill_kernel_attr(refs[index], out);
}

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

// The same timing around the TMA bulk-copy kernel (16-byte aligned src, dst and n).  *status
// receives the kernel's status word (0, or 1 when a bounded wait ran out).
int ugdr_x_bulk_copy_bench(void *dst, const void *src, uint64_t n, int ctas, int iters, void *stream,
                           float *ms_per_copy, unsigned int *status) noexcept {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dst == nullptr || src == nullptr) return int(cudaErrorInvalidValue);
    if (ctas <= 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&ctas, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || ctas <= 0)
            return int(cudaErrorInvalidValue);
    }
    unsigned int *st = nullptr;
    if (cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&st), sizeof(unsigned int)); e != cudaSuccess) return int(e);
    cudaMemsetAsync(st, 0, sizeof(unsigned int), s);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    int rc = ugdr::gpu::launch_bulk_copy(dst, src, n, ctas, st, s);  // warm-up
    cudaEventRecord(a, s);
    for (int i = 0; i < iters && rc == 0; ++i) rc = ugdr::gpu::launch_bulk_copy(dst, src, n, ctas, st, s);
    cudaEventRecord(b, s);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    if (ms_per_copy) *ms_per_copy = iters > 0 ? ms / iters : 0.f;
    unsigned int host_status = 0;
    cudaMemcpy(&host_status, st, sizeof(host_status), cudaMemcpyDeviceToHost);
    if (status) *status = host_status;
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFree(st);
    return rc != 0 ? rc : int(cudaGetLastError());
}

}  // extern "C"
