// Host entry points of the executor translation unit (executor.cu).
#pragma once

#include "gpu/device_abi.hpp"

#include <cuda_runtime_api.h>
#include <stddef.h>

namespace ugdr::gpu {

// Bytes to allocate for the job ring (ring + its 1024-bit active bitmap).
size_t job_ring_bytes();
int executor_threads();
// Launch the persistent executor; returns a cudaError_t value.
int launch_executor(const ExecParams &p, int ctas, cudaStream_t stream);
// One-warp copy-core test launch (alignment matrix).
int launch_copy_test(void *dst, const void *src, uint64_t n, cudaStream_t stream);
// Whole-grid copy with the executor's copy core (bandwidth ceiling / profiling).
int launch_grid_copy(void *dst, const void *src, uint64_t n, int ctas, cudaStream_t stream);

// Whole-grid copy through the TMA bulk-copy engine (bulk_copy.cu): src, dst and n multiples of
// 16 bytes; *status (device memory) becomes 1 if a bounded wait ran out.
int launch_bulk_copy(void *dst, const void *src, uint64_t n, int ctas, unsigned int *status, cudaStream_t stream);
size_t bulk_copy_smem_bytes();

// The translation unit's kernels with the block size they are launched with (resource reports).
struct KernelRef {
    const char *name;
    const void *fn;
    int threads;
};
int executor_kernels(const KernelRef **out);
KernelRef bulk_copy_kernel_ref();

}  // namespace ugdr::gpu
