// Whole-grid local copy through the TMA bulk-copy engine: global -> shared::cta -> global with
// cp.async.bulk (untiled, no tensor map, this CTA's own shared memory only), one issuing thread
// per CTA and a kStages-deep ring of shared-memory buffers tracked by mbarriers.  It is the staged
// counterpart of the executor's load/store copy core (grid_copy_kernel), kept as a diagnostic so
// the two can be timed against each other on the same buffers.
//
// Rules it keeps: every address and size is a multiple of 16 bytes (the host entry checks);
// every mbarrier wait is bounded by a %globaltimer deadline, after which the CTA stores 1 in
// *status, waits (bounded) for its own copies in flight and returns.
#include "gpu/executor.hpp"

#include <cuda_runtime.h>
#include <stdint.h>

namespace ugdr::gpu {
namespace {

constexpr uint32_t kStages = 4;
constexpr uint32_t kBulkChunk = 32768;  // bytes per stage (a multiple of 16)
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// True once the barrier's phase with the given parity has completed; false after the deadline.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    for (uint32_t spins = 0;; ++spins) {
        uint32_t done = 0;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spins & 15) == 15 && now_ns() > deadline) return false;
    }
}

__device__ __forceinline__ void bulk_load(void *smem, const void *gmem, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(smem)),
        "l"(gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_store(void *gmem, const void *smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem), "r"(smem_addr(smem)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// CTA b copies chunks b, b + grid, b + 2 grid, ... of kBulkChunk bytes (the last one shorter).
__global__ void __launch_bounds__(32, 1) bulk_copy_kernel(uint8_t *dst, const uint8_t *src, uint64_t n,
                                                          unsigned int *status) {
    extern __shared__ __align__(128) uint8_t buf[];  // kStages * kBulkChunk
    __shared__ __align__(8) uint64_t bar[kStages];
    if (threadIdx.x != 0) return;
    const uint64_t nchunks = (n + kBulkChunk - 1) / kBulkChunk;
    const uint64_t mine = blockIdx.x < nchunks ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    if (mine == 0) return;
    for (uint32_t s = 0; s < kStages; ++s) mbar_init(&bar[s]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    auto chunk_at = [&](uint64_t i, uint64_t *off) {
        *off = (blockIdx.x + i * gridDim.x) * uint64_t(kBulkChunk);
        const uint64_t left = n - *off;
        return uint32_t(left < kBulkChunk ? left : kBulkChunk);
    };
    auto issue_load = [&](uint64_t i) {
        uint64_t off;
        const uint32_t bytes = chunk_at(i, &off);
        const uint32_t s = uint32_t(i % kStages);
        mbar_expect_tx(&bar[s], bytes);
        bulk_load(buf + size_t(s) * kBulkChunk, src + off, bytes, &bar[s]);
    };
    const uint64_t pro = mine < kStages ? mine : kStages;
    for (uint64_t i = 0; i < pro; ++i) issue_load(i);
    uint64_t loaded = pro;  // loads issued
    bool ok = true;
    uint64_t i = 0;
    for (; i < mine; ++i) {
        const uint32_t s = uint32_t(i % kStages);
        const uint32_t parity = uint32_t((i / kStages) & 1);
        if (!mbar_wait(&bar[s], parity, now_ns() + kWaitNs)) {
            ok = false;
            break;
        }
        uint64_t off;
        const uint32_t bytes = chunk_at(i, &off);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bulk_store(dst + off, buf + size_t(s) * kBulkChunk, bytes);
        if (loaded < mine) {
            // Stage s is reloaded only after the store just issued has read it.
            bulk_wait_read_all();
            issue_load(loaded);
            ++loaded;
        }
    }
    if (!ok) {
        atomicExch(status, 1u);
        // Let every load still in flight (chunks i .. loaded - 1, one per stage) land before the
        // CTA and its shared memory go away.
        for (uint64_t j = i; j < loaded; ++j) {
            const uint32_t s = uint32_t(j % kStages);
            (void)mbar_wait(&bar[s], uint32_t((j / kStages) & 1), now_ns() + kWaitNs);
        }
    }
    bulk_wait_all();
}

}  // namespace

size_t bulk_copy_smem_bytes() { return size_t(kStages) * kBulkChunk; }

KernelRef bulk_copy_kernel_ref() {
    return KernelRef{"bulk_copy_kernel", reinterpret_cast<const void *>(&bulk_copy_kernel), 32};
}

int launch_bulk_copy(void *dst, const void *src, uint64_t n, int ctas, unsigned int *status, cudaStream_t stream) {
    if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | n) & 15u)
        return int(cudaErrorInvalidValue);
    const size_t smem = bulk_copy_smem_bytes();
    if (cudaError_t e = cudaFuncSetAttribute(bulk_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        e != cudaSuccess)
        return int(e);
    bulk_copy_kernel<<<ctas, 32, smem, stream>>>(static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), n,
                                                 status);
    return int(cudaGetLastError());
}

}  // namespace ugdr::gpu
