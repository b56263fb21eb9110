// C ABI of the collective kernels and the IPC helpers that build a peer set.
#include "collective/kernels.hpp"
#include "ugdr/collective.h"

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <atomic>
#include <cstring>

namespace {

static_assert(sizeof(ugdr_x_peerset) == sizeof(ugdr::coll::PeerSet), "peer set layout");
// Bound on every cross-GPU wait inside the collective kernels (ugdr_x_set_collective_wait_ns).
std::atomic<uint64_t> g_wait_ns{5ull * 1000 * 1000 * 1000};

const ugdr::coll::PeerSet &as_ps(const ugdr_x_peerset *p) {
    return *reinterpret_cast<const ugdr::coll::PeerSet *>(p);
}

int default_ctas() {
    int dev = 0;
    cudaGetDevice(&dev);
    return ugdr::coll::grid_for(dev);
}

using GetRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

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

int ugdr_x_collective_kernel_attributes(int index, ugdr_x_kernel_attr *out) {
    const ugdr::coll::KernelRef *refs = nullptr;
    const int n = ugdr::coll::collective_kernels(&refs);
    if (out == nullptr || index < 0) return int(cudaErrorInvalidValue);
    if (index >= n) return -1;
    return fill_kernel_attr(refs[index], out);
}

uint64_t ugdr_x_set_collective_wait_ns(uint64_t ns) {
    return g_wait_ns.exchange(ns == 0 ? 5ull * 1000 * 1000 * 1000 : ns);
}

int ugdr_x_ipc_export(void *ptr, uint8_t handle[UGDR_X_IPC_HANDLE_BYTES], uint64_t *offset) {
    static GetRangeFn range = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return GetRangeFn(nullptr);
        return reinterpret_cast<GetRangeFn>(p);
    }();
    if (ptr == nullptr || handle == nullptr || offset == nullptr || range == nullptr)
        return int(cudaErrorInvalidValue);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, CUdeviceptr(reinterpret_cast<uintptr_t>(ptr))) != CUDA_SUCCESS)
        return int(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h{};
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return int(e);
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<uintptr_t>(ptr) - base;
    return 0;
}

int ugdr_x_ipc_open(const uint8_t handle[UGDR_X_IPC_HANDLE_BYTES], void **base) {
    if (handle == nullptr || base == nullptr) return int(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return int(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
}

int ugdr_x_ipc_close(void *base) { return int(cudaIpcCloseMemHandle(base)); }

int ugdr_x_allreduce_bf16(const ugdr_x_peerset *ps, uint64_t offset, uint64_t count, uint64_t epoch, int ctas,
                          void *stream) {
    if (ps == nullptr || ps->n < 1 || ps->n > UGDR_X_MAX_RANKS) return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_allreduce_bf16(as_ps(ps), offset, count, epoch, ctas > 0 ? ctas : default_ctas(),
                                             g_wait_ns.load(std::memory_order_relaxed), static_cast<cudaStream_t>(stream));
}

int ugdr_x_allreduce_bf16_nvls(const ugdr_x_peerset *ps, const ugdr_x_nvls *h, uint64_t offset, uint64_t count,
                               uint64_t epoch, int ctas, void *stream) {
    if (ps == nullptr || h == nullptr || ps->n < 1 || ps->n > UGDR_X_MAX_RANKS || h->mc == nullptr ||
        offset + count * 2 > h->bytes)
        return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_allreduce_bf16_nvls(as_ps(ps), h->mc, offset, count, epoch,
                                                  ctas > 0 ? ctas : default_ctas(), g_wait_ns.load(std::memory_order_relaxed),
                                                  static_cast<cudaStream_t>(stream));
}

size_t ugdr_x_moe_route_scratch_bytes(uint64_t rows, int nexp) {
    return ugdr::coll::route_scratch_bytes(rows, nexp);
}

int ugdr_x_moe_route(const int32_t *expert_ids, uint64_t rows, int nexp, int32_t *counts, int32_t *positions,
                     void *scratch, size_t scratch_bytes, void *stream) {
    if (counts == nullptr || (rows > 0 && (expert_ids == nullptr || positions == nullptr)))
        return int(cudaErrorInvalidValue);
    if (scratch_bytes < ugdr::coll::route_scratch_bytes(rows, nexp) || (scratch == nullptr && rows > 0))
        return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_route(expert_ids, rows, nexp, counts, positions, static_cast<uint32_t *>(scratch),
                                    static_cast<cudaStream_t>(stream));
}

int ugdr_x_moe_layout(const ugdr_x_peerset *ps, const int32_t *counts, int nexp, int experts_per_rank,
                      uint64_t table_offset, int64_t *group_base, int64_t *recv_used, uint64_t epoch,
                      void *stream) {
    if (ps == nullptr || nexp <= 0 || experts_per_rank <= 0 || table_offset % 4 != 0)
        return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_layout(as_ps(ps), counts, nexp, experts_per_rank, table_offset, group_base,
                                     recv_used, epoch, g_wait_ns.load(std::memory_order_relaxed), static_cast<cudaStream_t>(stream));
}

int ugdr_x_moe_dispatch(const ugdr_x_peerset *ps, const void *x, uint64_t row_bytes, const int32_t *expert_ids,
                        const int32_t *positions, const int64_t *group_base, uint64_t tokens, int topk,
                        int experts_per_rank, uint64_t recv_offset, uint64_t recv_rows, uint64_t epoch, int ctas,
                        void *stream) {
    if (ps == nullptr || topk <= 0 || experts_per_rank <= 0) return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_dispatch(as_ps(ps), x, row_bytes, expert_ids, positions, group_base, tokens, topk,
                                       experts_per_rank, recv_offset, recv_rows, epoch,
                                       ctas > 0 ? ctas : default_ctas(), g_wait_ns.load(std::memory_order_relaxed),
                                       static_cast<cudaStream_t>(stream));
}

int ugdr_x_moe_combine(const ugdr_x_peerset *ps, void *out, uint64_t row_bytes, const int32_t *expert_ids,
                       const int32_t *positions, const int64_t *group_base, const float *weights, uint64_t tokens,
                       int topk, int experts_per_rank, uint64_t recv_offset, uint64_t recv_rows, uint64_t epoch,
                       int ctas, void *stream) {
    if (ps == nullptr || topk <= 0 || experts_per_rank <= 0) return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_combine(as_ps(ps), out, row_bytes, expert_ids, positions, group_base, weights,
                                      tokens, topk, experts_per_rank, recv_offset, recv_rows, epoch,
                                      ctas > 0 ? ctas : default_ctas(), g_wait_ns.load(std::memory_order_relaxed),
                                      static_cast<cudaStream_t>(stream));
}

int ugdr_x_moe_weighted_sum(void *out, const void *rows, const float *weights, uint64_t tokens, int topk,
                            uint64_t row_bytes, int ctas, void *stream) {
    if (out == nullptr || rows == nullptr || weights == nullptr) return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_weighted_rows(out, rows, weights, tokens, topk, row_bytes,
                                            ctas > 0 ? ctas : default_ctas(), static_cast<cudaStream_t>(stream));
}

int ugdr_x_moe_weighted_sum_grouped(void *out, const void *rows, const int32_t *ids, const int32_t *pos,
                                    const int64_t *start, const float *weights, uint64_t tokens, int topk,
                                    uint64_t row_bytes, int ctas, void *stream) {
    if (out == nullptr || rows == nullptr || weights == nullptr || ids == nullptr || pos == nullptr || start == nullptr)
        return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_weighted_rows(out, rows, weights, tokens, topk, row_bytes,
                                            ctas > 0 ? ctas : default_ctas(), static_cast<cudaStream_t>(stream), ids,
                                            pos, start);
}

int ugdr_x_moe_pack_grouped(void *rows, const void *x, const int32_t *ids, const int32_t *pos, const int64_t *start,
                            uint64_t tokens, int topk, uint64_t row_bytes, int ctas, void *stream) {
    if (rows == nullptr || x == nullptr || ids == nullptr || pos == nullptr || start == nullptr)
        return int(cudaErrorInvalidValue);
    return ugdr::coll::launch_pack_rows(rows, x, tokens, topk, row_bytes, ids, pos, start,
                                        ctas > 0 ? ctas : default_ctas(), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
