// ugdr_x_moe_route_noalloc: the MoE routing kernels with their scratch in a fixed device array
// (see include/ugdr/route_noalloc.h for who needs it and its limits).  No counterpart in the reference.
#include "collective/kernels.hpp"
#include "ugdr/route_noalloc.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

namespace {

// Per-block expert histograms / offsets of the counting sort.  In host code this name is only a
// handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) uint32_t g_route_scratch[UGDR_X_ROUTE_NOALLOC_MAX_ENTRIES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t *g_scratch_ptr[kMaxDevices] = {};

// Device address of g_route_scratch on `device` (which is current), looked up once.
cudaError_t scratch_for(int device, uint32_t **out) {
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_scratch_ptr[device] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[device] = static_cast<uint32_t *>(p);
    }
    *out = g_scratch_ptr[device];
    return cudaSuccess;
}

}  // namespace

extern "C" int ugdr_x_moe_route_noalloc(const int32_t *expert_ids, uint64_t rows, int nexp, int32_t *counts,
                                        int32_t *positions, void *stream) {
    if (counts == nullptr || (rows > 0 && (expert_ids == nullptr || positions == nullptr)) || nexp <= 0 ||
        nexp > ugdr::coll::kRouteMaxExperts)
        return int(cudaErrorInvalidValue);
    const size_t need = ugdr::coll::route_scratch_bytes(rows, nexp) / sizeof(uint32_t);
    if (need > UGDR_X_ROUTE_NOALLOC_MAX_ENTRIES) {
        std::fprintf(stderr,
                     "ugdr_x_moe_route_noalloc: %llu rows x %d experts need %zu scratch entries, "
                     "above the fixed %u\n",
                     static_cast<unsigned long long>(rows), nexp, need, UGDR_X_ROUTE_NOALLOC_MAX_ENTRIES);
        return int(cudaErrorInvalidValue);
    }
    int device = 0;
    if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return int(e);
    uint32_t *scratch = nullptr;
    if (cudaError_t e = scratch_for(device, &scratch); e != cudaSuccess) return int(e);
    return ugdr::coll::launch_route(expert_ids, rows, nexp, counts, positions, scratch,
                                    static_cast<cudaStream_t>(stream));
}

extern "C" int ugdr_x_moe_route_noalloc_reset(void) {
    int device = 0;
    if (cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return int(e);
    if (device < 0 || device >= kMaxDevices) return int(cudaErrorInvalidDevice);
    std::lock_guard<std::mutex> lk(g_mu);
    g_scratch_ptr[device] = nullptr;
    return int(cudaSuccess);
}
