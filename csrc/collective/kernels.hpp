// Host launch interface of the collective kernels (kernels.cu).
#pragma once

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

namespace ugdr::coll {

constexpr int kMaxRanks = 8;
constexpr int kRouteRowsPerBlock = 4096;  // fixed, so routing output never depends on the GPU
constexpr int kRouteMaxExperts = 4096;
// Signal slots (each kMaxRanks uint64 words per rank, plus one arrival counter per slot).
constexpr uint32_t kSlotArEnd = 0, kSlotDispatch = 2, kSlotCombine = 3, kSlotCounts = 4, kSlotArEntry = 5;
constexpr uint32_t kSignalSlots = 8;

// One rank's view of a symmetric allocation: every rank's buffer and signal words mapped into
// this process (CUDA IPC), plus this rank's own arrival counters and status word.
struct PeerSet {
    void *buf[kMaxRanks];
    uint64_t *signal[kMaxRanks];  // each rank's signal words: [slot * kMaxRanks + sender]
    unsigned int *arrive;         // this rank's per-slot arrival counters (zero-initialised)
    unsigned int *status;         // this rank's status word: 0 ok, 1 peer wait ran out, 2 overflow
    int n;
    int rank;
};

int grid_for(int device);

// The collective kernels with the block size they are launched with (resource reports).
struct KernelRef {
    const char *name;
    const void *fn;
    int threads;
};
int collective_kernels(const KernelRef **out);
int launch_allreduce_bf16(const PeerSet &ps, uint64_t offset, uint64_t count, uint64_t epoch, int ctas,
                          uint64_t max_ns, cudaStream_t s);
int launch_allreduce_bf16_nvls(const PeerSet &ps, void *mc, uint64_t offset, uint64_t count, uint64_t epoch,
                               int ctas, uint64_t max_ns, cudaStream_t s);
size_t route_scratch_bytes(uint64_t rows, int nexp);
int launch_route(const int32_t *idx, uint64_t rows, int nexp, int32_t *counts, int32_t *pos, uint32_t *scratch,
                 cudaStream_t s);
int launch_layout(const PeerSet &ps, const int32_t *counts, int nexp, int exp_per_rank, uint64_t table_off,
                  int64_t *gbase, int64_t *recv_used, uint64_t epoch, uint64_t max_ns, cudaStream_t s);
int launch_dispatch(const PeerSet &ps, const void *x, uint64_t row_bytes, const int32_t *idx, const int32_t *pos,
                    const int64_t *gbase, uint64_t ntok, int topk, int exp_per_rank, uint64_t recv_off,
                    uint64_t recv_rows, uint64_t epoch, int ctas, uint64_t max_ns, cudaStream_t s);
int launch_weighted_rows(void *out, const void *rows, const float *w, uint64_t ntok, int topk, uint64_t row_bytes,
                         int ctas, cudaStream_t s, const int32_t *ids = nullptr, const int32_t *pos = nullptr,
                         const int64_t *start = nullptr);
// rows[start[ids[t, k]] + pos[t, k]] = x[t] for every (t, k): x's rows grouped by expert.
int launch_pack_rows(void *rows, const void *x, uint64_t ntok, int topk, uint64_t row_bytes, const int32_t *ids,
                     const int32_t *pos, const int64_t *start, int ctas, cudaStream_t s);
int launch_combine(const PeerSet &ps, void *out, uint64_t row_bytes, const int32_t *idx, const int32_t *pos,
                   const int64_t *gbase, const float *w, uint64_t ntok, int topk, int exp_per_rank,
                   uint64_t recv_off, uint64_t recv_rows, uint64_t epoch, int ctas, uint64_t max_ns,
                   cudaStream_t s);

}  // namespace ugdr::coll
