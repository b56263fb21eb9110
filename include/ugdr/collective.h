/* ugdr collective extensions: allreduce (bf16, fused sum) and MoE all-to-all (fused permutes)
 * over CUDA-IPC mapped peer buffers, plus the IPC export / open helpers that build the peer view.
 * No counterpart in the reference (it has no collectives); they reuse its memory model.
 *
 * All launch functions are asynchronous on `stream` (a cudaStream_t, NULL for the legacy
 * stream) and return a cudaError_t value.  Cross-GPU waits inside the kernels are bounded; when
 * one runs out the kernel stores 1 in *status of the peer set (2 = receive buffer overflow). */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UGDR_X_MAX_RANKS 8
#define UGDR_X_IPC_HANDLE_BYTES 64

/* Layout identical to the kernels' peer set.  signal[q] is rank q's signal buffer (mapped here):
 * UGDR_X_SIGNAL_SLOTS x UGDR_X_MAX_RANKS zero-initialised uint64 words; arrive points at
 * UGDR_X_SIGNAL_SLOTS zero-initialised counters of this rank; status at one word of this rank. */
#define UGDR_X_SIGNAL_SLOTS 8
typedef struct ugdr_x_peerset {
    void *buf[UGDR_X_MAX_RANKS];
    uint64_t *signal[UGDR_X_MAX_RANKS];
    unsigned int *arrive;
    unsigned int *status;
    int n;
    int rank;
} ugdr_x_peerset;

/* Bound (ns) on every cross-GPU wait of the collective kernels launched after the call; 0
 * restores the default (5 s).  Returns the previous bound. */
uint64_t ugdr_x_set_collective_wait_ns(uint64_t ns);

#ifndef UGDR_X_KERNEL_ATTR_DEFINED
#define UGDR_X_KERNEL_ATTR_DEFINED
/* Compiled resources of one kernel on the current CUDA device, with the block size it is
 * launched with and the resident blocks per SM that gives (cudaFuncGetAttributes and the
 * occupancy calculator; static shared memory only). */
typedef struct ugdr_x_kernel_attr {
    char name[48];
    int threads_per_block;
    int registers_per_thread;
    int local_bytes_per_thread; /* spill and stack */
    int static_smem_bytes;
    int max_threads_per_block;
    int blocks_per_sm;
} ugdr_x_kernel_attr;
#endif

/* Kernel `index` of the collective kernels.  Returns 0, -1 past the last kernel, or a
 * cudaError_t value. */
int ugdr_x_collective_kernel_attributes(int index, ugdr_x_kernel_attr *out);

/* Export the allocation holding `ptr` (cudaMalloc memory) for another process: the handle of
 * the allocation base and the offset of `ptr` inside it. */
int ugdr_x_ipc_export(void *ptr, uint8_t handle[UGDR_X_IPC_HANDLE_BYTES], uint64_t *offset);
/* Open an exported allocation in the current device's context; *base receives the mapping. */
int ugdr_x_ipc_open(const uint8_t handle[UGDR_X_IPC_HANDLE_BYTES], void **base);
int ugdr_x_ipc_close(void *base);

/* In-place allreduce of `count` bf16 elements at byte `offset` of every rank's buffer (count a
 * multiple of 8, offset a multiple of 16).  `epoch` increases by one per call on every rank. */
int ugdr_x_allreduce_bf16(const ugdr_x_peerset *ps, uint64_t offset, uint64_t count, uint64_t epoch,
                          int ctas, void *stream);

/* NVLink SHARP (NVLS) multicast memory.  Every rank's GPU binds `bytes` of its own memory to one
 * multicast object; `uc` is this GPU's memory (ordinary access), `mc` the multicast view that
 * only multimem instructions use.  Set-up order across the ranks:
 *   rank 0: ugdr_x_nvls_create (gives a POSIX fd to pass to the others over a Unix socket);
 *   others: ugdr_x_nvls_import(fd);
 *   every rank: ugdr_x_nvls_add_device; then, once every rank has added its GPU, ugdr_x_nvls_bind.
 * Sizes are rounded up to the multicast granularity (h->bytes).  All calls act on the current
 * CUDA device and return 0 or a CUDA error value. */
typedef struct ugdr_x_nvls {
    uint64_t mc_handle;  /* multicast object (driver allocation handle) */
    uint64_t mem_handle; /* this GPU's memory bound to it */
    void *uc;            /* this GPU's memory, unicast mapping */
    void *mc;            /* multicast mapping of the same bytes */
    uint64_t bytes;
    int device;
} ugdr_x_nvls;
int ugdr_x_nvls_supported(int device);
int ugdr_x_nvls_create(int ndev, uint64_t bytes, ugdr_x_nvls *h, int *fd);
int ugdr_x_nvls_import(int fd, int ndev, uint64_t bytes, ugdr_x_nvls *h);
int ugdr_x_nvls_add_device(ugdr_x_nvls *h);
int ugdr_x_nvls_bind(ugdr_x_nvls *h);
int ugdr_x_nvls_release(ugdr_x_nvls *h);

/* In-place allreduce of `count` bf16 elements at byte `offset` of the NVLS memory `h` (count a
 * multiple of 8, offset a multiple of 16): rank r reduces shard r in the switch
 * (multimem.ld_reduce, fp32 accumulation) and stores the sum to every GPU (multimem.st).  `ps`
 * supplies the entry / exit signals (its buffers are not touched). */
int ugdr_x_allreduce_bf16_nvls(const ugdr_x_peerset *ps, const ugdr_x_nvls *h, uint64_t offset, uint64_t count,
                               uint64_t epoch, int ctas, void *stream);

/* MoE routing: rows = tokens * topk expert ids (int32, row r = token r / topk).  Writes the row
 * count of every expert and each row's position inside its expert group, in row order (rows
 * with an id outside [0, nexp) get position -1).  `scratch` holds
 * ugdr_x_moe_route_scratch_bytes(rows, nexp) bytes of device memory. */
size_t ugdr_x_moe_route_scratch_bytes(uint64_t rows, int nexp);
int ugdr_x_moe_route(const int32_t *expert_ids, uint64_t rows, int nexp, int32_t *counts, int32_t *positions,
                     void *scratch, size_t scratch_bytes, void *stream);

/* Layout: exchange every rank's expert counts through the peer buffers (an nranks * nexp int32
 * table at byte `table_offset` of each buffer), then compute group_base[e] for this rank's rows
 * and *recv_used, the rows this rank will receive.  Experts are owned in blocks of
 * experts_per_rank (expert e lives on rank e / experts_per_rank). */
int ugdr_x_moe_layout(const ugdr_x_peerset *ps, const int32_t *counts, int nexp, int experts_per_rank,
                      uint64_t table_offset, int64_t *group_base, int64_t *recv_used, uint64_t epoch,
                      void *stream);

/* Dispatch: row (t, k) of this rank is stored into the receive area of the owner of expert
 * e = expert_ids[t*topk+k] (owner = e / experts_per_rank) at row group_base[e] + positions[r].
 * group_base[e] already includes the rows that lower ranks send to expert e. */
int ugdr_x_moe_dispatch(const ugdr_x_peerset *ps, const void *x, uint64_t row_bytes, const int32_t *expert_ids,
                        const int32_t *positions, const int64_t *group_base, uint64_t tokens, int topk,
                        int experts_per_rank, uint64_t recv_offset, uint64_t recv_rows, uint64_t epoch,
                        int ctas, void *stream);
/* Combine: out[t] = sum_k weights[t*topk+k] * (the owner's row for (t, k)), fp32 accumulation. */
/* out[t] = sum_k weights[t * topk + k] * rows[t * topk + k] over rows already on this GPU
 * ([tokens * topk][row_bytes] bf16 in (token, k) order; fp32 accumulation): the last step of the
 * MoE combine on the verbs, after its READs brought the rows back.  row_bytes a multiple of 16. */
int ugdr_x_moe_weighted_sum(void *out, const void *rows, const float *weights, uint64_t tokens, int topk,
                            uint64_t row_bytes, int ctas, void *stream);
/* The same from rows grouped by expert: row (t, k) is rows[start[ids[t * topk + k]] +
 * pos[t * topk + k]], with ids / pos as ugdr_x_moe_route gives them and start[e] the first row
 * of expert e (all on the device).  The gather is the combine's unpermute. */
int ugdr_x_moe_weighted_sum_grouped(void *out, const void *rows, const int32_t *ids, const int32_t *pos,
                                    const int64_t *start, const float *weights, uint64_t tokens, int topk,
                                    uint64_t row_bytes, int ctas, void *stream);
/* The inverse gather: rows[start[ids[t * topk + k]] + pos[t * topk + k]] = x[t] for every (t, k)
 * (all on the device), so every expert's rows are contiguous: the pack before the MoE dispatch on
 * the verbs (ugdr_x_verbs_moe_dispatch_packed).  Each x row is read once.  row_bytes a multiple
 * of 16. */
int ugdr_x_moe_pack_grouped(void *rows, const void *x, const int32_t *ids, const int32_t *pos, const int64_t *start,
                            uint64_t tokens, int topk, uint64_t row_bytes, int ctas, void *stream);
int ugdr_x_moe_combine(const ugdr_x_peerset *ps, void *out, uint64_t row_bytes, const int32_t *expert_ids,
                       const int32_t *positions, const int64_t *group_base, const float *weights,
                       uint64_t tokens, int topk, int experts_per_rank, uint64_t recv_offset, uint64_t recv_rows,
                       uint64_t epoch, int ctas, void *stream);

#ifdef __cplusplus
}
#endif
