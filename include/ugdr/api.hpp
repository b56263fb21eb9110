/* ugdr public C ABI: a libibverbs-shaped device / context / PD / MR / CQ / RC QP interface.
 *
 * Names, field order and numeric values follow the reference API (include/ugdr/api.hpp:13-204
 * of xuOAO/ugdr), which in turn mirrors libibverbs.  This build appends, with their libibverbs
 * values, the operations the reference lists as non-goals: RDMA READ (opcode 4), 8-byte
 * compare-and-swap (5) and fetch-and-add (6), their WC opcodes (2, 3, 4), the remote-read /
 * remote-atomic access bits, and the `wr.atomic` member of the send-WR union.
 *
 * Extensions with no libibverbs counterpart carry a `ugdr_x_` prefix and live at the end of
 * the file: shareable host buffers (so host memory can be registered with the daemon), and
 * engine statistics.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
#define UGDR_NOEXCEPT noexcept
extern "C" {
#else
#define UGDR_NOEXCEPT
#endif

typedef struct ugdr_device ugdr_device;
typedef struct ugdr_context ugdr_context;
typedef struct ugdr_pd ugdr_pd;
typedef struct ugdr_mr ugdr_mr;
typedef struct ugdr_cq ugdr_cq;
typedef struct ugdr_comp_channel ugdr_comp_channel;
typedef struct ugdr_qp ugdr_qp;

typedef struct ugdr_qp_init_attr ugdr_qp_init_attr;
typedef struct ugdr_qp_attr ugdr_qp_attr;
typedef struct ugdr_qp_conn_info ugdr_qp_conn_info;
typedef struct ugdr_sge ugdr_sge;
typedef struct ugdr_send_wr ugdr_send_wr;
typedef struct ugdr_recv_wr ugdr_recv_wr;
typedef struct ugdr_wc ugdr_wc;

typedef enum ugdr_qp_type {
    UGDR_QPT_RC = 2,
} ugdr_qp_type;

typedef enum ugdr_qp_state {
    UGDR_QPS_RESET = 0,
    UGDR_QPS_INIT = 1,
    UGDR_QPS_RTR = 2,
    UGDR_QPS_RTS = 3,
    UGDR_QPS_SQD = 4,
    UGDR_QPS_SQE = 5,
    UGDR_QPS_ERR = 6,
    UGDR_QPS_UNKNOWN = 7,
} ugdr_qp_state;

typedef enum ugdr_qp_attr_mask {
    UGDR_QP_STATE = 1U << 0U,
    UGDR_QP_CUR_STATE = 1U << 1U,
    UGDR_QP_ACCESS_FLAGS = 1U << 3U,
    UGDR_QP_TIMEOUT = 1U << 9U,
    UGDR_QP_RETRY_CNT = 1U << 10U,
    UGDR_QP_RNR_RETRY = 1U << 11U,
    UGDR_QP_MIN_RNR_TIMER = 1U << 15U,
} ugdr_qp_attr_mask;

typedef enum ugdr_wr_opcode {
    UGDR_WR_RDMA_WRITE = 0,
    UGDR_WR_RDMA_WRITE_WITH_IMM = 1,
    UGDR_WR_RDMA_READ = 4,
    UGDR_WR_ATOMIC_CMP_AND_SWP = 5,
    UGDR_WR_ATOMIC_FETCH_AND_ADD = 6,
    /* Extension (no libibverbs counterpart): RDMA WRITE of an elementwise bf16 sum.  The WR's
     * n >= 1 SGEs all have the same even length L; the remote range [remote_addr, +L) receives,
     * element by element, the bf16 (round to nearest even) of the fp32 sum of the n SGEs' bf16
     * elements, added in SGE order.  Every address is 2-byte aligned.  The remote range may be
     * one of the SGEs (in place).  Needs REMOTE_WRITE; completes as UGDR_WC_RDMA_WRITE with
     * byte_len L.  Unequal or odd lengths give UGDR_WC_LOC_LEN_ERR, a misaligned local address
     * UGDR_WC_LOC_PROT_ERR, a misaligned remote address UGDR_WC_REM_INV_REQ_ERR. */
    UGDR_X_WR_RDMA_WRITE_SUM_BF16 = 24,
} ugdr_wr_opcode;

typedef enum ugdr_send_flags {
    UGDR_SEND_SIGNALED = 1U << 1U,
} ugdr_send_flags;

typedef enum ugdr_wc_status {
    UGDR_WC_SUCCESS = 0,
    UGDR_WC_LOC_LEN_ERR = 1,
    UGDR_WC_LOC_QP_OP_ERR = 2,
    UGDR_WC_LOC_PROT_ERR = 4,
    UGDR_WC_WR_FLUSH_ERR = 5,
    UGDR_WC_LOC_ACCESS_ERR = 8,
    UGDR_WC_REM_INV_REQ_ERR = 9,
    UGDR_WC_REM_ACCESS_ERR = 10,
    UGDR_WC_REM_OP_ERR = 11,
    UGDR_WC_RETRY_EXC_ERR = 12,
    UGDR_WC_RNR_RETRY_EXC_ERR = 13,
    UGDR_WC_GENERAL_ERR = 21,
} ugdr_wc_status;

typedef enum ugdr_wc_opcode {
    UGDR_WC_RDMA_WRITE = 1,
    UGDR_WC_RDMA_READ = 2,
    UGDR_WC_COMP_SWAP = 3,
    UGDR_WC_FETCH_ADD = 4,
    UGDR_WC_RECV_RDMA_WITH_IMM = 129,
} ugdr_wc_opcode;

typedef enum ugdr_wc_flags {
    UGDR_WC_WITH_IMM = 1U << 1U,
} ugdr_wc_flags;

typedef enum ugdr_access_flags {
    UGDR_ACCESS_LOCAL_WRITE = 1U << 0U,
    UGDR_ACCESS_REMOTE_WRITE = 1U << 1U,
    UGDR_ACCESS_REMOTE_READ = 1U << 2U,
    UGDR_ACCESS_REMOTE_ATOMIC = 1U << 3U,
} ugdr_access_flags;

struct ugdr_mr {
    ugdr_context *context;
    ugdr_pd *pd;
    void *addr;
    size_t length;
    uint32_t handle;
    uint32_t lkey;
    uint32_t rkey;
};

struct ugdr_sge {
    uint64_t addr;
    uint32_t length;
    uint32_t lkey;
};

struct ugdr_send_wr {
    uint64_t wr_id;
    ugdr_send_wr *next;
    ugdr_sge *sg_list;
    int num_sge;
    ugdr_wr_opcode opcode;
    unsigned int send_flags;
    union {
        uint32_t imm_data;
    };
    union {
        struct {
            uint64_t remote_addr;
            uint32_t rkey;
        } rdma;
        struct {
            uint64_t remote_addr;
            uint64_t compare_add;
            uint64_t swap;
            uint32_t rkey;
        } atomic;
    } wr;
};

struct ugdr_recv_wr {
    uint64_t wr_id;
    ugdr_recv_wr *next;
    ugdr_sge *sg_list;
    int num_sge;
};

struct ugdr_wc {
    uint64_t wr_id;
    ugdr_wc_status status;
    ugdr_wc_opcode opcode;
    uint32_t vendor_err;
    uint32_t byte_len;
    union {
        uint32_t imm_data;
    };
    uint32_t qp_num;
    uint32_t src_qp;
    unsigned int wc_flags;
    uint16_t pkey_index;
    uint16_t slid;
    uint8_t sl;
    uint8_t dlid_path_bits;
};

struct ugdr_qp_init_attr {
    ugdr_cq *send_cq;
    ugdr_cq *recv_cq;
    uint32_t max_send_wr;
    uint32_t max_recv_wr;
    uint32_t max_send_sge;
    uint32_t max_recv_sge;
    ugdr_qp_type qp_type;
    int sq_sig_all;
};

struct ugdr_qp_attr {
    ugdr_qp_state qp_state;
    ugdr_qp_state cur_qp_state;
    int qp_access_flags;
    uint8_t timeout;
    uint8_t retry_cnt;
    uint8_t rnr_retry;
    uint8_t min_rnr_timer;
};

struct ugdr_qp_conn_info {
    uint32_t qp_num;
};

ugdr_device **ugdr_get_device_list(int *num_devices) UGDR_NOEXCEPT;
void ugdr_free_device_list(ugdr_device **list) UGDR_NOEXCEPT;

ugdr_context *ugdr_open_device(ugdr_device *device) UGDR_NOEXCEPT;
int ugdr_close_device(ugdr_context *context) UGDR_NOEXCEPT;

ugdr_pd *ugdr_alloc_pd(ugdr_context *context) UGDR_NOEXCEPT;
int ugdr_dealloc_pd(ugdr_pd *pd) UGDR_NOEXCEPT;

ugdr_mr *ugdr_reg_mr(ugdr_pd *pd, void *address, size_t length, int access) UGDR_NOEXCEPT;
int ugdr_dereg_mr(ugdr_mr *mr) UGDR_NOEXCEPT;

ugdr_cq *ugdr_create_cq(ugdr_context *context, int cqe, void *cq_context,
                        ugdr_comp_channel *channel, int comp_vector) UGDR_NOEXCEPT;
int ugdr_destroy_cq(ugdr_cq *cq) UGDR_NOEXCEPT;
int ugdr_poll_cq(ugdr_cq *cq, int num_entries, ugdr_wc *wc) UGDR_NOEXCEPT;

ugdr_qp *ugdr_create_qp(ugdr_pd *pd, ugdr_qp_init_attr *init_attr) UGDR_NOEXCEPT;
int ugdr_destroy_qp(ugdr_qp *qp) UGDR_NOEXCEPT;
int ugdr_modify_qp(ugdr_qp *qp, ugdr_qp_attr *attr, int attr_mask) UGDR_NOEXCEPT;
int ugdr_query_qp(ugdr_qp *qp, ugdr_qp_attr *attr, int attr_mask,
                  ugdr_qp_init_attr *init_attr) UGDR_NOEXCEPT;

int ugdr_query_qp_conn_info(ugdr_qp *qp, ugdr_qp_conn_info *info) UGDR_NOEXCEPT;
int ugdr_connect_qp(ugdr_qp *qp, const ugdr_qp_conn_info *remote_info, const ugdr_qp_attr *attr,
                    int attr_mask) UGDR_NOEXCEPT;

int ugdr_post_send(ugdr_qp *qp, ugdr_send_wr *wr, ugdr_send_wr **bad_wr) UGDR_NOEXCEPT;
int ugdr_post_recv(ugdr_qp *qp, ugdr_recv_wr *wr, ugdr_recv_wr **bad_wr) UGDR_NOEXCEPT;

/* ---- ugdr extensions (no libibverbs counterpart) ------------------------------------------ */

/* Device attributes.  `kind` is 0 for the host-memory (CPU) engine device and 1 for a GPU
 * engine device; `gpu_ordinal` is the daemon's CUDA ordinal for GPU devices, -1 otherwise. */
typedef struct ugdr_x_device_info {
    char name[32];
    int kind;
    int gpu_ordinal;
    uint64_t identity;
} ugdr_x_device_info;

int ugdr_x_query_device(ugdr_device *device, ugdr_x_device_info *info) UGDR_NOEXCEPT;

/* Host memory that the daemon can reach: a memfd-backed shared mapping.  Only ranges inside
 * such a buffer (or `cudaMalloc` device memory) can be registered with ugdr_reg_mr. */
/* Register an NVLink multicast object (NVLS; see ugdr_x_nvls_* in ugdr/collective.h) as an MR.
 * `mc_fd` is the object's POSIX shareable handle, `address` this process's multicast mapping of
 * it (SGE and remote addresses are given in it) and `length` the bytes registered from offset 0.
 * The daemon maps the object itself.  Reading through such an MR returns the sum over every GPU
 * bound to the object (the NVSwitch reduces), writing stores to every one of them; the
 * executors accept it only as the single SGE and as the remote range of
 * UGDR_X_WR_RDMA_WRITE_SUM_BF16 (16-byte aligned), so one such WR is an allreduce of its range.
 * Every rank's physical memory stays bound while the MR exists: deregister before releasing
 * the object.  GPU contexts only (EOPNOTSUPP elsewhere). */
ugdr_mr *ugdr_x_reg_mr_multicast(ugdr_pd *pd, void *address, size_t length, int access, int mc_fd) UGDR_NOEXCEPT;
void *ugdr_x_alloc_host(size_t length) UGDR_NOEXCEPT;
int ugdr_x_free_host(void *address) UGDR_NOEXCEPT;

/* Per-device engine counters, summed over the device's executor. */
typedef struct ugdr_x_engine_stats {
    uint64_t wrs_completed;
    uint64_t bytes_moved;
    uint64_t error_completions;
    uint64_t launches;
    uint64_t wait_timeouts;
    uint64_t first_start_ns; /* device clock of the first WR picked up since the last reset */
    uint64_t last_end_ns;    /* device clock of the last completion since the last reset */
    uint64_t chunks_run;     /* large-WR pieces copied by the GPU executor */
    uint64_t claim_misses;   /* chunk claims that found no free piece */
    uint64_t jobs_published; /* WRs split across the grid */
    uint64_t inline_runs;    /* WRs copied by their owner warp */
    uint64_t busy_ns;        /* summed warp time spent copying chunks */
    /* small-WR fast path (lane-parallel batches): batch count and summed phase times */
    uint64_t fast_batches, fast_fetch_ns, fast_exec_ns, fast_reserve_ns, fast_publish_ns;
    /* WRs staged one per warp round (multi-SGE, WRITE_WITH_IMM, atomics) and their summed issue
     * time; issue attempts that found no free job slot; CQ publishes that had to wait for their turn
     * behind other producers of the same CQ, and the summed wait */
    uint64_t slow_wrs, slow_issue_ns, job_slot_misses, publish_waits, publish_wait_ns;
    /* MR deregistrations finished while the executor kept running (grace period), and those
     * that had to stop it (not reset by `reset`) */
    uint64_t mr_detach_live, mr_detach_quiesced;
    /* issue passes that stopped before a WR touching bytes an earlier in-flight WR of its QP
     * still moves (the per-QP ordering rule) */
    uint64_t order_waits;
    /* issue passes that found earlier WRs of the QP still in flight (pipelining depth) */
    uint64_t overlap_issues;
} ugdr_x_engine_stats;

int ugdr_x_query_engine_stats(ugdr_context *context, ugdr_x_engine_stats *stats,
                              int reset) UGDR_NOEXCEPT;

/* Hold (hold=1) or release (hold=0) a context's device executor.  While held, posted WRs stay
 * in their rings and the executor is only launched by ugdr_x_timed_drain; the hold persists
 * across drains until released. */
int ugdr_x_engine_hold(ugdr_context *context, int hold) UGDR_NOEXCEPT;

/* Per-QP counters.  The WR counts are the QP's ring cursors since creation: send WRs posted and
 * retired (completed, flushed or silently retired when unsignaled), receive WRs posted and
 * consumed.  `bytes` sums the payload of retired successful send WRs; `error_completions`
 * counts this QP's error and flush completions; `rnr_waits` counts the times a WRITE_WITH_IMM
 * found no receive posted (host engine; 0 on a GPU).  `state` is the current ugdr_qp_state. */
typedef struct ugdr_x_qp_stats {
    uint64_t send_posted, send_retired, recv_posted, recv_consumed;
    uint64_t bytes, error_completions, rnr_waits;
    uint32_t state;
    uint32_t reserved;
} ugdr_x_qp_stats;

int ugdr_x_query_qp_stats(ugdr_qp *qp, ugdr_x_qp_stats *stats) UGDR_NOEXCEPT;

/* The daemon's live objects over all sessions, and its device count. */
typedef struct ugdr_x_daemon_stats {
    uint64_t devices, contexts, pds, mrs, cqs, qps;
} ugdr_x_daemon_stats;

int ugdr_x_query_daemon_stats(ugdr_x_daemon_stats *stats) UGDR_NOEXCEPT;

/* Busy-polls `cq` until at least `min_entries` completions (at most `max_entries`) were taken
 * into `wc`, or `timeout_ns` passed.  Returns the number taken (possibly fewer than min_entries
 * on timeout) or a negative errno, like ugdr_poll_cq. */
int ugdr_x_poll_cq_wait(ugdr_cq *cq, int min_entries, int max_entries, ugdr_wc *wc,
                        uint64_t timeout_ns) UGDR_NOEXCEPT;

/* Device trace of a GPU context's executor.  ugdr_x_engine_trace keeps up to
 * `records_per_cta` events per CTA from the next launch on (0 turns it off): lane-parallel
 * batches, in-order retires, chunk copies and bounded-wait errors, each with %globaltimer start
 * and end.  ugdr_x_engine_trace_dump has the daemon write the events kept since the last dump to
 * `path` (on the daemon's file system) as Chrome trace-event JSON, and returns how many were
 * kept and dropped.  EOPNOTSUPP on the host-memory device. */
int ugdr_x_engine_trace(ugdr_context *context, uint32_t records_per_cta) UGDR_NOEXCEPT;
int ugdr_x_engine_trace_dump(ugdr_context *context, const char *path, uint64_t *kept,
                             uint64_t *dropped) UGDR_NOEXCEPT;

/* Timed drain (benchmarks): the daemon launches the device executors of `num_contexts`
 * contexts together, each bracketed by CUDA events on its launching stream, and returns once
 * every executor has retired `expected_wrs[i]` send WRs or `timeout_ms` passed.  `elapsed_ms[i]`
 * receives the event time of context i.  Returns 0 or a positive errno (ETIMEDOUT). */
int ugdr_x_timed_drain(ugdr_context **contexts, int num_contexts, const uint64_t *expected_wrs,
                       uint32_t timeout_ms, float *elapsed_ms) UGDR_NOEXCEPT;

/* Diagnostics on the current CUDA device (no daemon involved).  ugdr_x_copy_core_test runs the
 * executor's warp copy core once (one warp) over [src, src + n) -> dst, for alignment-matrix
 * tests; ugdr_x_grid_copy_bench times `iters` whole-grid copies with CUDA events on `stream` and
 * writes the mean milliseconds per copy.  Both return a cudaError_t value. */
int ugdr_x_copy_core_test(void *dst, const void *src, uint64_t n, void *stream) UGDR_NOEXCEPT;
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

/* Kernel `index` of the executor translation unit (executor, whole-grid copy, copy-core test).
 * Returns 0, -1 past the last kernel, or a cudaError_t value. */
int ugdr_x_kernel_attributes(int index, ugdr_x_kernel_attr *out) UGDR_NOEXCEPT;

/* The same timing for the TMA bulk-copy kernel (cp.async.bulk global -> shared -> global;
 * src, dst and n multiples of 16).  *status: 0, or 1 if a bounded wait ran out. */
int ugdr_x_bulk_copy_bench(void *dst, const void *src, uint64_t n, int ctas, int iters, void *stream,
                           float *ms_per_copy, unsigned int *status) UGDR_NOEXCEPT;

int ugdr_x_grid_copy_bench(void *dst, const void *src, uint64_t n, int ctas, int iters, void *stream,
                           float *ms_per_copy) UGDR_NOEXCEPT;

#ifdef __cplusplus
}
#endif

#undef UGDR_NOEXCEPT
