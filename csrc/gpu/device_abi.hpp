// Structures shared by the GPU engine's host code and the sm_100a executor kernel.
//
// Every table lives in device memory of the GPU whose engine owns it and is reachable from the
// other GPUs' executors through peer access (the daemon enables it for every pair), so a
// requester on GPU a can consume the RQ and fill the receive CQ of a responder on GPU b.
// Rings (SQ / RQ / CQ) stay in the memfd mappings clients already share with the daemon; the
// daemon registers them with CUDA as mapped host memory so kernels read WQEs and write CQEs in
// place, with .sys-scope acquire / release on the cursors.
//
// Host writes only `DevQpConfig`, `DevMr` and `DevCqConfig` (by copies on a side stream);
// the `...State` halves belong to the kernel.
#pragma once

#include "queue/layout.hpp"

#include <stdint.h>

namespace ugdr::gpu {

constexpr uint32_t kMaxMrs = 1u << 16;       // key slots (matches the control plane's keys)
constexpr uint32_t kMaxQpsPerEngine = 4096;
constexpr uint32_t kMaxCqsPerEngine = 4096;
constexpr uint32_t kBatch = 32;              // WRs one owner pass issues or retires (one per lane)
constexpr uint32_t kWindow = 64;             // in-flight WRs per QP: two batches
constexpr uint32_t kMaxSge = 32;
constexpr uint32_t kJobSlots = 1024;         // chunked-job slots per engine
constexpr uint32_t kInlineBytes = 4096;      // WRs up to this size are copied by the owner warp

// DevMr::pad bits.
constexpr uint32_t kMrMulticast = 1;  // an NVLink multicast view: multimem loads reduce, stores broadcast

struct DevMr {
    uint64_t base;         // device-usable address of the first registered byte; 0 = unusable
    uint64_t client_base;  // client address of that byte
    uint64_t length;
    uint32_t access;
    uint32_t pd_num;
    uint32_t lkey;
    uint32_t rkey;
    uint32_t valid;
    uint32_t pad;  // flags (kMrMulticast)
};

struct DevCqConfig {
    queue::RingHeader *ring;  // device pointer of the mapped ring
    uint8_t *slots;
    unsigned long long *ready;  // per slot: s + 1 once slot s's CQE is written (device memory)
    uint32_t capacity;
    uint32_t stride;
    uint32_t valid;
    uint32_t pad;
};

struct DevCqState {
    unsigned long long reserve;    // next slot to hand out (CAS, .sys)
    unsigned long long published;  // device mirror of the ring tail: slots below are visible
    unsigned long long head_seen;  // cached consumer cursor
    unsigned long long pad[5];
};

struct DevCq {
    DevCqConfig cfg;
    DevCqState st;
};

struct DevQp;

struct DevQpConfig {
    queue::RingHeader *sq;
    uint8_t *sq_slots;
    queue::RingHeader *rq;
    uint8_t *rq_slots;
    DevCq *send_cq;
    DevCq *recv_cq;
    DevQp *peer;  // responder (may live on another GPU); null when unbound
    uint32_t sq_cap, sq_stride, rq_cap, rq_stride;
    uint32_t qpn, pd_num, access, max_send_sge;
    uint32_t state;  // ugdr_qp_state as set by the control plane
    uint32_t sq_sig_all;
    uint32_t peer_lost;
    uint32_t active;
    uint8_t timeout, retry_cnt, rnr_retry, min_rnr_timer;
    uint32_t pad[3];
};

struct DevSeg {
    uint64_t local;  // device address
    uint64_t length;
};

struct WrRec {
    unsigned long long wr_id;
    unsigned long long remote;  // device address of the remote range start
    unsigned long long total;
    unsigned long long recv_claim;  // RQ cursor claimed for WRITE_WITH_IMM
    unsigned long long recv_wr_id;
    unsigned int chunks_done;
    unsigned int nchunks;
    uint32_t opcode;
    uint32_t status;
    uint32_t signaled;
    uint32_t imm;
    uint32_t nseg;
    uint32_t recv_cqe_done;
    uint32_t pad[2];
    // Device-address extent of the WR's local segments, [lo, hi) (empty when lo == hi): with
    // `remote` and `total` it gives the ranges a later WR of the same QP must not touch while
    // this one may still be moving bytes (see the ordering rule in executor.cu).
    unsigned long long lo, hi;
    DevSeg seg[kMaxSge];
};

struct DevQpState {
    unsigned long long sq_head;   // next WQE to retire (== ring head)
    unsigned long long sq_issue;  // next WQE to issue
    unsigned long long rq_claim;  // RQ WRs handed out (CAS by requesters, .sys)
    unsigned long long rq_released;  // RQ head published in order
    unsigned long long rnr_next_ns;
    uint32_t rnr_attempts;
    uint32_t err;  // executor-detected error: the QP is in ERR
    // A WR that completes in error has been issued but not yet retired: nothing behind it may
    // be issued (RC semantics: every later WR is flushed once it retires).  Owner warp only.
    uint32_t err_issued;
    uint32_t pad0;
    unsigned long long bytes;   // payload bytes of retired successful send WRs (owner warp writes)
    unsigned long long errors;  // error and flush completions of this QP (owner warp writes)
    WrRec win[kWindow];
};

struct DevQp {
    DevQpConfig cfg;
    DevQpState st;
};

// Per QP slot, written by the owner warp at the end of every service pass: the MR epoch the
// pass started with, and the QP's issue and retire cursors after it.  An MR is deregistered
// without stopping the executor once every active QP has begun a pass under the new epoch (no
// later resolution can use the invalidated entry: per-warp MR caches are keyed by epoch) and has
// retired everything issued until then (no in-flight WR still addresses the memory).
// The epoch and the issue cursor share one 8-byte word, written by one store, so the host never
// pairs an epoch with an older cursor and the owner needs no fence between them.
struct QpProgress {
    unsigned long long epoch_issue;  // seen epoch << 32 | issue cursor mod 2^32
    unsigned long long head;         // retire cursor
};

// One chunked job: WRs [first, first + nwr) of one QP's window (indices mod kWindow), cut into
// `chunk_bytes` chunks numbered across the WRs (WR i owns chunks [start[i], start[i + 1])).
// `ctl` = generation (high 32) | next unclaimed chunk (low 32); claims are fetch-and-adds on it.
// `seq` is even while the slot is free and odd while a job owns it; the slot is freed when
// `done` reaches `nchunks`, so no field changes under a worker that holds an unfinished chunk.
struct alignas(64) Job {
    unsigned long long ctl;
    unsigned long long seq;
    WrRec *win;  // 16-byte aligned with the two words after it: read as one vector
    uint32_t nchunks;
    uint32_t chunk_bytes;
    uint32_t first;
    uint32_t nwr;
    uint32_t done;
    uint32_t pad0;
    uint32_t pad1[4];
    uint32_t start[kBatch];
};

struct JobRing {
    unsigned long long tail;       // tickets handed out
    unsigned long long head_hint;  // no unclaimed job below this ticket
    unsigned long long pad[6];
    Job slots[kJobSlots];
};

// Executor status / statistics, in device memory.  The counters (up to `retired`) reset
// together; `qp_slots` is written by the host whenever a QP slot above the current bound is
// activated, so a running kernel starts polling it.
struct DevStats {
    unsigned long long wrs_completed;
    unsigned long long bytes_moved;
    unsigned long long error_completions;
    unsigned long long wait_timeouts;
    unsigned long long first_start_ns;
    unsigned long long last_end_ns;
    unsigned long long chunks_run;      // chunked-job pieces copied
    unsigned long long claim_misses;    // chunk-claim attempts that found nothing to take
    unsigned long long jobs_published;  // WRs split into chunks
    unsigned long long inline_runs;     // WRs copied by their owner warp
    unsigned long long busy_ns;         // summed warp time inside chunk copies
    unsigned long long launches_seen;   // kernel launches (block 0 thread 0)
    // Small-WR fast path, summed per batch: batches, WQE fetch, validate+copy, CQ reserve, publish.
    unsigned long long fast_batches, fast_fetch_ns, fast_exec_ns, fast_reserve_ns, fast_publish_ns;
    // One-per-round issue path and CQ publish waits (see ugdr_x_engine_stats).
    unsigned long long slow_wrs, slow_issue_ns, job_slot_misses, publish_waits, publish_wait_ns;
    unsigned long long order_waits;  // issue passes cut short by the per-QP ordering rule
    unsigned long long overlap_issues;  // issue passes that found earlier WRs of the QP in flight
    unsigned long long last_work_ns;
    unsigned long long retired;  // WRs retired since the last reset (drain mode exit test)
    unsigned int exiting;
    unsigned int error_code;  // first bounded wait that gave up (see ExecError)
    unsigned int qp_slots;
    unsigned int mr_epoch;  // bumped by the host when an MR entry is invalidated (see QpProgress)
    unsigned int pad[12];
};

enum ExecError : uint32_t {
    kErrNone = 0,
    kErrCqPublishTimeout = 1,
    kErrRqReleaseTimeout = 2,
    kErrJobSlotTimeout = 3,
    kErrBulkCopyTimeout = 4,  // a TMA bulk copy of a chunk did not complete in time
};

// Host-mapped control word the host flips while the kernel runs.
struct HostCtrl {
    volatile uint32_t stop;
    uint32_t pad[15];
};

enum ExecMode : uint32_t { kPersistent = 0, kDrain = 1 };

// Optional device trace: one 32-byte record per event, appended by lane 0 of the warp that saw
// it into its CTA's segment of the trace buffer (`trace_cap` records per CTA; later events are
// only counted).  Times are %globaltimer nanoseconds.
enum TraceEvent : uint32_t {
    kTraceFastBatch = 1,  // lane-parallel batch: fetch .. CQ publish; value = WRs
    kTraceRetire = 2,     // in-order retire of staged / chunked WRs; value = WRs retired
    kTraceChunk = 3,      // one chunk copied by a worker warp; value = bytes
    kTraceError = 4,      // a bounded wait ran out; value = error code
    kTraceIssue = 5,      // an issue pass: WQE fetch .. fast-path issue; value = see executor.cu
};

struct TraceRec {
    unsigned long long t0, t1;
    uint32_t event;  // TraceEvent << 16 | global warp index & 0xffff
    uint32_t qp;     // QP slot (0xffffffff when none)
    uint32_t value;
    uint32_t cta;
};

struct ExecParams {
    DevMr *mrs;
    DevQp *qps;
    JobRing *jobs;
    DevStats *stats;
    HostCtrl *ctrl;
    uint32_t mode;
    unsigned long long expected;  // drain: exit once this many WRs retired
    unsigned long long idle_exit_ns;
    unsigned long long max_wait_ns;  // bound on every internal spin
    TraceRec *trace;             // null: tracing off
    unsigned int *trace_count;   // one append counter per CTA
    uint32_t trace_cap;          // records per CTA
    QpProgress *progress;        // one per QP slot
    uint32_t bulk_min;           // chunk pieces of at least this many 16-byte aligned bytes go
                                 // through the TMA bulk-copy engine (0: never)
};

}  // namespace ugdr::gpu
