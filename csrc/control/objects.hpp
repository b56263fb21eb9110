// Daemon-side object model and the interfaces the control plane drives.
//
// The control plane (service.hpp) owns every object's lifetime and validates every request.
// Two pluggable pieces sit below it:
//  * MemoryBackend opens client memory inside the daemon (CUDA IPC for cudaMalloc ranges, a
//    memfd mapping for ugdr host buffers); tests substitute a fake.
//  * Engine executes the work queued on a device's QPs.  One engine per ugdr device: the
//    host-memory CPU engine, and one sm_100a executor per GPU.  Each engine is told about
//    every MR (any QP may name any MR by key), about CQs and QPs of its own device, and about
//    state changes; it keeps whatever device-side mirror it needs.
#pragma once

#include "common/fd.hpp"
#include "common/shm.hpp"
#include "queue/ring.hpp"

#include <array>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace ugdr::control {

enum class DeviceKind : int { cpu = 0, gpu = 1 };

struct DeviceInfo {
    uint64_t identity = 0;
    std::string name;
    DeviceKind kind = DeviceKind::cpu;
    int gpu_ordinal = -1;
};

// ---- memory --------------------------------------------------------------------------------

enum class MemKind : uint8_t { cuda = 1, host = 2, multicast = 3 };

// What a client sends to register memory (decoded from the register-MR opaque).
struct MemoryDescriptor {
    MemKind kind = MemKind::cuda;
    uint64_t client_address = 0;  // start of the registered range in the client
    // cuda: allocation identity
    std::array<uint8_t, 16> uuid{};
    uint64_t allocation_bytes = 0;
    uint64_t allocation_offset = 0;  // registered range start - allocation base
    std::vector<uint8_t> ipc_handle;
    // host: the memfd region holding the range; multicast: the NVLink multicast object (a CUDA
    // POSIX-fd shareable handle), mapped from offset 0 over region_bytes
    uint64_t region_bytes = 0;
    uint64_t region_offset = 0;
    Fd region_fd;
};

struct OpenedMemory {
    void *address = nullptr;  // daemon address of the registered range start
    // The same byte as seen by the executor of each daemon GPU (index = CUDA ordinal; null:
    // unreachable).  A CUDA IPC handle maps an allocation only into the context it is opened
    // in, so device memory is opened once per GPU; pinned host memory has one portable address.
    std::vector<void *> device_address;
    int gpu = -1;             // owning CUDA ordinal, -1 for host memory
    std::vector<void *> bases;  // per-GPU IPC mapping bases to close (device memory)
    void *host_registered = nullptr;  // pinned host region to unregister (host memory)
    SharedMapping host;       // host regions stay mapped while registered
    // NVLink multicast memory: loads through it are multimem reductions over every GPU bound to
    // the object, stores reach every one of them.  The executors use it only as the source and
    // destination of UGDR_X_WR_RDMA_WRITE_SUM_BF16.
    bool multicast = false;
    uint64_t mc_handle = 0;  // imported object
    uint64_t mc_bytes = 0;   // mapped bytes at `address`
};

class MemoryBackend {
  public:
    virtual ~MemoryBackend() = default;
    // Returns 0 or a positive errno (EOPNOTSUPP for memory kinds the backend cannot open).
    virtual int open(MemoryDescriptor &desc, uint64_t length, OpenedMemory *out) = 0;
    virtual void close(OpenedMemory &mem) noexcept = 0;
};

// ---- objects -------------------------------------------------------------------------------

struct Context {
    uint32_t device = 0;  // index into the daemon's device list
    size_t children = 0;  // PDs + CQs
};

struct Pd {
    uint64_t context_id = 0;
    uint32_t pd_num = 0;  // daemon-unique, used for PD checks on the data path
    size_t mrs = 0;
    size_t qps = 0;
};

struct Mr {
    uint64_t pd_id = 0;
    uint32_t pd_num = 0;
    uint32_t device = 0;  // device of the registering context
    uint64_t client_address = 0;
    uint64_t length = 0;
    uint32_t access = 0;
    uint32_t lkey = 0, rkey = 0;
    uint32_t handle = 0;
    uint32_t table_slot = 0;
    OpenedMemory mem;
};

struct Cq {
    uint64_t context_id = 0;
    uint32_t device = 0;
    uint32_t cq_num = 0;
    queue::Ring ring;
    size_t qp_refs = 0;
    void *engine_block = nullptr;  // engine-private control block (e.g. device reservation counters)
};

struct QpCaps {
    uint32_t max_send_wr = 0, max_recv_wr = 0, max_send_sge = 0, max_recv_sge = 0;
};

struct Qp {
    uint64_t pd_id = 0;
    uint32_t pd_num = 0;
    uint32_t device = 0;
    uint32_t qpn = 0;
    uint64_t send_cq_id = 0, recv_cq_id = 0;
    Cq *send_cq = nullptr;
    Cq *recv_cq = nullptr;
    QpCaps caps;
    bool sq_sig_all = false;
    queue::Ring sq, rq;
    // verbs state
    int state = 0;  // ugdr_qp_state
    uint32_t access = 0;
    uint8_t timeout = 0, retry_cnt = 0, rnr_retry = 0, min_rnr_timer = 0;
    Qp *peer = nullptr;   // bound responder (after connect)
    uint32_t peer_qpn = 0;
    bool peer_lost = false;  // the bound responder was destroyed
    void *engine_block = nullptr;  // engine-private per-QP state
};

// ---- engines -------------------------------------------------------------------------------

struct EngineStats {
    uint64_t wrs_completed = 0, bytes_moved = 0, error_completions = 0, launches = 0,
             wait_timeouts = 0, first_start_ns = 0, last_end_ns = 0, chunks_run = 0, claim_misses = 0,
             jobs_published = 0, inline_runs = 0, busy_ns = 0, fast_batches = 0, fast_fetch_ns = 0,
             fast_exec_ns = 0, fast_reserve_ns = 0, fast_publish_ns = 0, slow_wrs = 0, slow_issue_ns = 0,
             job_slot_misses = 0, publish_waits = 0, publish_wait_ns = 0, mr_detach_live = 0,
             mr_detach_quiesced = 0, order_waits = 0, overlap_issues = 0;
};

// Per-QP counters an engine keeps on top of the ring cursors (which the control plane reads
// itself): payload bytes moved by the QP's successful send WRs, its error completions (flushes
// included), and receiver-not-ready waits it entered.
struct QpCounters {
    uint64_t bytes = 0, error_completions = 0, rnr_waits = 0;
};

class Engine {
  public:
    virtual ~Engine() = default;
    virtual DeviceInfo info() const = 0;

    // MR table: every engine sees every MR.  attach may refuse memory it cannot reach only by
    // leaving the entry unusable (the data path then reports an access error).
    virtual int attach_mr(Mr &mr) = 0;
    virtual void detach_mr(Mr &mr) noexcept = 0;
    // CQs and QPs of this engine's device.
    virtual int attach_cq(Cq &cq) = 0;
    virtual void detach_cq(Cq &cq) noexcept = 0;
    virtual int attach_qp(Qp &qp) = 0;
    // The QP's verbs state, peer binding or retry attributes changed.
    virtual void update_qp(Qp &qp) = 0;
    virtual void detach_qp(Qp &qp) noexcept = 0;
    // Stop executing and wait until nothing of this engine touches daemon objects.
    virtual void quiesce() = 0;
    // Allow execution again after quiesce().
    virtual void resume() = 0;
    // True when this engine's detach_qp / detach_cq / update_qp are safe while it runs, for
    // objects that only this engine's own execution may still touch (it keeps their memory
    // until it is not running).  The control plane then stops it only for peers on other engines.
    virtual bool detaches_live() const noexcept { return false; }
    // Forget cached object views: the engine's execution reloads them before using any object
    // again (a CQ slot of another engine may be reused later).  No wait.
    virtual void invalidate_caches() noexcept {}
    // Wait until everything running on this engine has seen the objects' current bindings and
    // retired the WRs issued under the old ones.  False when that did not happen in time (or is
    // not supported): the caller then stops the engine instead.
    virtual bool settle() noexcept { return false; }

    virtual int stats(EngineStats *out, bool reset) = 0;
    // Device trace: keep up to `records_per_unit` events per execution unit from the next launch
    // on (0 turns tracing off and frees the buffer); trace_dump writes what was kept, as Chrome
    // trace-event JSON, to `path`.
    virtual int trace(uint32_t records_per_unit) {
        (void)records_per_unit;
        return EOPNOTSUPP;
    }
    virtual int trace_dump(const std::string &path, uint64_t *kept, uint64_t *dropped) {
        (void)path;
        (void)kept;
        (void)dropped;
        return EOPNOTSUPP;
    }
    virtual int qp_counters(Qp &qp, QpCounters *out) {
        (void)qp;
        (void)out;
        return EOPNOTSUPP;
    }
    virtual int hold(bool on) = 0;
    // Launch (held) executor for a timed drain; complete with finish_drain.
    virtual int start_drain(uint64_t expected_wrs) { (void)expected_wrs; return EOPNOTSUPP; }
    virtual int finish_drain(uint32_t timeout_ms, float *elapsed_ms) {
        (void)timeout_ms;
        (void)elapsed_ms;
        return EOPNOTSUPP;
    }
};

}  // namespace ugdr::control
