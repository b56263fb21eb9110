#include "gpu/gpu_engine.hpp"
#include "gpu/cuda_memory.hpp"

#include "control/service.hpp"
#include "gpu/device_abi.hpp"
#include "gpu/executor.hpp"
#include "gpu/trace_writer.hpp"
#include "gpu/visibility.hpp"
#include "common/trace.hpp"
#include "ugdr/api.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

namespace ugdr::gpu {
namespace {

using Clock = std::chrono::steady_clock;

// Register a daemon ring mapping with CUDA (portable, mapped); returns the device pointer.
void *register_ring(queue::Ring &ring) {
    if (cudaHostRegister(ring.mapping(), ring.bytes(),
                         cudaHostRegisterMapped | cudaHostRegisterPortable) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    void *dev = nullptr;
    if (cudaHostGetDevicePointer(&dev, ring.mapping(), 0) != cudaSuccess) {
        (void)cudaGetLastError();
        cudaHostUnregister(ring.mapping());
        return nullptr;
    }
    return dev;
}

class GpuEngine final : public control::Engine {
  public:
    GpuEngine(const GpuEngineConfig &cfg) : cfg_(cfg) {}
    ~GpuEngine() override;

    int init();

    control::DeviceInfo info() const override {
        control::DeviceInfo d;
        d.name = "ugdr_gpu" + std::to_string(cfg_.ordinal);
        d.kind = control::DeviceKind::gpu;
        d.gpu_ordinal = cfg_.ordinal;
        return d;
    }
    int attach_mr(control::Mr &mr) override;
    void detach_mr(control::Mr &mr) noexcept override;
    int attach_cq(control::Cq &cq) override;
    void detach_cq(control::Cq &cq) noexcept override;
    int attach_qp(control::Qp &qp) override;
    void update_qp(control::Qp &qp) override;
    void detach_qp(control::Qp &qp) noexcept override;
    void quiesce() override;
    bool detaches_live() const noexcept override { return true; }
    void invalidate_caches() noexcept override;
    bool settle() noexcept override;
    void resume() override;
    int stats(control::EngineStats *out, bool reset) override;
    int qp_counters(control::Qp &qp, control::QpCounters *out) override;
    int trace(uint32_t records_per_unit) override;
    int trace_dump(const std::string &path, uint64_t *kept, uint64_t *dropped) override;
    int hold(bool on) override;
    int start_drain(uint64_t expected) override;
    int finish_drain(uint32_t timeout_ms, float *elapsed_ms) override;

  private:
    struct QpEntry {
        control::Qp *qp = nullptr;
        uint32_t slot = 0;
        void *sq_dev = nullptr, *rq_dev = nullptr;
        bool error = false;
    };

    void set_device() const { cudaSetDevice(cfg_.ordinal); }
    int copy_to_device(void *dst, const void *src, size_t n);
    int copy_from_device(void *dst, const void *src, size_t n);
    bool has_work_locked();
    int launch_locked(uint32_t mode, uint64_t expected, bool timed);
    // Ask a running kernel to exit and wait (bounded); returns false if it did not stop.
    bool stop_kernel_locked(uint32_t timeout_ms);
    bool kernel_done_locked();
    // True while some chunked copy still has pieces nobody has claimed (job bitmap non-zero).
    // A stopped kernel has finished every piece it claimed, so with the bitmap clear no copy
    // into any MR is left half done.
    bool copies_pending_locked();
    bool mr_grace_locked();
    void monitor();
    void fill_qp_config(control::Qp &qp, DevQpConfig *cfg);

    GpuEngineConfig cfg_;
    std::mutex mu_;
    cudaStream_t exec_stream_ = nullptr, ctl_stream_ = nullptr;
    cudaEvent_t ev_start_ = nullptr, ev_done_ = nullptr;
    DevMr *mrs_ = nullptr;
    DevQp *qps_ = nullptr;
    QpProgress *progress_ = nullptr;  // per QP slot, written by the owner warps
    // Pinned staging for the control copies: copies between device memory and pageable host
    // memory were slow while the executor ran (an MR registration took 5-19 ms, 3 ms through
    // this buffer), so every control copy goes through it.
    static constexpr size_t kStageBytes = 128 << 10;
    uint8_t *stage_ = nullptr;
    std::mutex stage_mu_;
    uint32_t mr_epoch_ = 0;           // last value stored in DevStats::mr_epoch
    uint64_t mr_fast_detaches_ = 0, mr_slow_detaches_ = 0;
    DevCq *cqs_ = nullptr;
    JobRing *jobs_ = nullptr;
    DevStats *stats_ = nullptr;
    HostCtrl *ctrl_ = nullptr;  // mapped pinned host memory
    HostCtrl *ctrl_dev_ = nullptr;
    std::vector<uint32_t> free_qp_slots_, free_cq_slots_;
    std::vector<unsigned long long *> cq_ready_ = std::vector<unsigned long long *>(kMaxCqsPerEngine, nullptr);
    uint32_t next_qp_slot_ = 0, next_cq_slot_ = 0, qp_slot_bound_ = 0;
    std::vector<QpEntry> qps_host_;
    bool running_ = false;
    bool held_ = false;
    int paused_ = 0;
    // Set when quiesce() could not stop the executor: host memory it may still read stays
    // registered (leaked) instead of being unregistered under a running kernel.
    bool wedged_ = false;
    TraceRec *trace_ = nullptr;          // device trace buffer (ctas x trace_cap_ records)
    unsigned int *trace_count_ = nullptr;
    uint32_t trace_cap_ = 0;
    std::vector<queue::Ring> graveyard_;  // rings of objects destroyed while wedged (kept mapped)
    // Destroyed while the executor ran: a warp's cached view may still reach the rings, the CQ
    // `ready` arrays and the slots, so they are released (and the slots reused) only while no
    // executor runs and no chunk job is pending (reap_locked).  cudaHostUnregister and cudaFree
    // would also wait for the persistent kernel.
    std::vector<queue::Ring> deferred_rings_;
    std::vector<unsigned long long *> deferred_ready_;
    std::vector<uint32_t> cooling_qp_slots_, cooling_cq_slots_;
    void reap_locked();
    // All slots in use and some cooling: stop the executor once so that they can be reused.
    void reclaim_slots(bool qp);
    uint64_t launches_ = 0;
    std::atomic<bool> stop_monitor_{false};
    std::thread monitor_;
    CudaVisibilitySource vis_src_;
    VisibilityGate vis_{vis_src_};
};

GpuEngine::~GpuEngine() {
    stop_monitor_.store(true);
    if (monitor_.joinable()) monitor_.join();
    std::lock_guard<std::mutex> lk(mu_);
    set_device();
    stop_kernel_locked(5000);
    for (queue::Ring &r : deferred_rings_) cudaHostUnregister(r.mapping());
    deferred_rings_.clear();
    for (unsigned long long *p : deferred_ready_)
        if (p) cudaFree(p);
    deferred_ready_.clear();
    if (exec_stream_) cudaStreamDestroy(exec_stream_);
    if (ctl_stream_) cudaStreamDestroy(ctl_stream_);
    if (ev_start_) cudaEventDestroy(ev_start_);
    if (ev_done_) cudaEventDestroy(ev_done_);
    cudaFree(mrs_);
    cudaFree(qps_);
    cudaFree(cqs_);
    for (unsigned long long *r : cq_ready_)
        if (r) cudaFree(r);
    cudaFree(jobs_);
    cudaFree(stats_);
    cudaFree(trace_);
    cudaFree(trace_count_);
    if (ctrl_) cudaFreeHost(ctrl_);
    if (stage_) cudaFreeHost(stage_);
}

int GpuEngine::init() {
    set_device();
    auto ok = [](cudaError_t e) { return e == cudaSuccess; };
    if (!ok(cudaStreamCreateWithFlags(&exec_stream_, cudaStreamNonBlocking)) ||
        !ok(cudaStreamCreateWithFlags(&ctl_stream_, cudaStreamNonBlocking)) ||
        !ok(cudaEventCreate(&ev_start_)) || !ok(cudaEventCreate(&ev_done_)) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&mrs_), sizeof(DevMr) * kMaxMrs)) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&qps_), sizeof(DevQp) * kMaxQpsPerEngine)) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&progress_), sizeof(QpProgress) * kMaxQpsPerEngine)) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&cqs_), sizeof(DevCq) * kMaxCqsPerEngine)) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&jobs_), job_ring_bytes())) ||
        !ok(cudaMalloc(reinterpret_cast<void **>(&stats_), sizeof(DevStats))) ||
        !ok(cudaHostAlloc(reinterpret_cast<void **>(&ctrl_), sizeof(HostCtrl), cudaHostAllocMapped | cudaHostAllocPortable)) ||
        !ok(cudaHostAlloc(reinterpret_cast<void **>(&stage_), kStageBytes, cudaHostAllocPortable)) ||
        !ok(cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctrl_dev_), ctrl_, 0))) {
        (void)cudaGetLastError();
        return ENODEV;
    }
    std::memset(ctrl_, 0, sizeof(HostCtrl));
    cudaMemsetAsync(mrs_, 0, sizeof(DevMr) * kMaxMrs, ctl_stream_);
    cudaMemsetAsync(qps_, 0, sizeof(DevQp) * kMaxQpsPerEngine, ctl_stream_);
    cudaMemsetAsync(progress_, 0, sizeof(QpProgress) * kMaxQpsPerEngine, ctl_stream_);
    cudaMemsetAsync(cqs_, 0, sizeof(DevCq) * kMaxCqsPerEngine, ctl_stream_);
    cudaMemsetAsync(jobs_, 0, job_ring_bytes(), ctl_stream_);
    cudaMemsetAsync(stats_, 0, sizeof(DevStats), ctl_stream_);
    if (!ok(cudaStreamSynchronize(ctl_stream_))) return ENODEV;
    // Third-party (GPUDirect RDMA) writes into this GPU's MRs are visible to the executor in
    // order only with owner ordering; otherwise every launch is preceded by a host flush.
    vis_.init(cfg_.ordinal);
    monitor_ = std::thread([this] { monitor(); });
    return 0;
}

int GpuEngine::copy_to_device(void *dst, const void *src, size_t n) {
    set_device();
    std::lock_guard<std::mutex> lk(stage_mu_);
    for (size_t o = 0; o < n; o += kStageBytes) {
        const size_t k = n - o < kStageBytes ? n - o : kStageBytes;
        std::memcpy(stage_, static_cast<const uint8_t *>(src) + o, k);
        if (cudaMemcpyAsync(static_cast<uint8_t *>(dst) + o, stage_, k, cudaMemcpyHostToDevice, ctl_stream_) !=
                cudaSuccess ||
            cudaStreamSynchronize(ctl_stream_) != cudaSuccess) {
            (void)cudaGetLastError();
            return EIO;
        }
    }
    return 0;
}

int GpuEngine::copy_from_device(void *dst, const void *src, size_t n) {
    set_device();
    std::lock_guard<std::mutex> lk(stage_mu_);
    for (size_t o = 0; o < n; o += kStageBytes) {
        const size_t k = n - o < kStageBytes ? n - o : kStageBytes;
        if (cudaMemcpyAsync(stage_, static_cast<const uint8_t *>(src) + o, k, cudaMemcpyDeviceToHost, ctl_stream_) !=
                cudaSuccess ||
            cudaStreamSynchronize(ctl_stream_) != cudaSuccess) {
            (void)cudaGetLastError();
            return EIO;
        }
        std::memcpy(static_cast<uint8_t *>(dst) + o, stage_, k);
    }
    return 0;
}

// ---- MRs --------------------------------------------------------------------------------------

int GpuEngine::attach_mr(control::Mr &mr) {
    DevMr d{};
    const auto &addr = mr.mem.device_address;
    d.base = size_t(cfg_.ordinal) < addr.size() ? reinterpret_cast<uint64_t>(addr[cfg_.ordinal]) : 0;
    d.client_base = mr.client_address;
    d.length = mr.length;
    d.access = mr.access;
    d.pd_num = mr.pd_num;
    d.lkey = mr.lkey;
    d.rkey = mr.rkey;
    d.valid = 1;
    d.pad = mr.mem.multicast ? kMrMulticast : 0u;
    return copy_to_device(&mrs_[mr.table_slot], &d, sizeof(d));
}

void GpuEngine::detach_mr(control::Mr &mr) noexcept {
    // Clear the entry's `valid` word first (one aligned 4-byte store, so a running warp sees
    // either the whole old entry or an invalid one): from then on no WR resolves against it.
    // Then, without stopping the executor, wait for a grace period (mr_grace_locked): every
    // active QP has started a service pass under a new MR epoch (so no per-warp cache still
    // serves the entry) and has retired every WR issued before that (so nothing in flight
    // still addresses the memory).  Only if that does not happen in time is the executor
    // quiesced, as for the other destructive operations.
    {
        std::lock_guard<std::mutex> lk(mu_);
        const uint32_t invalid = 0;
        copy_to_device(&mrs_[mr.table_slot].valid, &invalid, sizeof(invalid));
        if (mr_grace_locked()) {
            DevMr d{};
            copy_to_device(&mrs_[mr.table_slot], &d, sizeof(d));
            mr_fast_detaches_ += 1;
            return;
        }
        mr_slow_detaches_ += 1;
    }
    quiesce();
    {
        std::lock_guard<std::mutex> lk(mu_);
        DevMr d{};
        copy_to_device(&mrs_[mr.table_slot], &d, sizeof(d));
    }
    resume();
}

// ---- CQs --------------------------------------------------------------------------------------

void GpuEngine::reclaim_slots(bool qp) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        const bool full = qp ? free_qp_slots_.empty() && next_qp_slot_ >= kMaxQpsPerEngine
                             : free_cq_slots_.empty() && next_cq_slot_ >= kMaxCqsPerEngine;
        const bool cooling = qp ? !cooling_qp_slots_.empty() : !cooling_cq_slots_.empty();
        if (!full || !cooling) return;
    }
    quiesce();
    {
        std::lock_guard<std::mutex> lk(mu_);
        reap_locked();
    }
    resume();
}

int GpuEngine::attach_cq(control::Cq &cq) {
    reclaim_slots(false);
    std::lock_guard<std::mutex> lk(mu_);
    uint32_t slot;
    if (!free_cq_slots_.empty()) {
        slot = free_cq_slots_.back();
        free_cq_slots_.pop_back();
    } else {
        if (next_cq_slot_ >= kMaxCqsPerEngine) return ENOSPC;
        slot = next_cq_slot_++;
    }
    set_device();
    void *dev = register_ring(cq.ring);
    if (dev == nullptr) {
        free_cq_slots_.push_back(slot);
        return ENOMEM;
    }
    DevCq d{};
    const uint32_t cap = cq.ring.geometry().capacity;
    if (cudaMalloc(reinterpret_cast<void **>(&d.cfg.ready), sizeof(unsigned long long) * cap) != cudaSuccess ||
        cudaMemset(d.cfg.ready, 0, sizeof(unsigned long long) * cap) != cudaSuccess) {
        (void)cudaGetLastError();
        if (d.cfg.ready) cudaFree(d.cfg.ready);
        cudaHostUnregister(cq.ring.mapping());
        free_cq_slots_.push_back(slot);
        return ENOMEM;
    }
    d.cfg.ring = static_cast<queue::RingHeader *>(dev);
    d.cfg.slots = static_cast<uint8_t *>(dev) + queue::kRingHeaderBytes;
    d.cfg.capacity = cq.ring.geometry().capacity;
    d.cfg.stride = cq.ring.geometry().stride;
    d.cfg.valid = 1;
    d.st.reserve = d.st.published = cq.ring.tail();
    d.st.head_seen = cq.ring.head();
    if (int rc = copy_to_device(&cqs_[slot], &d, sizeof(d)); rc != 0) {
        cudaFree(d.cfg.ready);
        cudaHostUnregister(cq.ring.mapping());
        free_cq_slots_.push_back(slot);
        return rc;
    }
    cq_ready_[slot] = d.cfg.ready;
    cq.engine_block = &cqs_[slot];
    return 0;
}

void GpuEngine::detach_cq(control::Cq &cq) noexcept {
    if (cq.engine_block == nullptr) return;
    // No QP uses the CQ any more (the control plane refuses otherwise), but a warp that retired a
    // destroyed QP's WRs a moment ago may still hold it in its CQ cache: its device entry stays as
    // it is, and the ring, the `ready` array and the slot go only in reap_locked().
    std::lock_guard<std::mutex> lk(mu_);
    DevCq *d = static_cast<DevCq *>(cq.engine_block);
    const uint32_t slot = uint32_t(d - cqs_);
    if (!wedged_) {
        deferred_rings_.push_back(std::move(cq.ring));
        deferred_ready_.push_back(cq_ready_[slot]);
        cq_ready_[slot] = nullptr;
        cooling_cq_slots_.push_back(slot);
    } else {
        graveyard_.push_back(std::move(cq.ring));
    }
    cq.engine_block = nullptr;
}

// ---- QPs --------------------------------------------------------------------------------------

void GpuEngine::fill_qp_config(control::Qp &qp, DevQpConfig *c) {
    std::memset(c, 0, sizeof(*c));
    for (const QpEntry &e : qps_host_) {
        if (e.qp != &qp) continue;
        c->sq = static_cast<queue::RingHeader *>(e.sq_dev);
        c->sq_slots = static_cast<uint8_t *>(e.sq_dev) + queue::kRingHeaderBytes;
        c->rq = static_cast<queue::RingHeader *>(e.rq_dev);
        c->rq_slots = static_cast<uint8_t *>(e.rq_dev) + queue::kRingHeaderBytes;
    }
    c->send_cq = static_cast<DevCq *>(qp.send_cq->engine_block);
    c->recv_cq = static_cast<DevCq *>(qp.recv_cq->engine_block);
    c->peer = (qp.peer != nullptr) ? static_cast<DevQp *>(qp.peer->engine_block) : nullptr;
    c->sq_cap = qp.sq.geometry().capacity;
    c->sq_stride = qp.sq.geometry().stride;
    c->rq_cap = qp.rq.geometry().capacity;
    c->rq_stride = qp.rq.geometry().stride;
    c->qpn = qp.qpn;
    c->pd_num = qp.pd_num;
    c->access = qp.access;
    c->max_send_sge = qp.caps.max_send_sge;
    c->state = uint32_t(qp.state);
    c->sq_sig_all = qp.sq_sig_all ? 1u : 0u;
    c->peer_lost = qp.peer_lost ? 1u : 0u;
    c->active = 1;
    c->timeout = qp.timeout;
    c->retry_cnt = qp.retry_cnt;
    c->rnr_retry = qp.rnr_retry;
    c->min_rnr_timer = qp.min_rnr_timer;
}

int GpuEngine::attach_qp(control::Qp &qp) {
    reclaim_slots(true);
    std::lock_guard<std::mutex> lk(mu_);
    uint32_t slot;
    if (!free_qp_slots_.empty()) {
        slot = free_qp_slots_.back();
        free_qp_slots_.pop_back();
    } else {
        if (next_qp_slot_ >= kMaxQpsPerEngine) return ENOSPC;
        slot = next_qp_slot_++;
    }
    set_device();
    QpEntry e;
    e.qp = &qp;
    e.slot = slot;
    e.sq_dev = register_ring(qp.sq);
    e.rq_dev = register_ring(qp.rq);
    if (e.sq_dev == nullptr || e.rq_dev == nullptr) {
        if (e.sq_dev) cudaHostUnregister(qp.sq.mapping());
        if (e.rq_dev) cudaHostUnregister(qp.rq.mapping());
        free_qp_slots_.push_back(slot);
        return ENOMEM;
    }
    qps_host_.push_back(e);
    qp.engine_block = &qps_[slot];
    // Whole slot: config (inactive for now) and a zeroed device state.
    std::unique_ptr<DevQp> d(new DevQp());
    std::memset(d.get(), 0, sizeof(DevQp));
    fill_qp_config(qp, &d->cfg);
    d->cfg.active = 0;
    int rc = copy_to_device(&qps_[slot], d.get(), sizeof(DevQp));
    const uint32_t one = 1;
    if (rc == 0) rc = copy_to_device(&qps_[slot].cfg.active, &one, sizeof(one));
    if (rc == 0 && slot + 1 > qp_slot_bound_) {
        qp_slot_bound_ = slot + 1;
        rc = copy_to_device(&stats_->qp_slots, &qp_slot_bound_, sizeof(uint32_t));
    }
    if (rc != 0) {
        qps_host_.pop_back();
        cudaHostUnregister(qp.sq.mapping());
        cudaHostUnregister(qp.rq.mapping());
        free_qp_slots_.push_back(slot);
        qp.engine_block = nullptr;
    }
    return rc;
}

void GpuEngine::update_qp(control::Qp &qp) {
    std::lock_guard<std::mutex> lk(mu_);
    if (qp.engine_block == nullptr) return;
    DevQp *d = static_cast<DevQp *>(qp.engine_block);
    DevQpConfig c;
    fill_qp_config(qp, &c);
    // Everything but the state first, then the state word, so a running kernel never sees the
    // new state with a half-written peer binding.
    DevQpConfig staged = c;
    uint32_t old_state = 0;
    copy_from_device(&old_state, &d->cfg.state, sizeof(old_state));
    staged.state = old_state;
    copy_to_device(&d->cfg, &staged, sizeof(staged));
    copy_to_device(&d->cfg.state, &c.state, sizeof(c.state));
    for (QpEntry &e : qps_host_)
        if (e.qp == &qp) e.error = qp.state == UGDR_QPS_ERR;
}

void GpuEngine::detach_qp(control::Qp &qp) noexcept {
    if (qp.engine_block == nullptr) return;
    // The owner warp stops servicing the slot at its next configuration refresh (within 20 us);
    // until the executor is not running its cached view may still read the rings, so they and
    // the slot are released only in reap_locked().  WRs still in flight are discarded.
    std::lock_guard<std::mutex> lk(mu_);
    DevQp *d = static_cast<DevQp *>(qp.engine_block);
    const uint32_t zero = 0;
    copy_to_device(&d->cfg.active, &zero, sizeof(zero));
    for (size_t i = 0; i < qps_host_.size(); ++i) {
        if (qps_host_[i].qp != &qp) continue;
        if (!wedged_) {
            deferred_rings_.push_back(std::move(qp.sq));
            deferred_rings_.push_back(std::move(qp.rq));
            cooling_qp_slots_.push_back(qps_host_[i].slot);
        } else {
            graveyard_.push_back(std::move(qp.sq));
            graveyard_.push_back(std::move(qp.rq));
        }
        qps_host_[i] = qps_host_.back();
        qps_host_.pop_back();
        break;
    }
    qp.engine_block = nullptr;
}

void GpuEngine::invalidate_caches() noexcept {
    std::lock_guard<std::mutex> lk(mu_);
    mr_epoch_ += 1;  // every warp reloads its MR, QP-view and CQ caches at its next pass
    copy_to_device(&stats_->mr_epoch, &mr_epoch_, sizeof(mr_epoch_));
}

bool GpuEngine::settle() noexcept {
    std::lock_guard<std::mutex> lk(mu_);
    return mr_grace_locked();
}

void GpuEngine::reap_locked() {
    if (running_ || (deferred_rings_.empty() && deferred_ready_.empty() && cooling_qp_slots_.empty() &&
                     cooling_cq_slots_.empty()))
        return;
    if (copies_pending_locked()) return;  // a relaunch finishes them first
    set_device();
    for (queue::Ring &r : deferred_rings_) cudaHostUnregister(r.mapping());
    (void)cudaGetLastError();
    deferred_rings_.clear();  // unmaps
    for (unsigned long long *p : deferred_ready_)
        if (p) cudaFree(p);
    deferred_ready_.clear();
    free_qp_slots_.insert(free_qp_slots_.end(), cooling_qp_slots_.begin(), cooling_qp_slots_.end());
    free_cq_slots_.insert(free_cq_slots_.end(), cooling_cq_slots_.begin(), cooling_cq_slots_.end());
    cooling_qp_slots_.clear();
    cooling_cq_slots_.clear();
}

// ---- kernel life cycle ------------------------------------------------------------------------

bool GpuEngine::kernel_done_locked() {
    if (!running_) return true;
    const cudaError_t e = cudaEventQuery(ev_done_);
    if (e == cudaErrorNotReady) return false;
    (void)cudaGetLastError();
    running_ = false;
    DevStats st{};
    if (copy_from_device(&st, stats_, sizeof(st)) == 0 && st.error_code != 0) {
        std::fprintf(stderr, "ugdr: GPU %d executor stopped a bounded wait (code %u)\n",
                     cfg_.ordinal, st.error_code);
        const uint32_t zero = 0;
        copy_to_device(&stats_->error_code, &zero, sizeof(zero));
    }
    return true;
}

bool GpuEngine::mr_grace_locked() {
    if (!running_) return !copies_pending_locked();  // no kernel: nothing resolves or copies
    mr_epoch_ += 1;
    if (copy_to_device(&stats_->mr_epoch, &mr_epoch_, sizeof(mr_epoch_)) != 0) return false;
    const uint32_t epoch = mr_epoch_;
    uint32_t nslots = 0;
    for (const QpEntry &e : qps_host_) nslots = std::max(nslots, e.slot + 1);
    if (nslots == 0) return !copies_pending_locked();
    std::vector<QpProgress> pr(nslots);
    std::vector<uint32_t> issued(nslots, 0);
    const auto deadline = Clock::now() + std::chrono::milliseconds(cfg_.max_wait_ms);
    for (int phase = 0; phase < 2;) {
        if (copy_from_device(pr.data(), progress_, sizeof(QpProgress) * nslots) != 0) return false;
        bool all = true;
        for (const QpEntry &e : qps_host_) {
            const QpProgress &q = pr[e.slot];
            if (phase == 0)
                all &= int32_t(uint32_t(q.epoch_issue >> 32) - epoch) >= 0;
            else
                all &= int32_t(uint32_t(q.head) - issued[e.slot]) >= 0;
        }
        if (all) {
            if (phase == 0)
                for (const QpEntry &e : qps_host_) issued[e.slot] = uint32_t(pr[e.slot].epoch_issue);
            ++phase;
            continue;
        }
        if (kernel_done_locked()) return !copies_pending_locked();  // it went idle or stopped
        if (Clock::now() > deadline) return false;
        std::this_thread::sleep_for(std::chrono::microseconds(10));
    }
    return true;
}

bool GpuEngine::copies_pending_locked() {
    uint32_t words[32] = {};
    if (copy_from_device(words, reinterpret_cast<uint8_t *>(jobs_) + sizeof(JobRing), sizeof(words)) != 0)
        return false;
    for (uint32_t x : words)
        if (x != 0) return true;
    return false;
}

bool GpuEngine::stop_kernel_locked(uint32_t timeout_ms) {
    if (!running_) return true;
    set_device();
    __atomic_store_n(&ctrl_->stop, 1u, __ATOMIC_RELEASE);
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    while (!kernel_done_locked()) {
        if (Clock::now() > deadline) {
            std::fprintf(stderr, "ugdr: GPU %d executor did not stop within %u ms\n", cfg_.ordinal,
                         timeout_ms);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    __atomic_store_n(&ctrl_->stop, 0u, __ATOMIC_RELEASE);
    return true;
}

bool GpuEngine::has_work_locked() {
    for (const QpEntry &e : qps_host_) {
        const queue::Ring &sq = e.qp->sq;
        if (sq.tail() != sq.head()) return true;
        const bool err = e.error || sq.error_word() == UGDR_QPS_ERR;
        if (err && e.qp->rq.tail() != e.qp->rq.head()) return true;
    }
    return false;
}

int GpuEngine::launch_locked(uint32_t mode, uint64_t expected, bool timed) {
    TraceRange range(mode == kDrain ? "ugdr.executor.launch_drain" : "ugdr.executor.launch");
    set_device();
    // Reset the per-launch words: exiting flag, and (drain) the retired counter.
    const uint32_t zero = 0;
    if (copy_to_device(&stats_->exiting, &zero, sizeof(zero)) != 0) return EIO;
    if (mode == kDrain) {
        const uint64_t z = 0;
        if (copy_to_device(&stats_->retired, &z, sizeof(z)) != 0) return EIO;
    }
    ExecParams p{};
    p.mrs = mrs_;
    p.qps = qps_;
    p.jobs = jobs_;
    p.stats = stats_;
    p.ctrl = ctrl_dev_;
    p.mode = mode;
    p.expected = expected;
    p.idle_exit_ns = uint64_t(cfg_.idle_exit_us) * 1000ull;
    p.max_wait_ns = uint64_t(cfg_.max_wait_ms) * 1000000ull;
    p.trace = trace_;
    p.trace_count = trace_count_;
    p.trace_cap = trace_cap_;
    p.bulk_min = cfg_.bulk_min_bytes;
    p.progress = progress_;
    if (vis_.mode() == VisibilityGate::Mode::kFlush && vis_.before_publish() != 0) return EIO;
    if (timed) cudaEventRecord(ev_start_, exec_stream_);
    const int rc = launch_executor(p, cfg_.ctas, exec_stream_);
    if (rc != 0) {
        std::fprintf(stderr, "ugdr: GPU %d executor launch failed: %s\n", cfg_.ordinal,
                     cudaGetErrorString(cudaError_t(rc)));
        return EIO;
    }
    cudaEventRecord(ev_done_, exec_stream_);
    running_ = true;
    launches_ += 1;
    return 0;
}

void GpuEngine::monitor() {
    set_device();
    while (!stop_monitor_.load()) {
        bool idle = true;
        {
            std::lock_guard<std::mutex> lk(mu_);
            kernel_done_locked();
            if (!running_) {  // what destroyed objects left behind is released only now
                reap_ipc_closes(cfg_.ordinal);
                reap_locked();
            }
            if (!running_ && !held_ && paused_ == 0 && has_work_locked()) {
                launch_locked(kPersistent, 0, false);
                idle = false;
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(idle ? 20 : 5));
    }
}

void GpuEngine::quiesce() {
    TraceRange range("ugdr.engine.quiesce");
    std::lock_guard<std::mutex> lk(mu_);
    paused_ += 1;
    // Every device wait is bounded by max_wait_ms and the kernel checks the stop flag between
    // waits, so one round normally suffices; a few more cover a pass that chains several waits.
    bool stopped = false;
    for (int round = 0; round < 4 && !stopped; ++round) stopped = stop_kernel_locked(cfg_.max_wait_ms * 4);
    // The caller is about to take memory away (an MR, a ring).  A stop can leave chunked copies
    // with unclaimed pieces whose resolved addresses point into it, so run the executor on until
    // none is left (bounded; a held engine is not restarted).
    const auto deadline = Clock::now() + std::chrono::milliseconds(cfg_.max_wait_ms);
    while (stopped && !held_ && copies_pending_locked() && Clock::now() < deadline) {
        if (launch_locked(kPersistent, 0, false) != 0) break;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
        stopped = stop_kernel_locked(cfg_.max_wait_ms * 4);
    }
    if (stopped && copies_pending_locked())
        std::fprintf(stderr, "ugdr: GPU %d stopped with chunked copies still pending\n", cfg_.ordinal);
    wedged_ = !stopped;
    if (wedged_)
        std::fprintf(stderr, "ugdr: GPU %d executor did not stop; ring memory of destroyed objects stays registered\n",
                     cfg_.ordinal);
}

void GpuEngine::resume() {
    std::lock_guard<std::mutex> lk(mu_);
    if (paused_ > 0) paused_ -= 1;
}

int GpuEngine::trace(uint32_t records_per_unit) {
    if (records_per_unit > (1u << 20)) return EINVAL;
    quiesce();
    int rc = 0;
    {
        std::lock_guard<std::mutex> lk(mu_);
        set_device();
        cudaFree(trace_);
        cudaFree(trace_count_);
        trace_ = nullptr;
        trace_count_ = nullptr;
        trace_cap_ = 0;
        if (records_per_unit > 0) {
            const size_t n = size_t(cfg_.ctas) * records_per_unit;
            if (cudaMalloc(reinterpret_cast<void **>(&trace_), n * sizeof(TraceRec)) != cudaSuccess ||
                cudaMalloc(reinterpret_cast<void **>(&trace_count_), size_t(cfg_.ctas) * sizeof(unsigned int)) !=
                    cudaSuccess ||
                cudaMemsetAsync(trace_count_, 0, size_t(cfg_.ctas) * sizeof(unsigned int), ctl_stream_) !=
                    cudaSuccess ||
                cudaStreamSynchronize(ctl_stream_) != cudaSuccess) {
                (void)cudaGetLastError();
                cudaFree(trace_);
                cudaFree(trace_count_);
                trace_ = nullptr;
                trace_count_ = nullptr;
                rc = ENOMEM;
            } else {
                trace_cap_ = records_per_unit;
            }
        }
    }
    resume();
    return rc;
}

// Chrome trace-event JSON ("X" events, microseconds from the first record): one row per warp,
// grouped by CTA.  The counters restart, so each dump holds the events since the last one.
int GpuEngine::trace_dump(const std::string &path, uint64_t *kept, uint64_t *dropped) {
    quiesce();
    int rc = 0;
    std::vector<unsigned int> counts;
    std::vector<TraceRec> recs;
    uint32_t cap = 0;
    {
        std::lock_guard<std::mutex> lk(mu_);
        if (trace_ == nullptr) {
            rc = EINVAL;
        } else {
            cap = trace_cap_;
            counts.resize(size_t(cfg_.ctas));
            recs.resize(size_t(cfg_.ctas) * trace_cap_);
            if (copy_from_device(counts.data(), trace_count_, counts.size() * sizeof(unsigned int)) != 0 ||
                copy_from_device(recs.data(), trace_, recs.size() * sizeof(TraceRec)) != 0) {
                rc = EIO;
            } else {
                cudaMemsetAsync(trace_count_, 0, counts.size() * sizeof(unsigned int), ctl_stream_);
                cudaStreamSynchronize(ctl_stream_);
            }
        }
    }
    resume();
    if (rc != 0) return rc;
    return write_chrome_trace(path, recs, counts, cap, cfg_.ordinal, kept, dropped);
}

// The owner warp keeps each QP's byte and error counts in its device state; RNR waits are not
// counted per QP on the device (the engine-wide wait counters cover them).
int GpuEngine::qp_counters(control::Qp &qp, control::QpCounters *out) {
    std::lock_guard<std::mutex> lk(mu_);
    const auto *d = static_cast<const DevQp *>(qp.engine_block);
    if (d == nullptr) return ENOENT;
    unsigned long long v[2] = {0, 0};
    static_assert(offsetof(DevQpState, errors) == offsetof(DevQpState, bytes) + sizeof(unsigned long long));
    if (int rc = copy_from_device(v, &d->st.bytes, sizeof(v)); rc != 0) return rc;
    out->bytes = v[0];
    out->error_completions = v[1];
    out->rnr_waits = 0;
    return 0;
}

int GpuEngine::stats(control::EngineStats *out, bool reset) {
    std::lock_guard<std::mutex> lk(mu_);
    DevStats st{};
    if (int rc = copy_from_device(&st, stats_, sizeof(st)); rc != 0) return rc;
    out->wrs_completed = st.wrs_completed;
    out->bytes_moved = st.bytes_moved;
    out->error_completions = st.error_completions;
    out->wait_timeouts = st.wait_timeouts;
    out->first_start_ns = st.first_start_ns;
    out->last_end_ns = st.last_end_ns;
    out->launches = launches_;
    out->chunks_run = st.chunks_run;
    out->claim_misses = st.claim_misses;
    out->jobs_published = st.jobs_published;
    out->inline_runs = st.inline_runs;
    out->busy_ns = st.busy_ns;
    out->fast_batches = st.fast_batches;
    out->fast_fetch_ns = st.fast_fetch_ns;
    out->fast_exec_ns = st.fast_exec_ns;
    out->fast_reserve_ns = st.fast_reserve_ns;
    out->fast_publish_ns = st.fast_publish_ns;
    out->slow_wrs = st.slow_wrs;
    out->slow_issue_ns = st.slow_issue_ns;
    out->job_slot_misses = st.job_slot_misses;
    out->publish_waits = st.publish_waits;
    out->publish_wait_ns = st.publish_wait_ns;
    out->mr_detach_live = mr_fast_detaches_;
    out->mr_detach_quiesced = mr_slow_detaches_;
    out->order_waits = st.order_waits;
    out->overlap_issues = st.overlap_issues;
    if (reset) {
        // Counters only (a running kernel may race a few increments into the fresh window).
        cudaMemsetAsync(stats_, 0, offsetof(DevStats, last_work_ns), ctl_stream_);
        cudaStreamSynchronize(ctl_stream_);
        launches_ = 0;
    }
    return 0;
}

int GpuEngine::hold(bool on) {
    std::lock_guard<std::mutex> lk(mu_);
    held_ = on;
    if (on) stop_kernel_locked(cfg_.max_wait_ms * 4);
    return 0;
}

int GpuEngine::start_drain(uint64_t expected) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!stop_kernel_locked(cfg_.max_wait_ms * 4)) return EBUSY;
    return launch_locked(kDrain, expected, true);
}

int GpuEngine::finish_drain(uint32_t timeout_ms, float *elapsed_ms) {
    TraceRange range("ugdr.engine.drain_wait");
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (kernel_done_locked()) break;
            if (Clock::now() > deadline) {
                stop_kernel_locked(cfg_.max_wait_ms * 4);
                return ETIMEDOUT;
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(10));
    }
    std::lock_guard<std::mutex> lk(mu_);
    set_device();
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, ev_start_, ev_done_) != cudaSuccess) {
        (void)cudaGetLastError();
        return EIO;
    }
    *elapsed_ms = ms;
    return 0;
}

}  // namespace

int make_gpu_engine(const GpuEngineConfig &cfg, std::mutex &, std::unique_ptr<control::Engine> *out) {
    auto e = std::make_unique<GpuEngine>(cfg);
    if (int rc = e->init(); rc != 0) return rc;
    *out = std::move(e);
    return 0;
}

}  // namespace ugdr::gpu
