// Host-memory engine: executes WRITE / WRITE_WITH_IMM / READ / atomics on QPs of the CPU
// device with plain memcpy over memfd-mapped host MRs.
//
// It is the CPU-only data path (a daemon with no GPU still serves host-memory MRs) and the
// byte-exact oracle the GPU executors are tested against.  It replaces the reference's
// LoopWorker + LocalTransport + copy backend chain (src/worker/worker.cpp:63-509) with a direct
// executor: the "transport" between requester and responder is a function call because both
// live in this daemon.
#pragma once

#include "control/objects.hpp"

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

namespace ugdr::engine {

class CpuEngine : public control::Engine {
  public:
    // `objects_mu` is the control plane's object lock; the worker holds it while it runs WRs.
    CpuEngine(std::mutex &objects_mu, bool start_thread = true);
    ~CpuEngine() override;

    control::DeviceInfo info() const override;
    int attach_mr(control::Mr &mr) override;
    void detach_mr(control::Mr &mr) noexcept override;
    int attach_cq(control::Cq &cq) override;
    void detach_cq(control::Cq &cq) noexcept override;
    int attach_qp(control::Qp &qp) override;
    void update_qp(control::Qp &qp) override;
    void detach_qp(control::Qp &qp) noexcept override;
    void quiesce() override {}
    void resume() override {}
    int stats(control::EngineStats *out, bool reset) override;
    int qp_counters(control::Qp &qp, control::QpCounters *out) override;
    int hold(bool on) override;

    // One pass over every QP; caller holds the object lock.  Returns WRs retired.  Public so
    // tests can drive the engine deterministically without the thread.
    size_t progress_locked();

  private:
    struct MrView {
        uint8_t *base = nullptr;  // daemon address of the registered range (host MRs only)
        uint64_t client_base = 0;  // client address of the same byte
        uint64_t length = 0;
        uint32_t access = 0, pd_num = 0, lkey = 0, rkey = 0;
    };
    struct QpView {
        control::Qp *qp = nullptr;
        uint32_t rnr_attempts = 0;
        uint64_t rnr_next_ns = 0;
        // Last local and remote key this QP resolved (WRs of one QP mostly reuse one MR pair);
        // cleared whenever an MR is detached.
        const MrView *lm = nullptr, *rm = nullptr;
        uint32_t lkey = 0, rkey = 0;
        control::QpCounters c;
        bool rnr_waiting = false;  // an RNR wait episode is open (counted once)
    };
    const MrView *find(uint32_t key, bool remote) const;
    const MrView *find_cached(QpView &v, uint32_t key, bool remote) const;
    static uint8_t *resolve(const MrView *m, uint64_t addr, uint64_t len);
    size_t progress_qp(QpView &v);
    bool produce(control::Cq *cq, const void *cqe);
    void enter_error(control::Qp &qp);
    void run();

    std::mutex &objects_mu_;
    std::unordered_map<uint32_t, MrView> mrs_;  // key slot -> view
    std::vector<QpView> qps_;
    std::atomic<bool> stop_{false};
    std::atomic<bool> held_{false};
    std::thread worker_;
    control::EngineStats stats_;
};

}  // namespace ugdr::engine
