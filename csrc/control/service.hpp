// The daemon control plane: device catalog, contexts, PDs, MRs, CQs and RC QPs.
//
// Parity: the reference splits this across DeviceContextService -> PdMrCqService -> QpService
// (src/control/device_context.cpp:146-236, src/control/pd_mr_cq.cpp:365-602,
// src/control/qp.cpp:450-741).  Here one class owns every registry so lifecycle checks
// (EBUSY on live children, session reclaim order QP -> MR -> CQ -> PD -> context) live in one
// place, and each data-path change is forwarded to the owning Engine.
//
// Error domain: every handler returns 0 or a positive errno that travels in the envelope.
// Invalid, stale or foreign handles are EINVAL; live children are EBUSY; an unknown remote QPN
// is ENOENT; SQD / SQE targets are EOPNOTSUPP.  All failures leave state unchanged.
#pragma once

#include "control/handles.hpp"
#include "control/objects.hpp"
#include "control/rpc.hpp"
#include "ipc/ipc.hpp"

#include <memory>
#include <unordered_map>
#include <vector>

namespace ugdr::control {

class ControlPlane : public ipc::Handler {
  public:
    // `engines[i]` executes device i; the daemon keeps ownership of engines and backend.
    ControlPlane(std::vector<Engine *> engines, MemoryBackend &memory);
    ~ControlPlane() override;

    ipc::Message handle(ipc::SessionId session, ipc::Message &&req) override;
    void on_disconnect(ipc::SessionId session) noexcept override;

    // Direct entry (tests drive the service without sockets).
    Response dispatch(ipc::SessionId session, Request &&req);

    size_t context_count() const { return contexts_.size(); }
    size_t pd_count() const { return pds_.size(); }
    size_t mr_count() const { return mrs_.size(); }
    size_t cq_count() const { return cqs_.size(); }
    size_t qp_count() const { return qps_.size(); }
    const std::vector<DeviceInfo> &devices() const { return devices_; }

  private:
    Response list_devices();
    Response create_context(uint64_t s, const Request &r);
    Response destroy_context(uint64_t s, const Request &r);
    Response create_pd(uint64_t s, const Request &r);
    Response destroy_pd(uint64_t s, const Request &r);
    Response register_mr(uint64_t s, Request &r);
    Response deregister_mr(uint64_t s, const Request &r);
    Response create_cq(uint64_t s, const Request &r);
    Response destroy_cq(uint64_t s, const Request &r);
    Response create_qp(uint64_t s, const Request &r);
    Response destroy_qp(uint64_t s, const Request &r);
    Response query_qp(uint64_t s, const Request &r);
    Response modify_qp(uint64_t s, const Request &r);
    Response query_conn_info(uint64_t s, const Request &r);
    Response connect_qp(uint64_t s, const Request &r);
    Response engine_stats(uint64_t s, const Request &r);
    Response engine_hold(uint64_t s, const Request &r);
    Response qp_stats(uint64_t s, const Request &r);
    Response engine_trace(uint64_t s, const Request &r);
    Response daemon_stats(uint64_t s, const Request &r);
    Response timed_drain(uint64_t s, const Request &r);

    void erase_qp(uint64_t id) noexcept;
    void erase_mr(uint64_t id) noexcept;
    void erase_cq(uint64_t id) noexcept;
    void set_error_state(Qp &qp);

    std::vector<Engine *> engines_;
    MemoryBackend &memory_;
    std::vector<DeviceInfo> devices_;

    Registry<Context> contexts_{ObjectType::context};
    Registry<Pd> pds_{ObjectType::pd};
    Registry<Mr> mrs_{ObjectType::mr};
    Registry<Cq> cqs_{ObjectType::cq};
    Registry<Qp> qps_{ObjectType::qp};

    std::unordered_map<uint32_t, uint64_t> qpn_index_;  // live QPN -> identity
    uint32_t next_qpn_ = 1;                             // never reused in a daemon lifetime
    uint32_t next_pd_num_ = 1;
    uint32_t next_cq_num_ = 1;
    uint32_t next_mr_handle_ = 1;
    // MR key table: slot -> MR identity; keys are (gen << 20 | slot) << 1 | {0 lkey, 1 rkey}.
    std::vector<uint64_t> key_slots_;
    std::vector<uint32_t> key_gens_;
    std::vector<uint32_t> free_key_slots_;
};

// Key helpers shared with the engines (device code re-derives them the same way).
constexpr uint32_t kKeySlotBits = 16;
constexpr uint32_t kMaxMrSlots = 1u << kKeySlotBits;
inline uint32_t key_slot(uint32_t key) { return (key >> 1) & (kMaxMrSlots - 1); }
inline uint32_t make_key(uint32_t gen, uint32_t slot, bool remote) {
    return (((gen & 0x3ffu) << kKeySlotBits | slot) << 1) | (remote ? 1u : 0u);
}

// Retry-attribute limits (standard RC encodings).
constexpr uint8_t kMaxTimeout = 31, kMaxRetryCnt = 7, kMaxRnrRetry = 7, kMaxMinRnrTimer = 31;

}  // namespace ugdr::control
