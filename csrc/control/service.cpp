#include "control/service.hpp"

#include "common/trace.hpp"

#include "common/bytes.hpp"
#include "ugdr/api.hpp"

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <unistd.h>

namespace ugdr::control {
namespace {

Response status(int code) {
    Response r;
    r.status = code;
    return r;
}

Response with_identity(uint64_t id) {
    Response r;
    r.identity = id;
    return r;
}

constexpr uint32_t kKnownAccess = UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE |
                                  UGDR_ACCESS_REMOTE_READ | UGDR_ACCESS_REMOTE_ATOMIC;
constexpr uint32_t kRemoteAccess =
    UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ | UGDR_ACCESS_REMOTE_ATOMIC;
constexpr uint32_t kKnownMask = UGDR_QP_STATE | UGDR_QP_CUR_STATE | UGDR_QP_ACCESS_FLAGS |
                                UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY |
                                UGDR_QP_MIN_RNR_TIMER;
constexpr uint32_t kConnectMask =
    UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
constexpr uint32_t kMaxQueueDepth = 1u << 20;
constexpr uint32_t kMaxSge = 32;

struct WireAttr {
    uint32_t state = 0, cur_state = 0;
    int32_t access = 0;
    uint8_t timeout = 0, retry_cnt = 0, rnr_retry = 0, min_rnr_timer = 0;
};

bool read_attr(ByteReader &r, WireAttr *a) {
    uint32_t access = 0;
    return r.be(&a->state) && r.be(&a->cur_state) && r.be(&access) && r.be(&a->timeout) &&
           r.be(&a->retry_cnt) && r.be(&a->rnr_retry) && r.be(&a->min_rnr_timer) &&
           ((a->access = int32_t(access)), true);
}

bool retry_encodings_ok(const WireAttr &a) {
    return a.timeout <= kMaxTimeout && a.retry_cnt <= kMaxRetryCnt && a.rnr_retry <= kMaxRnrRetry &&
           a.min_rnr_timer <= kMaxMinRnrTimer;
}

}  // namespace

ControlPlane::ControlPlane(std::vector<Engine *> engines, MemoryBackend &memory)
    : engines_(std::move(engines)), memory_(memory) {
    for (size_t i = 0; i < engines_.size(); ++i) {
        DeviceInfo d = engines_[i]->info();
        d.identity = i + 1;
        devices_.push_back(d);
    }
}

ControlPlane::~ControlPlane() {
    // Reclaim everything still alive, children first.
    std::vector<uint64_t> ids;
    qps_.for_each([&](uint64_t id, uint64_t, Qp &) { ids.push_back(id); });
    for (uint64_t id : ids) erase_qp(id);
    ids.clear();
    mrs_.for_each([&](uint64_t id, uint64_t, Mr &) { ids.push_back(id); });
    for (uint64_t id : ids) erase_mr(id);
    ids.clear();
    cqs_.for_each([&](uint64_t id, uint64_t, Cq &) { ids.push_back(id); });
    for (uint64_t id : ids) erase_cq(id);
}

ipc::Message ControlPlane::handle(ipc::SessionId session, ipc::Message &&msg) {
    const uint32_t method = msg.env.method;
    Request req;
    Response resp;
    // Descriptors lost on the way in (the daemon is at its descriptor limit): refuse the request
    // instead of running it without them; the ones that arrived close with `msg`.
    const int rc = msg.fds_truncated ? EMFILE : decode_request(std::move(msg), &req);
    if (rc != 0) {
        resp.status = rc;
    } else {
        resp = dispatch(session, std::move(req));
    }
    ipc::Message out;
    if (encode_response(method, std::move(resp), &out) != 0) {
        Response fallback;
        fallback.status = EPROTO;
        encode_response(method, std::move(fallback), &out);
    }
    return out;
}

namespace {
const char *method_range(uint32_t m) {
    static const char *names[] = {"ugdr.rpc.unknown",        "ugdr.rpc.list_devices",    "ugdr.rpc.create_context",
                                  "ugdr.rpc.destroy_context", "ugdr.rpc.create_pd",       "ugdr.rpc.destroy_pd",
                                  "ugdr.rpc.register_mr",    "ugdr.rpc.deregister_mr",   "ugdr.rpc.create_cq",
                                  "ugdr.rpc.destroy_cq",     "ugdr.rpc.create_qp",       "ugdr.rpc.destroy_qp",
                                  "ugdr.rpc.query_qp",       "ugdr.rpc.modify_qp",       "ugdr.rpc.query_conn_info",
                                  "ugdr.rpc.connect_qp"};
    if (m < sizeof(names) / sizeof(names[0])) return names[m];
    switch (m) {
    case kEngineStats: return "ugdr.rpc.engine_stats";
    case kEngineHold: return "ugdr.rpc.engine_hold";
    case kTimedDrain: return "ugdr.rpc.timed_drain";
    case kQpStats: return "ugdr.rpc.qp_stats";
    case kEngineTrace: return "ugdr.rpc.engine_trace";
    case kDaemonStats: return "ugdr.rpc.daemon_stats";
    default: return names[0];
    }
}
}  // namespace

Response ControlPlane::dispatch(ipc::SessionId s, Request &&r) {
    TraceRange range(method_range(r.method));
    switch (r.method) {
    case kListDevices: return list_devices();
    case kCreateContext: return create_context(s, r);
    case kDestroyContext: return destroy_context(s, r);
    case kCreatePd: return create_pd(s, r);
    case kDestroyPd: return destroy_pd(s, r);
    case kRegisterMr: return register_mr(s, r);
    case kDeregisterMr: return deregister_mr(s, r);
    case kCreateCq: return create_cq(s, r);
    case kDestroyCq: return destroy_cq(s, r);
    case kCreateQp: return create_qp(s, r);
    case kDestroyQp: return destroy_qp(s, r);
    case kQueryQp: return query_qp(s, r);
    case kModifyQp: return modify_qp(s, r);
    case kQueryQpConnInfo: return query_conn_info(s, r);
    case kConnectQp: return connect_qp(s, r);
    case kEngineStats: return engine_stats(s, r);
    case kEngineHold: return engine_hold(s, r);
    case kTimedDrain: return timed_drain(s, r);
    case kQpStats: return qp_stats(s, r);
    case kEngineTrace: return engine_trace(s, r);
    case kDaemonStats: return daemon_stats(s, r);
    default: return status(EOPNOTSUPP);
    }
}

// ---- devices and contexts ---------------------------------------------------------------------

Response ControlPlane::list_devices() {
    Response r;
    ByteWriter w(&r.opaque);
    w.be(uint32_t(devices_.size()));
    for (const DeviceInfo &d : devices_) {
        w.be(d.identity).be(uint32_t(d.kind)).be(uint32_t(d.gpu_ordinal));
        w.be(uint16_t(d.name.size())).raw(d.name.data(), d.name.size());
    }
    return r;
}

Response ControlPlane::create_context(uint64_t s, const Request &r) {
    if (r.identity == 0 || r.identity > devices_.size()) return status(ENODEV);
    auto ctx = std::make_unique<Context>();
    ctx->device = uint32_t(r.identity - 1);
    const uint64_t id = contexts_.insert(s, std::move(ctx));
    return id == 0 ? status(ENOSPC) : with_identity(id);
}

Response ControlPlane::destroy_context(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr) return status(EINVAL);
    if (ctx->children != 0) return status(EBUSY);
    contexts_.erase(r.identity);
    return status(0);
}

// ---- PDs ------------------------------------------------------------------------------------

Response ControlPlane::create_pd(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr) return status(EINVAL);
    auto pd = std::make_unique<Pd>();
    pd->context_id = r.identity;
    pd->pd_num = next_pd_num_++;
    const uint64_t id = pds_.insert(s, std::move(pd));
    if (id == 0) return status(ENOSPC);
    ctx->children += 1;
    return with_identity(id);
}

Response ControlPlane::destroy_pd(uint64_t s, const Request &r) {
    Pd *pd = pds_.find(s, r.identity);
    if (pd == nullptr) return status(EINVAL);
    if (pd->mrs != 0 || pd->qps != 0) return status(EBUSY);
    if (Context *ctx = contexts_.find_any(pd->context_id)) ctx->children -= 1;
    pds_.erase(r.identity);
    return status(0);
}

// ---- MRs ------------------------------------------------------------------------------------

Response ControlPlane::register_mr(uint64_t s, Request &r) {
    Pd *pd = pds_.find(s, r.identity);
    if (pd == nullptr) return status(EINVAL);
    Context *ctx = contexts_.find_any(pd->context_id);
    if (ctx == nullptr) return status(EINVAL);
    const uint32_t access = r.access;
    if (r.length == 0 || (access & ~kKnownAccess) != 0) return status(EINVAL);
    if ((access & (UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_ATOMIC)) != 0 &&
        (access & UGDR_ACCESS_LOCAL_WRITE) == 0)
        return status(EINVAL);

    MemoryDescriptor desc;
    ByteReader rd(r.opaque);
    uint8_t kind = 0, pad[3];
    if (!rd.be(&kind) || !rd.raw(pad, 3) || !rd.be(&desc.client_address)) return status(EPROTO);
    if (kind == uint8_t(MemKind::cuda)) {
        uint32_t handle_len = 0;
        desc.kind = MemKind::cuda;
        if (!rd.raw(desc.uuid.data(), 16) || !rd.be(&desc.allocation_bytes) ||
            !rd.be(&desc.allocation_offset) || !rd.be(&handle_len) || handle_len > 256)
            return status(EPROTO);
        desc.ipc_handle.resize(handle_len);
        if (!rd.raw(desc.ipc_handle.data(), handle_len) || !rd.done()) return status(EPROTO);
        if (desc.allocation_offset > desc.allocation_bytes ||
            r.length > desc.allocation_bytes - desc.allocation_offset)
            return status(EINVAL);
        if (!r.fds.empty()) return status(EPROTO);
    } else if (kind == uint8_t(MemKind::host)) {
        desc.kind = MemKind::host;
        if (!rd.be(&desc.region_bytes) || !rd.be(&desc.region_offset) || !rd.done())
            return status(EPROTO);
        if (r.fds.size() != 1) return status(EPROTO);
        if (desc.region_offset > desc.region_bytes || r.length > desc.region_bytes - desc.region_offset)
            return status(EINVAL);
        desc.region_fd = std::move(r.fds[0]);
    } else if (kind == uint8_t(MemKind::multicast)) {
        desc.kind = MemKind::multicast;
        if (!rd.be(&desc.region_bytes) || !rd.be(&desc.region_offset) || !rd.done()) return status(EPROTO);
        if (r.fds.size() != 1) return status(EPROTO);
        if (desc.region_offset != 0 || r.length > desc.region_bytes) return status(EINVAL);
        desc.region_fd = std::move(r.fds[0]);
    } else {
        return status(EOPNOTSUPP);
    }

    if (mrs_.full()) return status(ENOSPC);
    // Key slot.
    uint32_t slot;
    if (!free_key_slots_.empty()) {
        slot = free_key_slots_.back();
        free_key_slots_.pop_back();
    } else {
        if (key_slots_.size() >= kMaxMrSlots) return status(ENOSPC);
        slot = uint32_t(key_slots_.size());
        key_slots_.push_back(0);
        key_gens_.push_back(0);
    }
    const uint32_t gen = (key_gens_[slot] % 1023u) + 1u;

    auto mr = std::make_unique<Mr>();
    mr->pd_id = r.identity;
    mr->pd_num = pd->pd_num;
    mr->device = ctx->device;
    mr->client_address = desc.client_address;
    mr->length = r.length;
    mr->access = access;
    mr->lkey = make_key(gen, slot, false);
    mr->rkey = make_key(gen, slot, true);
    mr->handle = next_mr_handle_++;
    mr->table_slot = slot;
    if (int rc = memory_.open(desc, r.length, &mr->mem); rc != 0) {
        free_key_slots_.push_back(slot);
        return status(rc);
    }
    size_t attached = 0;
    int rc = 0;
    for (; attached < engines_.size(); ++attached) {
        if ((rc = engines_[attached]->attach_mr(*mr)) != 0) break;
    }
    if (rc != 0) {
        for (size_t i = 0; i < attached; ++i) engines_[i]->detach_mr(*mr);
        memory_.close(mr->mem);
        free_key_slots_.push_back(slot);
        return status(rc);
    }
    Mr *raw = mr.get();
    const uint64_t id = mrs_.insert(s, std::move(mr));
    key_slots_[slot] = id;
    key_gens_[slot] = gen;
    pd->mrs += 1;

    Response out;
    out.identity = id;
    ByteWriter w(&out.opaque);
    w.be(raw->client_address).be(raw->length).be(raw->lkey).be(raw->rkey).be(raw->handle);
    return out;
}

void ControlPlane::erase_mr(uint64_t id) noexcept {
    Mr *mr = mrs_.find_any(id);
    if (mr == nullptr) return;
    for (Engine *e : engines_) e->detach_mr(*mr);
    memory_.close(mr->mem);
    if (Pd *pd = pds_.find_any(mr->pd_id)) pd->mrs -= 1;
    key_slots_[mr->table_slot] = 0;
    free_key_slots_.push_back(mr->table_slot);
    mrs_.erase(id);
}

Response ControlPlane::deregister_mr(uint64_t s, const Request &r) {
    if (mrs_.find(s, r.identity) == nullptr) return status(EINVAL);
    erase_mr(r.identity);
    return status(0);
}

// ---- CQs ------------------------------------------------------------------------------------

Response ControlPlane::create_cq(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr) return status(EINVAL);
    if (r.length == 0 || r.length > kMaxQueueDepth) return status(EINVAL);
    auto cq = std::make_unique<Cq>();
    cq->context_id = r.identity;
    cq->device = ctx->device;
    cq->cq_num = next_cq_num_++;
    const queue::RingGeometry g{queue::kCompletionRing, uint32_t(r.length), queue::completion_stride()};
    if (int rc = queue::Ring::create(g, &cq->ring); rc != 0) return status(rc);
    if (cqs_.full()) return status(ENOSPC);
    Fd fd(::dup(cq->ring.fd()));
    if (!fd.valid()) return status(errno);
    if (int rc = engines_[cq->device]->attach_cq(*cq); rc != 0) return status(rc);
    Response out;
    const uint64_t id = cqs_.insert(s, std::move(cq));
    ctx->children += 1;
    out.identity = id;
    ByteWriter w(&out.opaque);
    w.be(g.capacity).be(g.stride);
    out.fds.push_back(std::move(fd));
    return out;
}

void ControlPlane::erase_cq(uint64_t id) noexcept {
    Cq *cq = cqs_.find_any(id);
    if (cq == nullptr) return;
    // Other engines' executors may cache this CQ (they produce receive completions into it).
    for (Engine *e : engines_)
        if (e != engines_[cq->device]) e->invalidate_caches();
    engines_[cq->device]->detach_cq(*cq);
    if (Context *ctx = contexts_.find_any(cq->context_id)) ctx->children -= 1;
    cqs_.erase(id);
}

Response ControlPlane::destroy_cq(uint64_t s, const Request &r) {
    Cq *cq = cqs_.find(s, r.identity);
    if (cq == nullptr) return status(EINVAL);
    if (cq->qp_refs != 0) return status(EBUSY);
    erase_cq(r.identity);
    return status(0);
}

// ---- QPs ------------------------------------------------------------------------------------

Response ControlPlane::create_qp(uint64_t s, const Request &r) {
    Pd *pd = pds_.find(s, r.identity);
    if (pd == nullptr) return status(EINVAL);
    ByteReader rd(r.opaque);
    uint64_t send_cq_id = 0, recv_cq_id = 0;
    QpCaps caps;
    uint32_t qp_type = 0, sig_all = 0;
    if (!rd.be(&send_cq_id) || !rd.be(&recv_cq_id) || !rd.be(&caps.max_send_wr) ||
        !rd.be(&caps.max_recv_wr) || !rd.be(&caps.max_send_sge) || !rd.be(&caps.max_recv_sge) ||
        !rd.be(&qp_type) || !rd.be(&sig_all) || !rd.done())
        return status(EPROTO);
    Cq *scq = cqs_.find(s, send_cq_id);
    Cq *rcq = cqs_.find(s, recv_cq_id);
    if (scq == nullptr || rcq == nullptr) return status(EINVAL);
    if (scq->context_id != pd->context_id || rcq->context_id != pd->context_id) return status(EINVAL);
    if (caps.max_send_wr == 0 || caps.max_recv_wr == 0 || caps.max_send_sge == 0 ||
        caps.max_recv_sge == 0 || qp_type != UGDR_QPT_RC || sig_all > 1)
        return status(EINVAL);
    if (caps.max_send_wr > kMaxQueueDepth || caps.max_recv_wr > kMaxQueueDepth ||
        caps.max_send_sge > kMaxSge || caps.max_recv_sge > kMaxSge)
        return status(EINVAL);
    if (next_qpn_ == 0 || next_qpn_ > 0x00ffffffu || qps_.full()) return status(ENOSPC);

    Context *ctx = contexts_.find_any(pd->context_id);
    auto qp = std::make_unique<Qp>();
    qp->pd_id = r.identity;
    qp->pd_num = pd->pd_num;
    qp->device = ctx->device;
    qp->send_cq_id = send_cq_id;
    qp->recv_cq_id = recv_cq_id;
    qp->send_cq = scq;
    qp->recv_cq = rcq;
    qp->caps = caps;
    qp->sq_sig_all = sig_all != 0;
    qp->state = UGDR_QPS_RESET;
    const queue::RingGeometry sg{queue::kSendRing, caps.max_send_wr, queue::send_stride(caps.max_send_sge)};
    const queue::RingGeometry rg{queue::kRecvRing, caps.max_recv_wr, queue::recv_stride(caps.max_recv_sge)};
    if (int rc = queue::Ring::create(sg, &qp->sq); rc != 0) return status(rc);
    if (int rc = queue::Ring::create(rg, &qp->rq); rc != 0) return status(rc);
    Fd sfd(::dup(qp->sq.fd())), rfd(::dup(qp->rq.fd()));
    if (!sfd.valid() || !rfd.valid()) return status(EMFILE);
    qp->qpn = next_qpn_;
    if (int rc = engines_[qp->device]->attach_qp(*qp); rc != 0) return status(rc);
    Qp *raw = qp.get();
    const uint64_t id = qps_.insert(s, std::move(qp));
    next_qpn_ += 1;
    qpn_index_[raw->qpn] = id;
    pd->qps += 1;
    scq->qp_refs += 1;
    rcq->qp_refs += 1;

    Response out;
    out.identity = id;
    ByteWriter w(&out.opaque);
    w.be(raw->qpn).be(caps.max_send_wr).be(caps.max_recv_wr).be(caps.max_send_sge).be(caps.max_recv_sge);
    w.be(sg.capacity).be(sg.stride).be(rg.capacity).be(rg.stride);
    out.fds.push_back(std::move(sfd));
    out.fds.push_back(std::move(rfd));
    return out;
}

void ControlPlane::erase_qp(uint64_t id) noexcept {
    Qp *qp = qps_.find_any(id);
    if (qp == nullptr) return;
    // Requesters bound to this QP lose their peer (later WRs fail with RETRY_EXC).  Their
    // engines may be on other GPUs and may be executing a WRITE_WITH_IMM into this QP's receive
    // ring at this moment, so each is stopped before the binding changes and stays stopped until
    // this QP's rings are gone from its own engine.
    // An engine that detaches live keeps the QP's memory until it is not running, which covers
    // its own requesters.  Requesters on other live engines are unbound while they run, and
    // their engine then settles (every QP re-reads its binding and retires what it issued under
    // the old one); an engine that cannot settle in time, or does not detach live, is stopped.
    std::vector<Engine *> held, settle;
    Engine *own = engines_[qp->device];
    qps_.for_each([&](uint64_t, uint64_t, Qp &other) {
        if (other.peer != qp) return;
        Engine *e = engines_[other.device];
        const bool live = e->detaches_live();
        if (!live && std::find(held.begin(), held.end(), e) == held.end()) {
            e->quiesce();
            held.push_back(e);
        }
        other.peer = nullptr;
        other.peer_lost = true;
        e->update_qp(other);
        if (live && e != own && std::find(settle.begin(), settle.end(), e) == settle.end()) settle.push_back(e);
    });
    for (Engine *e : settle) {
        if (!e->settle()) {
            e->quiesce();
            held.push_back(e);
        }
    }
    engines_[qp->device]->detach_qp(*qp);
    for (Engine *e : held) e->resume();
    qpn_index_.erase(qp->qpn);
    if (Pd *pd = pds_.find_any(qp->pd_id)) pd->qps -= 1;
    if (qp->send_cq) qp->send_cq->qp_refs -= 1;
    if (qp->recv_cq) qp->recv_cq->qp_refs -= 1;
    qps_.erase(id);
}

Response ControlPlane::destroy_qp(uint64_t s, const Request &r) {
    if (qps_.find(s, r.identity) == nullptr) return status(EINVAL);
    erase_qp(r.identity);
    return status(0);
}

Response ControlPlane::query_qp(uint64_t s, const Request &r) {
    Qp *qp = qps_.find(s, r.identity);
    if (qp == nullptr) return status(EINVAL);
    // An executor that hit an execution error moved the QP to ERR through the ring's error word.
    if (qp->state != UGDR_QPS_ERR && qp->sq.error_word() == UGDR_QPS_ERR) qp->state = UGDR_QPS_ERR;
    Response out;
    ByteWriter w(&out.opaque);
    w.be(uint32_t(qp->state)).be(qp->access).be(qp->timeout).be(qp->retry_cnt).be(qp->rnr_retry);
    w.be(qp->min_rnr_timer).be(qp->peer_qpn);
    return out;
}

void ControlPlane::set_error_state(Qp &qp) {
    qp.state = UGDR_QPS_ERR;
    qp.sq.set_error_word(UGDR_QPS_ERR);
    engines_[qp.device]->update_qp(qp);
}

Response ControlPlane::modify_qp(uint64_t s, const Request &r) {
    Qp *qp = qps_.find(s, r.identity);
    if (qp == nullptr) return status(EINVAL);
    const uint32_t mask = r.access;
    WireAttr a;
    ByteReader rd(r.opaque);
    if (!read_attr(rd, &a) || !rd.done()) return status(EPROTO);
    if ((mask & ~kKnownMask) != 0 || (mask & UGDR_QP_STATE) == 0) return status(EINVAL);
    if (a.state == UGDR_QPS_SQD || a.state == UGDR_QPS_SQE) return status(EOPNOTSUPP);
    const int from = qp->state;
    if ((mask & UGDR_QP_CUR_STATE) != 0 && int(a.cur_state) != from) return status(EINVAL);
    const uint32_t extra = mask & ~(UGDR_QP_STATE | UGDR_QP_CUR_STATE);
    if (a.state == UGDR_QPS_INIT) {
        if (from != UGDR_QPS_RESET || extra != UGDR_QP_ACCESS_FLAGS) return status(EINVAL);
        const uint32_t acc = uint32_t(a.access);
        if (acc == 0 || (acc & ~kRemoteAccess) != 0) return status(EINVAL);
        qp->access = acc;
        qp->state = UGDR_QPS_INIT;
        engines_[qp->device]->update_qp(*qp);
        return status(0);
    }
    if (a.state == UGDR_QPS_ERR) {
        if (extra != 0) return status(EINVAL);
        if (from != UGDR_QPS_RESET && from != UGDR_QPS_INIT && from != UGDR_QPS_RTR &&
            from != UGDR_QPS_RTS)
            return status(EINVAL);
        set_error_state(*qp);
        return status(0);
    }
    return status(EINVAL);
}

Response ControlPlane::query_conn_info(uint64_t s, const Request &r) {
    Qp *qp = qps_.find(s, r.identity);
    if (qp == nullptr) return status(EINVAL);
    Response out;
    ByteWriter w(&out.opaque);
    w.be(qp->qpn);
    return out;
}

Response ControlPlane::connect_qp(uint64_t s, const Request &r) {
    Qp *qp = qps_.find(s, r.identity);
    if (qp == nullptr) return status(EINVAL);
    ByteReader rd(r.opaque);
    uint32_t remote_qpn = 0;
    WireAttr a;
    if (!rd.be(&remote_qpn) || !read_attr(rd, &a) || !rd.done()) return status(EPROTO);
    if (remote_qpn == 0 || r.access != kConnectMask || !retry_encodings_ok(a)) return status(EINVAL);
    if (qp->peer_qpn != 0 && qp->peer_qpn != remote_qpn) return status(EBUSY);
    if (qp->state != UGDR_QPS_INIT) return status(EINVAL);
    auto it = qpn_index_.find(remote_qpn);
    if (it == qpn_index_.end()) return status(ENOENT);
    Qp *remote = qps_.find_any(it->second);
    if (remote == nullptr) return status(ENOENT);
    if (remote->state != UGDR_QPS_INIT && remote->state != UGDR_QPS_RTR &&
        remote->state != UGDR_QPS_RTS)
        return status(EINVAL);
    if (devices_[remote->device].kind != devices_[qp->device].kind) return status(EINVAL);
    // Stage everything, then commit once.
    qp->timeout = a.timeout;
    qp->retry_cnt = a.retry_cnt;
    qp->rnr_retry = a.rnr_retry;
    qp->min_rnr_timer = a.min_rnr_timer;
    qp->peer = remote;
    qp->peer_qpn = remote_qpn;
    qp->peer_lost = false;
    qp->state = UGDR_QPS_RTS;
    engines_[qp->device]->update_qp(*qp);
    return status(0);
}

// ---- extensions -----------------------------------------------------------------------------

Response ControlPlane::engine_stats(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr) return status(EINVAL);
    EngineStats st;
    if (int rc = engines_[ctx->device]->stats(&st, r.access != 0); rc != 0) return status(rc);
    Response out;
    ByteWriter w(&out.opaque);
    w.be(st.wrs_completed).be(st.bytes_moved).be(st.error_completions).be(st.launches);
    w.be(st.wait_timeouts).be(st.first_start_ns).be(st.last_end_ns);
    w.be(st.chunks_run).be(st.claim_misses).be(st.jobs_published).be(st.inline_runs).be(st.busy_ns);
    w.be(st.fast_batches).be(st.fast_fetch_ns).be(st.fast_exec_ns).be(st.fast_reserve_ns).be(st.fast_publish_ns);
    w.be(st.slow_wrs).be(st.slow_issue_ns).be(st.job_slot_misses).be(st.publish_waits).be(st.publish_wait_ns);
    w.be(st.mr_detach_live).be(st.mr_detach_quiesced).be(st.order_waits).be(st.overlap_issues);
    return out;
}

// Ring cursors give the WR counts for every engine: the SQ and RQ tails are what the client
// posted, their heads what the engine retired or consumed.  The engine adds its own counters
// (zero when it keeps none).
Response ControlPlane::qp_stats(uint64_t s, const Request &r) {
    Qp *qp = qps_.find(s, r.identity);
    if (qp == nullptr) return status(EINVAL);
    QpCounters c;
    if (int rc = engines_[qp->device]->qp_counters(*qp, &c); rc != 0 && rc != EOPNOTSUPP) return status(rc);
    if (qp->state != UGDR_QPS_ERR && qp->sq.error_word() == UGDR_QPS_ERR) qp->state = UGDR_QPS_ERR;
    Response out;
    ByteWriter w(&out.opaque);
    w.be(qp->sq.tail()).be(qp->sq.head()).be(qp->rq.tail()).be(qp->rq.head());
    w.be(c.bytes).be(c.error_completions).be(c.rnr_waits).be(uint32_t(qp->state));
    return out;
}

// access 0: keep r.length trace records per execution unit from now on (0 = off);
// access 1: write the kept records to the file named by the payload (the daemon's file system).
Response ControlPlane::engine_trace(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr || r.access > 1) return status(EINVAL);
    Engine *e = engines_[ctx->device];
    if (r.access == 0) {
        if (r.length > 0xffffffffull) return status(EINVAL);
        return status(e->trace(uint32_t(r.length)));
    }
    if (r.opaque.empty() || r.opaque.size() > 4096) return status(EINVAL);
    const std::string path(reinterpret_cast<const char *>(r.opaque.data()), r.opaque.size());
    if (path.find('\0') != std::string::npos) return status(EINVAL);
    uint64_t kept = 0, dropped = 0;
    if (int rc = e->trace_dump(path, &kept, &dropped); rc != 0) return status(rc);
    Response out;
    ByteWriter w(&out.opaque);
    w.be(kept).be(dropped);
    return out;
}

// Live objects of every session (operators' view of the daemon), and the device count.
Response ControlPlane::daemon_stats(uint64_t, const Request &) {
    Response out;
    ByteWriter w(&out.opaque);
    w.be(uint64_t(engines_.size())).be(uint64_t(contexts_.size())).be(uint64_t(pds_.size()));
    w.be(uint64_t(mrs_.size())).be(uint64_t(cqs_.size())).be(uint64_t(qps_.size()));
    return out;
}

Response ControlPlane::engine_hold(uint64_t s, const Request &r) {
    Context *ctx = contexts_.find(s, r.identity);
    if (ctx == nullptr) return status(EINVAL);
    return status(engines_[ctx->device]->hold(r.access != 0));
}

Response ControlPlane::timed_drain(uint64_t s, const Request &r) {
    ByteReader rd(r.opaque);
    uint32_t n = 0;
    if (!rd.be(&n) || n == 0 || n > engines_.size() * 64) return status(EINVAL);
    std::vector<std::pair<Engine *, uint64_t>> work;
    for (uint32_t i = 0; i < n; ++i) {
        uint64_t ctx_id = 0, expected = 0;
        if (!rd.be(&ctx_id) || !rd.be(&expected)) return status(EPROTO);
        // Contexts of other sessions are allowed: one rank drives the whole node's drain.
        Context *ctx = contexts_.find_any(ctx_id);
        if (ctx == nullptr) return status(EINVAL);
        work.emplace_back(engines_[ctx->device], expected);
    }
    if (!rd.done()) return status(EPROTO);
    int rc = 0;
    size_t started = 0;
    for (; started < work.size(); ++started) {
        if ((rc = work[started].first->start_drain(work[started].second)) != 0) break;
    }
    Response out;
    ByteWriter w(&out.opaque);
    for (size_t i = 0; i < started; ++i) {
        float ms = 0.f;
        const int frc = work[i].first->finish_drain(uint32_t(r.length), &ms);
        if (rc == 0) rc = frc;
        uint32_t bits;
        std::memcpy(&bits, &ms, 4);
        w.be(bits);
    }
    out.status = rc;
    return out;
}

// ---- session reclaim ------------------------------------------------------------------------

void ControlPlane::on_disconnect(ipc::SessionId s) noexcept {
    for (uint64_t id : qps_.owned_by(s)) erase_qp(id);
    for (uint64_t id : mrs_.owned_by(s)) erase_mr(id);
    for (uint64_t id : cqs_.owned_by(s)) erase_cq(id);
    for (uint64_t id : pds_.owned_by(s)) {
        if (Pd *pd = pds_.find_any(id))
            if (Context *ctx = contexts_.find_any(pd->context_id)) ctx->children -= 1;
        pds_.erase(id);
    }
    for (uint64_t id : contexts_.owned_by(s)) contexts_.erase(id);
}

}  // namespace ugdr::control
