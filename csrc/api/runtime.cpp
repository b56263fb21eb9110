// The public C ABI (include/ugdr/api.hpp), implemented as a process-global client runtime.
//
// Parity: reference src/api/api.cpp:26-976 (proxy records, lazy daemon connect from
// UGDR_DAEMON_SOCKET, per-CQ poll mutex, per-QP posting mutex, extern "C" surface).  Here the
// per-QP and per-CQ locks are spin locks: their critical sections are a few slot copies.
//
// Design here: every proxy starts with a magic word and the connection epoch it was created
// under.  A destroyed proxy keeps its (small) shell with a dead magic, so a repeated destroy or
// a use-after-destroy is detected without a registry lookup on the post / poll fast path; a
// proxy from an earlier connection fails its epoch check.  Control calls serialise on one
// mutex (one socket); posting and polling touch only the shared rings.
#include "api/memory_export.hpp"
#include "api/posting.hpp"
#include "common/bytes.hpp"
#include "common/spinlock.hpp"
#include "control/client.hpp"
#include "control/rpc.hpp"
#include "queue/ring.hpp"
#include "ugdr/api.hpp"

#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_set>
#include <vector>

using ugdr::ByteReader;
using ugdr::ByteWriter;
using ugdr::Fd;
using namespace ugdr::control;

namespace {

constexpr uint32_t kLive = 0x75676472u;  // "ugdr"
constexpr uint32_t kDead = 0xdeadbeefu;
constexpr const char *kDefaultSocket = "/run/ugdr/ugdr.sock";

struct ProxyBase {
    uint32_t magic = kLive;
    uint64_t epoch = 0;
    uint64_t identity = 0;
};

}  // namespace

struct ugdr_device : ProxyBase {
    std::string name;
    int kind = 0;
    int gpu = -1;
};

struct ugdr_context : ProxyBase {
    uint64_t device_identity = 0;
    int kind = 0;
};

struct ugdr_pd : ProxyBase {
    ugdr_context *context = nullptr;
};

namespace {
// The public record comes first so a ugdr_mr * converts back to its proxy.
struct MrProxy {
    ugdr_mr pub{};
    ProxyBase b;
};
}  // namespace

struct ugdr_cq : ProxyBase {
    ugdr_context *context = nullptr;
    ugdr::queue::Ring ring;
    ugdr::SpinLock poll_mu;
};

struct ugdr_qp : ProxyBase {
    ugdr_pd *pd = nullptr;
    uint32_t qpn = 0;
    ugdr_qp_init_attr init{};
    ugdr::queue::Ring sq, rq;
    ugdr::SpinLock post_mu;
    std::atomic<int> state{UGDR_QPS_RESET};
    int access = 0;
    uint8_t timeout = 0, retry_cnt = 0, rnr_retry = 0, min_rnr_timer = 0;
};

namespace {

class Runtime {
  public:
    static Runtime &get() {
        static Runtime *rt = new Runtime();  // never destroyed: proxies may outlive main()
        return *rt;
    }

    // One control round trip.  Returns 0 / positive errno (transport or service status).
    int call(Request &&req, Response *resp, uint64_t min_wait_ms = 0) {
        std::lock_guard<std::mutex> lk(mu_);
        const char *env = std::getenv("UGDR_DAEMON_SOCKET");
        const std::string path = (env != nullptr && env[0] != '\0') ? env : kDefaultSocket;
        // (Re)connect when there is no connection, the configured daemon changed, or this is a
        // forked child (the inherited socket is the parent's session); either way the epoch
        // advances and proxies of the previous connection become stale in this process.
        const pid_t pid = ::getpid();
        if (!client_.connected() || path != path_ || pid != pid_) {
            if (int rc = client_.connect(path); rc != 0) return rc;
            path_ = path;
            pid_ = pid;
        }
        if (int rc = client_.call(std::move(req), resp, min_wait_ms); rc != 0) return rc;
        return resp->status;
    }
    uint64_t epoch() {
        std::lock_guard<std::mutex> lk(mu_);
        return client_.epoch();
    }
    bool live(const ProxyBase *p) {
        return p != nullptr && p->magic == kLive && p->epoch == epoch_relaxed();
    }
    uint64_t epoch_relaxed() { return client_.epoch(); }

    std::mutex lists_mu;
    std::unordered_set<ugdr_device **> lists;

    // Destroyed proxies keep a dead magic for a while: a repeated destroy, or a use shortly
    // after destroy, finds kDead instead of freed memory.  The shells wait in a bounded
    // quarantine and the oldest is freed once it holds kQuarantine of them, so a client that
    // creates and destroys objects forever keeps a fixed amount of memory.
    template <typename T> void retire(T *obj, ProxyBase *base) {
        base->magic = kDead;
        Shell victim{nullptr, nullptr};
        {
            std::lock_guard<std::mutex> lk(quarantine_mu_);
            quarantine_.push_back(Shell{obj, [](void *o) { delete static_cast<T *>(o); }});
            if (quarantine_.size() > kQuarantine) {
                victim = quarantine_.front();
                quarantine_.pop_front();
            }
        }
        if (victim.obj != nullptr) victim.del(victim.obj);
    }

  private:
    pid_t pid_ = 0;  // process that opened the current connection
    struct Shell {
        void *obj;
        void (*del)(void *);
    };
    static constexpr size_t kQuarantine = 4096;
    std::mutex mu_;
    ControlClient client_;
    std::string path_;
    std::mutex quarantine_mu_;
    std::deque<Shell> quarantine_;
};

Runtime &rt() { return Runtime::get(); }

template <typename T> T *fail_null(int err) {
    errno = err;
    return nullptr;
}

Request make(uint32_t method, uint64_t identity = 0) {
    Request r;
    r.method = method;
    r.identity = identity;
    return r;
}


int qp_state(ugdr_qp *qp) {
    if (qp->sq.valid() && qp->sq.error_word() == UGDR_QPS_ERR) return UGDR_QPS_ERR;
    return qp->state.load(std::memory_order_acquire);
}

void put_attr(ByteWriter &w, const ugdr_qp_attr *a) {
    w.be(uint32_t(a->qp_state)).be(uint32_t(a->cur_qp_state)).be(uint32_t(a->qp_access_flags));
    w.be(a->timeout).be(a->retry_cnt).be(a->rnr_retry).be(a->min_rnr_timer);
}

}  // namespace

extern "C" {

ugdr_device **ugdr_get_device_list(int *num_devices) noexcept {
    try {
        Response resp;
        if (int rc = rt().call(make(kListDevices), &resp); rc != 0) return fail_null<ugdr_device *>(rc);
        ByteReader rd(resp.opaque);
        uint32_t n = 0;
        if (!rd.be(&n) || n > 4096) return fail_null<ugdr_device *>(EPROTO);
        const uint64_t epoch = rt().epoch();
        std::vector<ugdr_device *> devs;
        for (uint32_t i = 0; i < n; ++i) {
            auto *d = new ugdr_device();
            uint32_t kind = 0, gpu = 0;
            uint16_t name_len = 0;
            if (!rd.be(&d->identity) || !rd.be(&kind) || !rd.be(&gpu) || !rd.be(&name_len)) {
                delete d;
                for (auto *x : devs) delete x;
                return fail_null<ugdr_device *>(EPROTO);
            }
            d->name.resize(name_len);
            rd.raw(d->name.data(), name_len);
            d->kind = int(kind);
            d->gpu = int(int32_t(gpu));
            d->epoch = epoch;
            devs.push_back(d);
        }
        auto **list = new ugdr_device *[n + 1];
        for (uint32_t i = 0; i < n; ++i) list[i] = devs[i];
        list[n] = nullptr;
        {
            std::lock_guard<std::mutex> lk(rt().lists_mu);
            rt().lists.insert(list);
        }
        if (num_devices != nullptr) *num_devices = int(n);
        return list;
    } catch (...) {
        return fail_null<ugdr_device *>(ENOMEM);
    }
}

void ugdr_free_device_list(ugdr_device **list) noexcept {
    std::lock_guard<std::mutex> lk(rt().lists_mu);
    auto it = rt().lists.find(list);
    if (it == rt().lists.end()) {
        errno = EINVAL;
        return;
    }
    rt().lists.erase(it);
    for (ugdr_device **p = list; *p != nullptr; ++p) rt().retire(*p, *p);
    delete[] list;
}

int ugdr_x_query_device(ugdr_device *device, ugdr_x_device_info *info) noexcept {
    if (device == nullptr || device->magic != kLive || info == nullptr) return EINVAL;
    std::memset(info, 0, sizeof(*info));
    std::strncpy(info->name, device->name.c_str(), sizeof(info->name) - 1);
    info->kind = device->kind;
    info->gpu_ordinal = device->gpu;
    info->identity = device->identity;
    return 0;
}

ugdr_context *ugdr_open_device(ugdr_device *device) noexcept {
    if (device == nullptr || device->magic != kLive || device->epoch != rt().epoch())
        return fail_null<ugdr_context>(EINVAL);
    Response resp;
    if (int rc = rt().call(make(kCreateContext, device->identity), &resp); rc != 0)
        return fail_null<ugdr_context>(rc);
    auto *ctx = new ugdr_context();
    ctx->identity = resp.identity;
    ctx->epoch = rt().epoch();
    ctx->device_identity = device->identity;
    ctx->kind = device->kind;
    return ctx;
}

int ugdr_close_device(ugdr_context *ctx) noexcept {
    if (!rt().live(ctx)) {
        errno = EINVAL;
        return -1;
    }
    Response resp;
    if (int rc = rt().call(make(kDestroyContext, ctx->identity), &resp); rc != 0) {
        errno = rc;
        return -1;
    }
    rt().retire(ctx, ctx);
    return 0;
}

ugdr_pd *ugdr_alloc_pd(ugdr_context *ctx) noexcept {
    if (!rt().live(ctx)) return fail_null<ugdr_pd>(EINVAL);
    Response resp;
    if (int rc = rt().call(make(kCreatePd, ctx->identity), &resp); rc != 0) return fail_null<ugdr_pd>(rc);
    auto *pd = new ugdr_pd();
    pd->identity = resp.identity;
    pd->epoch = ctx->epoch;
    pd->context = ctx;
    return pd;
}

int ugdr_dealloc_pd(ugdr_pd *pd) noexcept {
    if (!rt().live(pd)) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kDestroyPd, pd->identity), &resp); rc != 0) return rc;
    rt().retire(pd, pd);
    return 0;
}

namespace {
ugdr_mr *register_mr(ugdr_pd *pd, void *address, size_t length, int access, int mc_fd) noexcept {
    if (!rt().live(pd) || address == nullptr || length == 0) return fail_null<ugdr_mr>(EINVAL);
    try {
        Request req = make(kRegisterMr, pd->identity);
        req.length = length;
        req.access = uint32_t(access);
        const int rc0 = mc_fd < 0 ? ugdr::api::export_memory(address, length, &req.opaque, &req.fds)
                                  : ugdr::api::export_multicast(mc_fd, reinterpret_cast<uint64_t>(address), length,
                                                                &req.opaque, &req.fds);
        if (rc0 != 0) return fail_null<ugdr_mr>(rc0);
        Response resp;
        if (int rc = rt().call(std::move(req), &resp); rc != 0) return fail_null<ugdr_mr>(rc);
        ByteReader rd(resp.opaque);
        uint64_t addr = 0, len = 0;
        uint32_t lkey = 0, rkey = 0, handle = 0;
        if (!rd.be(&addr) || !rd.be(&len) || !rd.be(&lkey) || !rd.be(&rkey) || !rd.be(&handle))
            return fail_null<ugdr_mr>(EPROTO);
        auto *mr = new MrProxy();
        mr->b.identity = resp.identity;
        mr->b.epoch = pd->epoch;
        mr->pub.context = pd->context;
        mr->pub.pd = pd;
        mr->pub.addr = address;
        mr->pub.length = length;
        mr->pub.handle = handle;
        mr->pub.lkey = lkey;
        mr->pub.rkey = rkey;
        return &mr->pub;
    } catch (...) {
        return fail_null<ugdr_mr>(ENOMEM);
    }
}
}  // namespace

ugdr_mr *ugdr_reg_mr(ugdr_pd *pd, void *address, size_t length, int access) noexcept {
    return register_mr(pd, address, length, access, -1);
}

ugdr_mr *ugdr_x_reg_mr_multicast(ugdr_pd *pd, void *address, size_t length, int access, int mc_fd) noexcept {
    if (mc_fd < 0) return fail_null<ugdr_mr>(EINVAL);
    return register_mr(pd, address, length, access, mc_fd);
}

int ugdr_dereg_mr(ugdr_mr *mr) noexcept {
    if (mr == nullptr) return EINVAL;
    MrProxy *p = reinterpret_cast<MrProxy *>(mr);
    if (!rt().live(&p->b)) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kDeregisterMr, p->b.identity), &resp); rc != 0) return rc;
    rt().retire(p, &p->b);
    return 0;
}

ugdr_cq *ugdr_create_cq(ugdr_context *ctx, int cqe, void *, ugdr_comp_channel *channel,
                        int comp_vector) noexcept {
    if (!rt().live(ctx) || cqe <= 0 || channel != nullptr || comp_vector != 0)
        return fail_null<ugdr_cq>(EINVAL);
    try {
        Request req = make(kCreateCq, ctx->identity);
        req.length = uint64_t(cqe);
        Response resp;
        if (int rc = rt().call(std::move(req), &resp); rc != 0) return fail_null<ugdr_cq>(rc);
        ByteReader rd(resp.opaque);
        uint32_t cap = 0, stride = 0;
        if (!rd.be(&cap) || !rd.be(&stride) || resp.fds.size() != 1) return fail_null<ugdr_cq>(EPROTO);
        auto *cq = new ugdr_cq();
        const ugdr::queue::RingGeometry g{ugdr::queue::kCompletionRing, cap, stride};
        if (int rc = ugdr::queue::Ring::attach(resp.fds[0].release(), g, &cq->ring); rc != 0) {
            Response ignored;
            rt().call(make(kDestroyCq, resp.identity), &ignored);
            delete cq;
            return fail_null<ugdr_cq>(rc);
        }
        cq->identity = resp.identity;
        cq->epoch = ctx->epoch;
        cq->context = ctx;
        return cq;
    } catch (...) {
        return fail_null<ugdr_cq>(ENOMEM);
    }
}

int ugdr_destroy_cq(ugdr_cq *cq) noexcept {
    if (!rt().live(cq)) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kDestroyCq, cq->identity), &resp); rc != 0) return rc;
    {
        std::lock_guard<ugdr::SpinLock> lk(cq->poll_mu);
        cq->magic = kDead;
        cq->ring = ugdr::queue::Ring();
    }
    rt().retire(cq, cq);
    return 0;
}

int ugdr_poll_cq(ugdr_cq *cq, int num_entries, ugdr_wc *wc) noexcept {
    if (cq == nullptr || cq->magic != kLive || num_entries < 0 || (num_entries > 0 && wc == nullptr))
        return -EINVAL;
    std::lock_guard<ugdr::SpinLock> lk(cq->poll_mu);
    if (cq->magic != kLive) return -EINVAL;
    ugdr::queue::SlotRun run = cq->ring.peek(uint32_t(num_entries));
    const uint32_t n = run.count();
    const uint32_t stride = cq->ring.geometry().stride;
    for (uint32_t i = 0; i < n; ++i) {
        const uint8_t *slot = i < run.first_count ? run.first + uint64_t(i) * stride
                                                  : run.second + uint64_t(i - run.first_count) * stride;
        ugdr::queue::Cqe c;
        std::memcpy(&c, slot, sizeof(c));
        ugdr::api::cqe_to_wc(c, &wc[i]);
    }
    cq->ring.release(n);
    return int(n);
}

int ugdr_x_poll_cq_wait(ugdr_cq *cq, int min_entries, int max_entries, ugdr_wc *wc, uint64_t timeout_ns) noexcept {
    if (min_entries < 0 || max_entries < min_entries || (max_entries > 0 && wc == nullptr)) return -EINVAL;
    int got = 0;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(timeout_ns);
    for (uint32_t spins = 0;; ++spins) {
        const int k = ugdr_poll_cq(cq, max_entries - got, wc + got);
        if (k < 0) return k;
        got += k;
        if (got >= min_entries) return got;
        // The clock is read now and then; a pause keeps the polling core's sibling responsive.
        if ((spins & 255u) == 255u && std::chrono::steady_clock::now() >= deadline) return got;
#if defined(__x86_64__) || defined(__i386__)
        __builtin_ia32_pause();
#endif
    }
}

ugdr_qp *ugdr_create_qp(ugdr_pd *pd, ugdr_qp_init_attr *init) noexcept {
    if (!rt().live(pd) || init == nullptr || !rt().live(init->send_cq) || !rt().live(init->recv_cq))
        return fail_null<ugdr_qp>(EINVAL);
    try {
        Request req = make(kCreateQp, pd->identity);
        ByteWriter w(&req.opaque);
        w.be(init->send_cq->identity).be(init->recv_cq->identity).be(init->max_send_wr);
        w.be(init->max_recv_wr).be(init->max_send_sge).be(init->max_recv_sge);
        w.be(uint32_t(init->qp_type)).be(uint32_t(init->sq_sig_all));
        Response resp;
        if (int rc = rt().call(std::move(req), &resp); rc != 0) return fail_null<ugdr_qp>(rc);
        ByteReader rd(resp.opaque);
        uint32_t qpn = 0, msw = 0, mrw = 0, mss = 0, mrs = 0, sc = 0, ss = 0, rc_ = 0, rs = 0;
        if (!rd.be(&qpn) || !rd.be(&msw) || !rd.be(&mrw) || !rd.be(&mss) || !rd.be(&mrs) ||
            !rd.be(&sc) || !rd.be(&ss) || !rd.be(&rc_) || !rd.be(&rs) || resp.fds.size() != 2)
            return fail_null<ugdr_qp>(EPROTO);
        auto *qp = new ugdr_qp();
        int rc = ugdr::queue::Ring::attach(resp.fds[0].release(), {ugdr::queue::kSendRing, sc, ss}, &qp->sq);
        if (rc == 0)
            rc = ugdr::queue::Ring::attach(resp.fds[1].release(), {ugdr::queue::kRecvRing, rc_, rs}, &qp->rq);
        if (rc != 0) {
            Response ignored;
            rt().call(make(kDestroyQp, resp.identity), &ignored);
            delete qp;
            return fail_null<ugdr_qp>(rc);
        }
        qp->identity = resp.identity;
        qp->epoch = pd->epoch;
        qp->pd = pd;
        qp->qpn = qpn;
        qp->init = *init;
        qp->init.max_send_wr = msw;
        qp->init.max_recv_wr = mrw;
        qp->init.max_send_sge = mss;
        qp->init.max_recv_sge = mrs;
        return qp;
    } catch (...) {
        return fail_null<ugdr_qp>(ENOMEM);
    }
}

int ugdr_destroy_qp(ugdr_qp *qp) noexcept {
    if (!rt().live(qp)) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kDestroyQp, qp->identity), &resp); rc != 0) return rc;
    {
        std::lock_guard<ugdr::SpinLock> lk(qp->post_mu);
        qp->magic = kDead;
        qp->sq = ugdr::queue::Ring();
        qp->rq = ugdr::queue::Ring();
    }
    rt().retire(qp, qp);
    return 0;
}

int ugdr_modify_qp(ugdr_qp *qp, ugdr_qp_attr *attr, int attr_mask) noexcept {
    if (!rt().live(qp) || attr == nullptr) return EINVAL;
    Request req = make(kModifyQp, qp->identity);
    req.access = uint32_t(attr_mask);
    ByteWriter w(&req.opaque);
    put_attr(w, attr);
    Response resp;
    if (int rc = rt().call(std::move(req), &resp); rc != 0) return rc;
    if (attr->qp_state == UGDR_QPS_INIT) qp->access = attr->qp_access_flags;
    qp->state.store(attr->qp_state, std::memory_order_release);
    return 0;
}

int ugdr_query_qp(ugdr_qp *qp, ugdr_qp_attr *attr, int attr_mask, ugdr_qp_init_attr *init) noexcept {
    constexpr int known = UGDR_QP_STATE | UGDR_QP_CUR_STATE | UGDR_QP_ACCESS_FLAGS | UGDR_QP_TIMEOUT |
                          UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    if (!rt().live(qp) || attr == nullptr || init == nullptr || (attr_mask & ~known) != 0)
        return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kQueryQp, qp->identity), &resp); rc != 0) return rc;
    ByteReader rd(resp.opaque);
    uint32_t state = 0, access = 0, peer = 0;
    uint8_t to = 0, rc_ = 0, rnr = 0, mrt = 0;
    if (!rd.be(&state) || !rd.be(&access) || !rd.be(&to) || !rd.be(&rc_) || !rd.be(&rnr) ||
        !rd.be(&mrt) || !rd.be(&peer))
        return EPROTO;
    if (attr_mask & UGDR_QP_STATE) attr->qp_state = ugdr_qp_state(state);
    if (attr_mask & UGDR_QP_CUR_STATE) attr->cur_qp_state = ugdr_qp_state(state);
    if (attr_mask & UGDR_QP_ACCESS_FLAGS) attr->qp_access_flags = int(access);
    if (attr_mask & UGDR_QP_TIMEOUT) attr->timeout = to;
    if (attr_mask & UGDR_QP_RETRY_CNT) attr->retry_cnt = rc_;
    if (attr_mask & UGDR_QP_RNR_RETRY) attr->rnr_retry = rnr;
    if (attr_mask & UGDR_QP_MIN_RNR_TIMER) attr->min_rnr_timer = mrt;
    *init = qp->init;
    qp->state.store(int(state), std::memory_order_release);
    return 0;
}

int ugdr_query_qp_conn_info(ugdr_qp *qp, ugdr_qp_conn_info *info) noexcept {
    if (!rt().live(qp) || info == nullptr) return EINVAL;
    info->qp_num = qp->qpn;
    return 0;
}

int ugdr_connect_qp(ugdr_qp *qp, const ugdr_qp_conn_info *remote, const ugdr_qp_attr *attr,
                    int attr_mask) noexcept {
    if (!rt().live(qp) || remote == nullptr || attr == nullptr) return EINVAL;
    Request req = make(kConnectQp, qp->identity);
    req.access = uint32_t(attr_mask);
    ByteWriter w(&req.opaque);
    w.be(remote->qp_num);
    put_attr(w, attr);
    Response resp;
    if (int rc = rt().call(std::move(req), &resp); rc != 0) return rc;
    qp->timeout = attr->timeout;
    qp->retry_cnt = attr->retry_cnt;
    qp->rnr_retry = attr->rnr_retry;
    qp->min_rnr_timer = attr->min_rnr_timer;
    qp->state.store(UGDR_QPS_RTS, std::memory_order_release);
    return 0;
}

int ugdr_post_send(ugdr_qp *qp, ugdr_send_wr *wr, ugdr_send_wr **bad_wr) noexcept {
    if (qp == nullptr || qp->magic != kLive) {
        if (bad_wr) *bad_wr = wr;
        return EINVAL;
    }
    std::lock_guard<ugdr::SpinLock> lk(qp->post_mu);
    if (qp->magic != kLive || qp_state(qp) != UGDR_QPS_RTS) {
        if (bad_wr) *bad_wr = wr;
        return EINVAL;
    }
    return ugdr::api::post_send_chain(qp->sq, qp->init.max_send_sge, wr, bad_wr);
}

int ugdr_post_recv(ugdr_qp *qp, ugdr_recv_wr *wr, ugdr_recv_wr **bad_wr) noexcept {
    if (qp == nullptr || qp->magic != kLive) {
        if (bad_wr) *bad_wr = wr;
        return EINVAL;
    }
    std::lock_guard<ugdr::SpinLock> lk(qp->post_mu);
    const int st = qp_state(qp);
    if (qp->magic != kLive || (st != UGDR_QPS_INIT && st != UGDR_QPS_RTR && st != UGDR_QPS_RTS)) {
        if (bad_wr) *bad_wr = wr;
        return EINVAL;
    }
    return ugdr::api::post_recv_chain(qp->rq, qp->init.max_recv_sge, wr, bad_wr);
}

void *ugdr_x_alloc_host(size_t length) noexcept { return ugdr::api::host_alloc(length); }

int ugdr_x_free_host(void *address) noexcept { return ugdr::api::host_free(address); }

int ugdr_x_query_engine_stats(ugdr_context *ctx, ugdr_x_engine_stats *stats, int reset) noexcept {
    if (!rt().live(ctx) || stats == nullptr) return EINVAL;
    Request req = make(kEngineStats, ctx->identity);
    req.access = reset ? 1u : 0u;
    Response resp;
    if (int rc = rt().call(std::move(req), &resp); rc != 0) return rc;
    ByteReader rd(resp.opaque);
    if (!rd.be(&stats->wrs_completed) || !rd.be(&stats->bytes_moved) ||
        !rd.be(&stats->error_completions) || !rd.be(&stats->launches) ||
        !rd.be(&stats->wait_timeouts) || !rd.be(&stats->first_start_ns) || !rd.be(&stats->last_end_ns) ||
        !rd.be(&stats->chunks_run) || !rd.be(&stats->claim_misses) || !rd.be(&stats->jobs_published) ||
        !rd.be(&stats->inline_runs) || !rd.be(&stats->busy_ns) || !rd.be(&stats->fast_batches) ||
        !rd.be(&stats->fast_fetch_ns) || !rd.be(&stats->fast_exec_ns) || !rd.be(&stats->fast_reserve_ns) ||
        !rd.be(&stats->fast_publish_ns) || !rd.be(&stats->slow_wrs) || !rd.be(&stats->slow_issue_ns) ||
        !rd.be(&stats->job_slot_misses) || !rd.be(&stats->publish_waits) || !rd.be(&stats->publish_wait_ns) ||
        !rd.be(&stats->mr_detach_live) || !rd.be(&stats->mr_detach_quiesced) || !rd.be(&stats->order_waits) ||
        !rd.be(&stats->overlap_issues))
        return EPROTO;
    return 0;
}

int ugdr_x_query_qp_stats(ugdr_qp *qp, ugdr_x_qp_stats *stats) noexcept {
    if (!rt().live(qp) || stats == nullptr) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kQpStats, qp->identity), &resp); rc != 0) return rc;
    ByteReader rd(resp.opaque);
    if (!rd.be(&stats->send_posted) || !rd.be(&stats->send_retired) || !rd.be(&stats->recv_posted) ||
        !rd.be(&stats->recv_consumed) || !rd.be(&stats->bytes) || !rd.be(&stats->error_completions) ||
        !rd.be(&stats->rnr_waits) || !rd.be(&stats->state))
        return EPROTO;
    stats->reserved = 0;
    return 0;
}

int ugdr_x_engine_trace(ugdr_context *ctx, uint32_t records_per_cta) noexcept {
    if (!rt().live(ctx)) return EINVAL;
    Request req = make(kEngineTrace, ctx->identity);
    req.length = records_per_cta;
    req.access = 0;
    Response resp;
    return rt().call(std::move(req), &resp);
}

int ugdr_x_engine_trace_dump(ugdr_context *ctx, const char *path, uint64_t *kept, uint64_t *dropped) noexcept {
    if (!rt().live(ctx) || path == nullptr || path[0] == '\0') return EINVAL;
    try {
        Request req = make(kEngineTrace, ctx->identity);
        req.access = 1;
        const size_t n = std::strlen(path);
        req.opaque.resize(n);
        std::memcpy(req.opaque.data(), path, n);
        Response resp;
        if (int rc = rt().call(std::move(req), &resp); rc != 0) return rc;
        ByteReader rd(resp.opaque);
        uint64_t k = 0, d = 0;
        if (!rd.be(&k) || !rd.be(&d)) return EPROTO;
        if (kept) *kept = k;
        if (dropped) *dropped = d;
        return 0;
    } catch (...) {
        return ENOMEM;
    }
}

int ugdr_x_query_daemon_stats(ugdr_x_daemon_stats *stats) noexcept {
    if (stats == nullptr) return EINVAL;
    Response resp;
    if (int rc = rt().call(make(kDaemonStats), &resp); rc != 0) return rc;
    ByteReader rd(resp.opaque);
    if (!rd.be(&stats->devices) || !rd.be(&stats->contexts) || !rd.be(&stats->pds) || !rd.be(&stats->mrs) ||
        !rd.be(&stats->cqs) || !rd.be(&stats->qps))
        return EPROTO;
    return 0;
}

int ugdr_x_engine_hold(ugdr_context *ctx, int hold) noexcept {
    if (!rt().live(ctx)) return EINVAL;
    Request req = make(kEngineHold, ctx->identity);
    req.access = hold ? 1u : 0u;
    Response resp;
    return rt().call(std::move(req), &resp);
}

int ugdr_x_timed_drain(ugdr_context **contexts, int n, const uint64_t *expected, uint32_t timeout_ms,
                       float *elapsed_ms) noexcept {
    if (contexts == nullptr || expected == nullptr || elapsed_ms == nullptr || n <= 0) return EINVAL;
    Request req = make(kTimedDrain);
    req.length = timeout_ms;
    ByteWriter w(&req.opaque);
    w.be(uint32_t(n));
    for (int i = 0; i < n; ++i) {
        if (!rt().live(contexts[i])) return EINVAL;
        w.be(contexts[i]->identity).be(expected[i]);
    }
    Response resp;
    // The daemon answers at the latest `timeout_ms` after it starts the drain.
    const int rc = rt().call(std::move(req), &resp, uint64_t(timeout_ms) + 30000);
    ByteReader rd(resp.opaque);
    for (int i = 0; i < n; ++i) {
        uint32_t bits = 0;
        if (!rd.be(&bits)) break;
        std::memcpy(&elapsed_ms[i], &bits, 4);
    }
    return rc;
}

}  // extern "C"
