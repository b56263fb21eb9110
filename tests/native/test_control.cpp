// Control plane + CPU engine, driven in-process without sockets (reference suite semantics:
// tests/unit/device_context_test.cpp, pd_mr_cq_test.cpp, qp_test.cpp with a fake memory backend;
// loop_worker_test.cpp for execution; mock_worker_test.cpp for ERR flush).
#include "harness.hpp"

#include "api/posting.hpp"
#include "common/bytes.hpp"
#include "control/service.hpp"
#include "engine/cpu_engine.hpp"
#include "ugdr/api.hpp"

#include <unistd.h>

#include <cstring>
#include <map>
#include <set>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <vector>

using namespace ugdr;
using namespace ugdr::control;

namespace {

// Host-memory backend: maps the memfd the request carries (what the daemon does for host MRs).
class HostBackend : public MemoryBackend {
  public:
    int open(MemoryDescriptor &d, uint64_t len, OpenedMemory *out) override {
        if (d.kind != MemKind::host) return EOPNOTSUPP;
        if (int rc = map_shared_fd(d.region_fd.release(), 0, &out->host); rc != 0) return rc;
        out->address = static_cast<uint8_t *>(out->host.address) + d.region_offset;
        out->gpu = -1;
        (void)len;
        opens++;
        return 0;
    }
    void close(OpenedMemory &m) noexcept override {
        m.host.unmap();
        closes++;
    }
    int opens = 0, closes = 0;
};

struct Fixture {
    std::mutex mu;
    engine::CpuEngine eng{mu, false};
    HostBackend mem;
    ControlPlane cp{{&eng}, mem};
    uint64_t s = 1;

    Response call(uint32_t method, uint64_t id = 0, uint64_t length = 0, uint32_t access = 0,
                  std::vector<std::byte> opaque = {}, std::vector<Fd> fds = {}, uint64_t session = 0) {
        Request r;
        r.method = method;
        r.identity = id;
        r.length = length;
        r.access = access;
        r.opaque = std::move(opaque);
        r.fds = std::move(fds);
        return cp.dispatch(session ? session : s, std::move(r));
    }
    uint64_t ctx() { return call(kCreateContext, 1).identity; }
    uint64_t pd(uint64_t c) { return call(kCreatePd, c).identity; }
    Response cq(uint64_t c, uint32_t n) { return call(kCreateCq, c, n); }
    Response qp(uint64_t pd, uint64_t scq, uint64_t rcq, uint32_t depth = 16, uint32_t sge = 4, uint32_t sig_all = 0) {
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(scq).be(rcq).be(depth).be(depth).be(sge).be(sge).be(uint32_t(UGDR_QPT_RC)).be(sig_all);
        return call(kCreateQp, pd, 0, 0, std::move(o));
    }
    // Register `len` bytes at `off` of a fresh memfd region; returns (response, region).
    Response mr(uint64_t pd, SharedMapping *region, size_t bytes, uint64_t off, uint64_t len, uint32_t access) {
        if (region->address == nullptr) CHECK_EQ(create_shared_mapping("t", bytes, region), 0);
        std::vector<std::byte> o;
        ByteWriter w(&o);
        const uint8_t pad[3] = {0, 0, 0};
        w.be(uint8_t(MemKind::host)).raw(pad, 3).be(uint64_t(reinterpret_cast<uintptr_t>(region->address) + off));
        w.be(uint64_t(region->bytes)).be(off);
        std::vector<Fd> fds;
        fds.emplace_back(::dup(region->fd.get()));
        return call(kRegisterMr, pd, len, access, std::move(o), std::move(fds));
    }
    int modify(uint64_t q, uint32_t mask, uint32_t state, uint32_t access = 0, uint32_t cur = 0) {
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(state).be(cur).be(access).be(uint8_t(14)).be(uint8_t(7)).be(uint8_t(7)).be(uint8_t(12));
        return call(kModifyQp, q, 0, mask, std::move(o)).status;
    }
    int connect(uint64_t q, uint32_t remote, uint8_t rnr_retry = 7, uint32_t mask = 0, uint8_t min_rnr = 1) {
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(remote).be(uint32_t(0)).be(uint32_t(0)).be(uint32_t(0)).be(uint8_t(14)).be(uint8_t(7));
        w.be(rnr_retry).be(min_rnr);
        const uint32_t m = mask ? mask
                                : (UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER);
        return call(kConnectQp, q, 0, m, std::move(o)).status;
    }
};

uint32_t qpn_of(const Response &r) {
    ByteReader rd(r.opaque);
    uint32_t q = 0;
    rd.be(&q);
    return q;
}

struct Keys {
    uint32_t lkey = 0, rkey = 0;
};
Keys keys_of(const Response &r) {
    ByteReader rd(r.opaque);
    uint64_t a, l;
    Keys k;
    rd.be(&a);
    rd.be(&l);
    rd.be(&k.lkey);
    rd.be(&k.rkey);
    return k;
}

constexpr uint32_t kAllAccess = UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ |
                                UGDR_ACCESS_REMOTE_ATOMIC;
constexpr uint32_t kRemoteAll = UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ | UGDR_ACCESS_REMOTE_ATOMIC;

// A connected pair of QPs on one PD with one CQ, plus two 1 MiB host MRs.
struct Pair {
    Fixture f;
    uint64_t c, p, cq, qa, qb;
    uint32_t qpn_a, qpn_b;
    SharedMapping ra, rb;
    Keys ka, kb;
    uint64_t mra, mrb;
    Qp *a = nullptr, *b = nullptr;
    queue::Ring *sqa_client = nullptr;

    explicit Pair(uint8_t rnr_retry = 7, uint32_t sig_all = 0, uint32_t cq_depth = 64) {
        c = f.ctx();
        p = f.pd(c);
        Response cr = f.cq(c, cq_depth);
        cq = cr.identity;
        Response x = f.qp(p, cq, cq, 16, 4, sig_all), y = f.qp(p, cq, cq, 16, 4, sig_all);
        qa = x.identity;
        qb = y.identity;
        qpn_a = qpn_of(x);
        qpn_b = qpn_of(y);
        CHECK_EQ(f.modify(qa, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
        CHECK_EQ(f.modify(qb, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
        CHECK_EQ(f.connect(qa, qpn_b, rnr_retry), 0);
        CHECK_EQ(f.connect(qb, qpn_a, rnr_retry), 0);
        Response m1 = f.mr(p, &ra, 1 << 20, 0, 1 << 20, kAllAccess), m2 = f.mr(p, &rb, 1 << 20, 0, 1 << 20, kAllAccess);
        CHECK_EQ(m1.status, 0);
        ka = keys_of(m1);
        kb = keys_of(m2);
        mra = m1.identity;
        mrb = m2.identity;
    }
    uint8_t *A() { return static_cast<uint8_t *>(ra.address); }
    uint8_t *B() { return static_cast<uint8_t *>(rb.address); }
    uint64_t addrA(uint64_t off = 0) { return reinterpret_cast<uintptr_t>(ra.address) + off; }
    uint64_t addrB(uint64_t off = 0) { return reinterpret_cast<uintptr_t>(rb.address) + off; }
};

}  // namespace

TEST(control_devices_and_contexts) {
    Fixture f;
    Response l = f.call(kListDevices);
    ByteReader rd(l.opaque);
    uint32_t n = 0;
    rd.be(&n);
    CHECK_EQ(n, 1u);
    CHECK_EQ(f.call(kCreateContext, 7).status, ENODEV);
    const uint64_t c = f.ctx();
    CHECK(c != 0);
    CHECK_EQ(f.call(kDestroyContext, c, 0, 0, {}, {}, 2).status, EINVAL);  // foreign session
    const uint64_t p = f.pd(c);
    CHECK_EQ(f.call(kDestroyContext, c).status, EBUSY);
    CHECK_EQ(f.call(kDestroyPd, p).status, 0);
    CHECK_EQ(f.call(kDestroyPd, p).status, EINVAL);  // stale
    CHECK_EQ(f.call(kDestroyContext, c).status, 0);
    CHECK_EQ(f.cp.context_count(), 0u);
    CHECK_EQ(f.call(999).status, EOPNOTSUPP);
}

TEST(control_mr_validation_and_keys) {
    Fixture f;
    const uint64_t c = f.ctx(), p = f.pd(c);
    SharedMapping r;
    CHECK_EQ(f.mr(p, &r, 8192, 0, 0, UGDR_ACCESS_LOCAL_WRITE).status, EINVAL);           // zero length
    CHECK_EQ(f.mr(p, &r, 8192, 0, 64, UGDR_ACCESS_REMOTE_WRITE).status, EINVAL);         // remote write w/o local
    CHECK_EQ(f.mr(p, &r, 8192, 0, 64, 1u << 9).status, EINVAL);                          // unknown bit
    CHECK_EQ(f.mr(p, &r, 8192, 4096, 8192, UGDR_ACCESS_LOCAL_WRITE).status, EINVAL);     // past the region
    Response a = f.mr(p, &r, 8192, 0, 4096, kAllAccess), b = f.mr(p, &r, 8192, 4096, 4096, kAllAccess);
    CHECK_EQ(a.status, 0);
    Keys ka = keys_of(a), kb = keys_of(b);
    CHECK(ka.lkey != 0 && ka.rkey != 0 && ka.lkey != ka.rkey && ka.lkey != kb.lkey);
    CHECK_EQ(key_slot(ka.lkey), key_slot(ka.rkey));
    CHECK_EQ(f.call(kDestroyPd, p).status, EBUSY);
    CHECK_EQ(f.call(kDeregisterMr, a.identity).status, 0);
    CHECK_EQ(f.call(kDeregisterMr, a.identity).status, EINVAL);
    CHECK_EQ(f.mem.closes, 1);
    Response again = f.mr(p, &r, 8192, 0, 4096, kAllAccess);
    CHECK(keys_of(again).lkey != ka.lkey);  // reused slot gets a new generation
}

TEST(control_qp_create_and_state_machine) {
    Fixture f;
    const uint64_t c = f.ctx(), p = f.pd(c);
    const uint64_t cq = f.cq(c, 16).identity;
    CHECK_EQ(f.cq(c, 0).status, EINVAL);
    Response bad = f.qp(p, cq, cq, 0);
    CHECK_EQ(bad.status, EINVAL);
    Response q1 = f.qp(p, cq, cq), q2 = f.qp(p, cq, cq);
    CHECK_EQ(q1.status, 0);
    CHECK_EQ(q1.fds.size(), 2u);
    const uint32_t n1 = qpn_of(q1), n2 = qpn_of(q2);
    CHECK(n1 != 0 && n2 == n1 + 1);
    CHECK_EQ(f.call(kDestroyCq, cq).status, EBUSY);
    // INIT requires the access mask and a remote-only access value.
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE, UGDR_QPS_INIT), EINVAL);
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, UGDR_ACCESS_LOCAL_WRITE), EINVAL);
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE | UGDR_QP_CUR_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT,
                      UGDR_ACCESS_REMOTE_WRITE, UGDR_QPS_RTS),
             EINVAL);  // guard mismatch
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE, UGDR_QPS_SQD), EOPNOTSUPP);
    CHECK_EQ(f.modify(q1.identity, 1u << 30, UGDR_QPS_INIT), EINVAL);
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, UGDR_ACCESS_REMOTE_WRITE), 0);
    // connect precedence: mask, then local state, then remote existence.
    CHECK_EQ(f.connect(q1.identity, n2, 7, UGDR_QP_TIMEOUT), EINVAL);
    CHECK_EQ(f.connect(q1.identity, 9999), ENOENT);
    CHECK_EQ(f.connect(q1.identity, n2), EINVAL);  // remote still RESET
    CHECK_EQ(f.modify(q2.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, UGDR_ACCESS_REMOTE_WRITE), 0);
    CHECK_EQ(f.connect(q1.identity, n2), 0);
    CHECK_EQ(f.connect(q1.identity, n2), EINVAL);  // already RTS
    Response q3 = f.qp(p, cq, cq);
    CHECK_EQ(f.connect(q1.identity, qpn_of(q3)), EBUSY);  // bound to a different peer
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE, UGDR_QPS_ERR), 0);
    CHECK_EQ(f.modify(q1.identity, UGDR_QP_STATE, UGDR_QPS_ERR), EINVAL);  // ERR is terminal
    CHECK_EQ(f.call(kDestroyQp, q2.identity).status, 0);
    CHECK_EQ(f.connect(q3.identity, n2), EINVAL);  // q3 is RESET
    // Session reclaim takes everything down in dependency order.
    f.cp.on_disconnect(f.s);
    CHECK_EQ(f.cp.qp_count(), 0u);
    CHECK_EQ(f.cp.cq_count(), 0u);
    CHECK_EQ(f.cp.pd_count(), 0u);
    CHECK_EQ(f.cp.context_count(), 0u);
}

namespace {

int post_write(queue::Ring &sq, uint32_t op, uint64_t wr_id, std::vector<ugdr_sge> sges, uint64_t raddr,
               uint32_t rkey, bool signaled = true, uint32_t imm = 0, uint64_t cmp = 0, uint64_t swap = 0) {
    ugdr_send_wr wr{};
    wr.wr_id = wr_id;
    wr.sg_list = sges.data();
    wr.num_sge = int(sges.size());
    wr.opcode = ugdr_wr_opcode(op);
    wr.send_flags = signaled ? UGDR_SEND_SIGNALED : 0;
    wr.imm_data = imm;
    if (op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD) {
        wr.wr.atomic.remote_addr = raddr;
        wr.wr.atomic.rkey = rkey;
        wr.wr.atomic.compare_add = cmp;
        wr.wr.atomic.swap = swap;
    } else {
        wr.wr.rdma.remote_addr = raddr;
        wr.wr.rdma.rkey = rkey;
    }
    ugdr_send_wr *bad = nullptr;
    return api::post_send_chain(sq, 4, &wr, &bad);
}

}  // namespace

TEST(cpu_engine_write_read_atomics) {
    Pair t;
    // A second connected pair whose send ring this test attaches like a client would.
    Response qx = t.f.qp(t.p, t.cq, t.cq), qy = t.f.qp(t.p, t.cq, t.cq);
    CHECK_EQ(t.f.modify(qx.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
    CHECK_EQ(t.f.modify(qy.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
    CHECK_EQ(t.f.connect(qx.identity, qpn_of(qy)), 0);
    CHECK_EQ(t.f.connect(qy.identity, qpn_of(qx)), 0);
    queue::Ring sq, cq;
    CHECK_EQ(queue::Ring::attach(qx.fds[0].release(), {queue::kSendRing, 16, queue::send_stride(4)}, &sq), 0);
    for (int i = 0; i < 4096; ++i) t.A()[i] = uint8_t(i * 13 + 1);
    CHECK_EQ(post_write(sq, UGDR_WR_RDMA_WRITE, 1, {{t.addrA(), 1000, t.ka.lkey}}, t.addrB(64), t.kb.rkey), 0);
    CHECK_EQ(post_write(sq, UGDR_WR_RDMA_READ, 2, {{t.addrA(2048), 1000, t.ka.lkey}}, t.addrB(64), t.kb.rkey), 0);
    uint64_t v = 40;
    std::memcpy(t.B() + 4096, &v, 8);
    CHECK_EQ(post_write(sq, UGDR_WR_ATOMIC_FETCH_AND_ADD, 3, {{t.addrA(8192), 8, t.ka.lkey}}, t.addrB(4096),
                        t.kb.rkey, true, 0, 2),
             0);
    CHECK_EQ(post_write(sq, UGDR_WR_ATOMIC_CMP_AND_SWP, 4, {{t.addrA(8200), 8, t.ka.lkey}}, t.addrB(4096),
                        t.kb.rkey, true, 0, 42, 99),
             0);
    {
        std::lock_guard<std::mutex> lk(t.f.mu);
        CHECK_EQ(t.f.eng.progress_locked(), 4u);
    }
    CHECK(std::memcmp(t.B() + 64, t.A(), 1000) == 0);
    CHECK(std::memcmp(t.A() + 2048, t.A(), 1000) == 0);
    uint64_t r = 0, old1 = 0, old2 = 0;
    std::memcpy(&r, t.B() + 4096, 8);
    std::memcpy(&old1, t.A() + 8192, 8);
    std::memcpy(&old2, t.A() + 8200, 8);
    CHECK_EQ(old1, 40u);
    CHECK_EQ(old2, 42u);
    CHECK_EQ(r, 99u);
}

TEST(posting_prefix_bad_wr_and_full) {
    queue::Ring sq;
    CHECK_EQ(queue::Ring::create({queue::kSendRing, 3, queue::send_stride(2)}, &sq), 0);
    ugdr_sge sg{0x1000, 16, 5};
    ugdr_send_wr w[5]{};
    for (int i = 0; i < 5; ++i) {
        w[i].wr_id = uint64_t(i);
        w[i].sg_list = &sg;
        w[i].num_sge = 1;
        w[i].opcode = UGDR_WR_RDMA_WRITE;
        w[i].next = i + 1 < 5 ? &w[i + 1] : nullptr;
    }
    w[1].send_flags = 1u << 7;  // unknown flag: WR 1 invalid, WR 0 accepted
    ugdr_send_wr *bad = nullptr;
    CHECK_EQ(api::post_send_chain(sq, 2, &w[0], &bad), EINVAL);
    CHECK(bad == &w[1]);
    CHECK_EQ(sq.tail(), 1u);
    w[1].send_flags = 0;
    CHECK_EQ(api::post_send_chain(sq, 2, &w[1], &bad), ENOMEM);  // 2 more fit, then full
    CHECK(bad == &w[3]);
    CHECK_EQ(sq.tail(), 3u);
    // Slot contents: header + SGE at 40.
    queue::SendWqe h;
    std::memcpy(&h, sq.slot(0), sizeof(h));
    CHECK_EQ(h.wr_id, 0u);
    CHECK_EQ(h.sge_count, 1u);
    queue::Sge s;
    std::memcpy(&s, sq.slot(0) + 40, sizeof(s));
    CHECK_EQ(s.address, 0x1000u);
    CHECK_EQ(s.lkey, 5u);
    // Too many SGEs, negative count, atomic with two SGEs.
    queue::Ring sq2;
    CHECK_EQ(queue::Ring::create({queue::kSendRing, 8, queue::send_stride(2)}, &sq2), 0);
    ugdr_send_wr x{};
    x.sg_list = &sg;
    x.num_sge = 3;
    CHECK_EQ(api::post_send_chain(sq2, 2, &x, &bad), EINVAL);
    x.num_sge = -1;
    CHECK_EQ(api::post_send_chain(sq2, 2, &x, &bad), EINVAL);
    ugdr_sge two[2] = {sg, sg};
    x.sg_list = two;
    x.num_sge = 2;
    x.opcode = UGDR_WR_ATOMIC_FETCH_AND_ADD;
    CHECK_EQ(api::post_send_chain(sq2, 2, &x, &bad), EINVAL);
    x.opcode = ugdr_wr_opcode(3);  // SEND is not supported
    x.num_sge = 1;
    CHECK_EQ(api::post_send_chain(sq2, 2, &x, &bad), EINVAL);
    CHECK_EQ(sq2.tail(), 0u);
}

TEST(posting_atomic_layout_fits_one_slot) {
    queue::Ring sq;
    CHECK_EQ(queue::Ring::create({queue::kSendRing, 4, queue::send_stride(1)}, &sq), 0);
    CHECK_EQ(queue::send_stride(1), 64u);
    ugdr_sge sg{0x2000, 8, 9};
    ugdr_send_wr x{};
    x.wr_id = 77;
    x.sg_list = &sg;
    x.num_sge = 1;
    x.opcode = UGDR_WR_ATOMIC_CMP_AND_SWP;
    x.wr.atomic.remote_addr = 0x3000;
    x.wr.atomic.rkey = 11;
    x.wr.atomic.compare_add = 0x1122334455667788ull;
    x.wr.atomic.swap = 0xaabbccdd00112233ull;
    ugdr_send_wr *bad = nullptr;
    CHECK_EQ(api::post_send_chain(sq, 1, &x, &bad), 0);
    queue::SendWqe h;
    std::memcpy(&h, sq.slot(0), sizeof(h));
    CHECK_EQ(h.immediate_data, 0x00112233u);
    CHECK_EQ(h.reserved, 0xaabbccddu);
    uint64_t cmp = 0;
    std::memcpy(&cmp, sq.slot(0) + queue::kAtomicCompareOffset, 8);
    CHECK_EQ(cmp, 0x1122334455667788ull);
}

TEST(cqe_to_wc_fields) {
    queue::Cqe c{5, UGDR_WC_SUCCESS, UGDR_WC_RECV_RDMA_WITH_IMM, 100, 0x01020304, 9, UGDR_WC_WITH_IMM};
    ugdr_wc wc;
    api::cqe_to_wc(c, &wc);
    CHECK_EQ(wc.wr_id, 5u);
    CHECK_EQ(uint32_t(wc.opcode), uint32_t(UGDR_WC_RECV_RDMA_WITH_IMM));
    CHECK_EQ(wc.byte_len, 100u);
    CHECK_EQ(wc.imm_data, 0x01020304u);
    CHECK_EQ(wc.qp_num, 9u);
    CHECK_EQ(wc.wc_flags, unsigned(UGDR_WC_WITH_IMM));
    CHECK_EQ(wc.vendor_err, 0u);
}

// A client that bypasses the library and writes arbitrary bytes into its SQ ring must not crash
// the host engine or make it touch memory outside registered ranges: every WQE either runs
// inside an MR, or fails with an error completion that moves the QP to ERR.
TEST(cpu_engine_survives_garbage_wqes) {
    Fixture f;
    const uint64_t c = f.ctx(), p = f.pd(c);
    const uint64_t cq = f.cq(c, 8192).identity;
    SharedMapping region;
    constexpr size_t kRegion = 512 << 10, kOff = 64 << 10, kLen = 256 << 10;
    Response m = f.mr(p, &region, kRegion, kOff, kLen, kAllAccess);
    CHECK_EQ(m.status, 0);
    const Keys k = keys_of(m);
    uint8_t *base = static_cast<uint8_t *>(region.address);
    for (size_t i = 0; i < kRegion; ++i) base[i] = uint8_t(i * 7 + 3);
    std::vector<uint8_t> before(base, base + kRegion);
    const uint64_t lo = reinterpret_cast<uintptr_t>(base) + kOff;
    std::mt19937_64 rng(5);
    auto pick_addr = [&]() -> uint64_t {
        switch (rng() % 4) {
        case 0: return lo + rng() % kLen;                  // inside the MR
        case 1: return lo + kLen - rng() % 64;             // at its end
        case 2: return reinterpret_cast<uintptr_t>(base) + rng() % kRegion;  // possibly outside
        default: return rng();                              // anywhere
        }
    };
    auto pick_key = [&](uint32_t good) -> uint32_t { return rng() % 4 ? good : uint32_t(rng()); };
    const uint32_t stride = queue::send_stride(4);
    for (int iter = 0; iter < 200; ++iter) {
        Response qx = f.qp(p, cq, cq), qy = f.qp(p, cq, cq);
        CHECK_EQ(f.modify(qx.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
        CHECK_EQ(f.modify(qy.identity, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, UGDR_QPS_INIT, kRemoteAll), 0);
        CHECK_EQ(f.connect(qx.identity, qpn_of(qy)), 0);
        CHECK_EQ(f.connect(qy.identity, qpn_of(qx)), 0);
        queue::Ring sq;
        CHECK_EQ(queue::Ring::attach(qx.fds[0].release(), {queue::kSendRing, 16, stride}, &sq), 0);
        queue::SlotRun run = sq.reserve(8);
        CHECK_EQ(run.count(), 8u);
        for (uint32_t i = 0; i < run.count(); ++i) {
            uint8_t *slot = i < run.first_count ? run.first + uint64_t(i) * stride
                                                : run.second + uint64_t(i - run.first_count) * stride;
            for (uint32_t b = 0; b < stride; ++b) slot[b] = uint8_t(rng());
            if (rng() % 8 == 0) continue;  // pure noise
            queue::SendWqe h;
            std::memcpy(&h, slot, sizeof(h));
            const uint32_t ops[] = {UGDR_WR_RDMA_WRITE, UGDR_WR_RDMA_READ, UGDR_WR_ATOMIC_FETCH_AND_ADD,
                                    UGDR_WR_ATOMIC_CMP_AND_SWP, uint32_t(rng())};
            h.opcode = ops[rng() % 5];
            h.sge_count = uint32_t(rng() % 6);
            h.send_flags = UGDR_SEND_SIGNALED;
            h.remote_address = pick_addr();
            h.rkey = pick_key(k.rkey);
            std::memcpy(slot, &h, sizeof(h));
            for (uint32_t s = 0; s < h.sge_count && s < 4; ++s) {
                queue::Sge sg{pick_addr(), uint32_t(rng() % 3 ? rng() % 4096 : rng()), pick_key(k.lkey)};
                if (h.opcode == UGDR_WR_ATOMIC_FETCH_AND_ADD || h.opcode == UGDR_WR_ATOMIC_CMP_AND_SWP)
                    sg.length = rng() % 4 ? 8 : sg.length;
                std::memcpy(slot + queue::kSendSgeOffset + s * sizeof(queue::Sge), &sg, sizeof(sg));
            }
        }
        sq.publish(run.count());
        {
            std::lock_guard<std::mutex> lk(f.mu);
            for (int k2 = 0; k2 < 16; ++k2) f.eng.progress_locked();
        }
        CHECK_EQ(f.call(kDestroyQp, qx.identity).status, 0);
        CHECK_EQ(f.call(kDestroyQp, qy.identity).status, 0);
    }
    // Bytes outside the registered range were never written.
    CHECK(std::memcmp(base, before.data(), kOff) == 0);
    CHECK(std::memcmp(base + kOff + kLen, before.data() + kOff + kLen, kRegion - kOff - kLen) == 0);
}

namespace {

// An engine that records the calls the control plane makes, for ordering checks.
class RecordingEngine : public Engine {
  public:
    RecordingEngine(std::vector<std::string> *log, std::string name, bool live = false, bool settles = true)
        : log_(log), name_(std::move(name)), live_(live), settles_(settles) {}
    bool detaches_live() const noexcept override { return live_; }
    bool settle() noexcept override {
        log_->push_back(name_ + ".settle");
        return settles_;
    }
    DeviceInfo info() const override {
        DeviceInfo d;
        d.name = name_;
        d.kind = DeviceKind::gpu;
        return d;
    }
    int attach_mr(Mr &) override { return 0; }
    void detach_mr(Mr &) noexcept override {}
    int attach_cq(Cq &) override { return 0; }
    void detach_cq(Cq &) noexcept override {}
    int attach_qp(Qp &) override { return 0; }
    void update_qp(Qp &q) override { log_->push_back(name_ + ".update_qp(" + std::to_string(q.qpn) + ")"); }
    void detach_qp(Qp &q) noexcept override { log_->push_back(name_ + ".detach_qp(" + std::to_string(q.qpn) + ")"); }
    void quiesce() override { log_->push_back(name_ + ".quiesce"); }
    void resume() override { log_->push_back(name_ + ".resume"); }
    int stats(EngineStats *, bool) override { return 0; }
    int hold(bool) override { return 0; }

  private:
    std::vector<std::string> *log_;
    std::string name_;
    bool live_ = false, settles_ = true;
};

}  // namespace

TEST(control_destroying_a_qp_stops_its_peers_engine_first) {
    // QP a on GPU engine 1 is bound to QP b on GPU engine 2.  Destroying b must stop engine 1
    // (which may be writing into b's receive ring), unbind a, drop b from engine 2, then let
    // engine 1 run again.
    std::vector<std::string> log;
    RecordingEngine e1(&log, "e1"), e2(&log, "e2");
    HostBackend mem;
    ControlPlane cp{{&e1, &e2}, mem};
    auto call = [&](uint32_t method, uint64_t id, uint64_t length = 0, uint32_t access = 0,
                    std::vector<std::byte> opaque = {}) {
        Request r;
        r.method = method;
        r.identity = id;
        r.length = length;
        r.access = access;
        r.opaque = std::move(opaque);
        return cp.dispatch(1, std::move(r));
    };
    uint64_t qp[2];
    uint32_t qpn[2];
    for (int i = 0; i < 2; ++i) {
        const uint64_t ctx = call(kCreateContext, uint64_t(i + 1)).identity;
        const uint64_t pd = call(kCreatePd, ctx).identity;
        const uint64_t cq = call(kCreateCq, ctx, 16).identity;
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(cq).be(cq).be(uint32_t(16)).be(uint32_t(16)).be(uint32_t(1)).be(uint32_t(1)).be(uint32_t(UGDR_QPT_RC));
        w.be(uint32_t(0));
        Response q = call(kCreateQp, pd, 0, 0, std::move(o));
        CHECK_EQ(q.status, 0);
        qp[i] = q.identity;
        qpn[i] = qpn_of(q);
        std::vector<std::byte> m;
        ByteWriter mw(&m);
        mw.be(uint32_t(UGDR_QPS_INIT)).be(uint32_t(0)).be(uint32_t(UGDR_ACCESS_REMOTE_WRITE));
        mw.be(uint8_t(14)).be(uint8_t(7)).be(uint8_t(7)).be(uint8_t(12));
        CHECK_EQ(call(kModifyQp, qp[i], 0, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, std::move(m)).status, 0);
    }
    for (int i = 0; i < 2; ++i) {
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(qpn[1 - i]).be(uint32_t(0)).be(uint32_t(0)).be(uint32_t(0)).be(uint8_t(14)).be(uint8_t(7));
        w.be(uint8_t(7)).be(uint8_t(1));
        CHECK_EQ(call(kConnectQp, qp[i], 0,
                      UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER, std::move(o))
                     .status,
                 0);
    }
    log.clear();
    CHECK_EQ(call(kDestroyQp, qp[1]).status, 0);
    const std::vector<std::string> want = {"e1.quiesce", "e1.update_qp(" + std::to_string(qpn[0]) + ")",
                                           "e2.detach_qp(" + std::to_string(qpn[1]) + ")", "e1.resume"};
    CHECK(log == want);
    if (log != want)
        for (const std::string &l : log) std::fprintf(stderr, "    got %s\n", l.c_str());
}

namespace {

// QP b on engine 2 has two requesters: a on engine 1 and c on engine 2, and both engines detach
// live.  Destroying b unbinds a and c while their engines run; engine 1 (whose kernel engine 2's
// idle point does not cover) then settles, or is stopped when it cannot; engine 2 never stops.
std::vector<std::string> destroy_shared_responder(bool e1_settles, uint32_t qpn_out[3]) {
    std::vector<std::string> log;
    RecordingEngine e1(&log, "e1", true, e1_settles), e2(&log, "e2", true);
    HostBackend mem;
    ControlPlane cp{{&e1, &e2}, mem};
    auto call = [&](uint32_t method, uint64_t id, uint64_t length = 0, uint32_t access = 0,
                    std::vector<std::byte> opaque = {}) {
        Request r;
        r.method = method;
        r.identity = id;
        r.length = length;
        r.access = access;
        r.opaque = std::move(opaque);
        return cp.dispatch(1, std::move(r));
    };
    const int device_of[3] = {1, 2, 2};  // a, b, c
    uint64_t qp[3];
    uint32_t qpn[3];
    for (int i = 0; i < 3; ++i) {
        const uint64_t ctx = call(kCreateContext, uint64_t(device_of[i])).identity;
        const uint64_t pd = call(kCreatePd, ctx).identity;
        const uint64_t cq = call(kCreateCq, ctx, 16).identity;
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(cq).be(cq).be(uint32_t(16)).be(uint32_t(16)).be(uint32_t(1)).be(uint32_t(1)).be(uint32_t(UGDR_QPT_RC));
        w.be(uint32_t(0));
        Response q = call(kCreateQp, pd, 0, 0, std::move(o));
        CHECK_EQ(q.status, 0);
        qp[i] = q.identity;
        qpn[i] = qpn_of(q);
        std::vector<std::byte> m;
        ByteWriter mw(&m);
        mw.be(uint32_t(UGDR_QPS_INIT)).be(uint32_t(0)).be(uint32_t(UGDR_ACCESS_REMOTE_WRITE));
        mw.be(uint8_t(14)).be(uint8_t(7)).be(uint8_t(7)).be(uint8_t(12));
        CHECK_EQ(call(kModifyQp, qp[i], 0, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, std::move(m)).status, 0);
    }
    const int target[3] = {1, 0, 1};  // a -> b, b -> a, c -> b
    for (int i = 0; i < 3; ++i) {
        std::vector<std::byte> o;
        ByteWriter w(&o);
        w.be(qpn[target[i]]).be(uint32_t(0)).be(uint32_t(0)).be(uint32_t(0)).be(uint8_t(14)).be(uint8_t(7));
        w.be(uint8_t(7)).be(uint8_t(1));
        CHECK_EQ(call(kConnectQp, qp[i], 0,
                      UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER, std::move(o))
                     .status,
                 0);
    }
    log.clear();
    CHECK_EQ(call(kDestroyQp, qp[1]).status, 0);
    for (int i = 0; i < 3; ++i) qpn_out[i] = qpn[i];
    std::vector<std::string> out = log;  // the teardown below logs more
    return out;
}

}  // namespace

TEST(control_live_detach_settles_other_engines_instead_of_stopping_them) {
    uint32_t qpn[3];
    const std::vector<std::string> log = destroy_shared_responder(true, qpn);
    const std::vector<std::string> want = {"e1.update_qp(" + std::to_string(qpn[0]) + ")",
                                           "e2.update_qp(" + std::to_string(qpn[2]) + ")", "e1.settle",
                                           "e2.detach_qp(" + std::to_string(qpn[1]) + ")"};
    CHECK(log == want);
    if (log != want)
        for (const std::string &l : log) std::fprintf(stderr, "    got %s\n", l.c_str());
}

TEST(control_live_detach_stops_an_engine_that_does_not_settle) {
    uint32_t qpn[3];
    const std::vector<std::string> log = destroy_shared_responder(false, qpn);
    const std::vector<std::string> want = {"e1.update_qp(" + std::to_string(qpn[0]) + ")",
                                           "e2.update_qp(" + std::to_string(qpn[2]) + ")", "e1.settle",
                                           "e1.quiesce", "e2.detach_qp(" + std::to_string(qpn[1]) + ")",
                                           "e1.resume"};
    CHECK(log == want);
    if (log != want)
        for (const std::string &l : log) std::fprintf(stderr, "    got %s\n", l.c_str());
}

namespace {

// An engine that checks, call by call, what the control plane asks of it during random
// create / connect / destroy sequences: no call names a QP it already detached, stops and resumes
// pair up, and when a QP is detached no QP still bound to it is left on any engine.
struct Bindings {
    std::map<uint32_t, uint32_t> peer_of;  // live QP -> the QPN it is bound to (0: none)
    std::set<uint32_t> detached;
    int violations = 0;
};

class CheckingEngine : public Engine {
  public:
    CheckingEngine(Bindings *b, bool live, bool settles) : b_(b), live_(live), settles_(settles) {}
    DeviceInfo info() const override {
        DeviceInfo d;
        d.name = "checking";
        d.kind = DeviceKind::gpu;
        return d;
    }
    int attach_mr(Mr &) override { return 0; }
    void detach_mr(Mr &) noexcept override {}
    int attach_cq(Cq &) override { return 0; }
    void detach_cq(Cq &) noexcept override {}
    int attach_qp(Qp &q) override {
        b_->peer_of[q.qpn] = 0;
        return 0;
    }
    void update_qp(Qp &q) override {
        if (b_->detached.count(q.qpn)) ++b_->violations;
        b_->peer_of[q.qpn] = q.peer != nullptr ? q.peer->qpn : 0;
    }
    void detach_qp(Qp &q) noexcept override {
        if (b_->detached.count(q.qpn)) ++b_->violations;
        for (const auto &[qpn, peer] : b_->peer_of)
            if (peer == q.qpn && qpn != q.qpn) ++b_->violations;  // a requester still bound to it
        b_->peer_of.erase(q.qpn);
        b_->detached.insert(q.qpn);
    }
    void quiesce() override { ++depth; }
    void resume() override {
        if (--depth < 0) ++b_->violations;
    }
    bool detaches_live() const noexcept override { return live_; }
    bool settle() noexcept override { return settles_; }
    int stats(EngineStats *, bool) override { return 0; }
    int hold(bool) override { return 0; }
    int depth = 0;

  private:
    Bindings *b_;
    bool live_, settles_;
};

}  // namespace

TEST(control_random_qp_lifecycles_never_leave_a_dangling_binding) {
    for (uint32_t seed = 1; seed <= 40; ++seed) {
        std::mt19937 rng(seed);
        Bindings b;
        CheckingEngine e1(&b, rng() % 2 == 0, rng() % 2 == 0), e2(&b, rng() % 2 == 0, rng() % 2 == 0);
        HostBackend mem;
        ControlPlane cp{{&e1, &e2}, mem};
        auto call = [&](uint32_t method, uint64_t id, uint64_t length = 0, uint32_t access = 0,
                        std::vector<std::byte> opaque = {}) {
            Request r;
            r.method = method;
            r.identity = id;
            r.length = length;
            r.access = access;
            r.opaque = std::move(opaque);
            return cp.dispatch(1, std::move(r));
        };
        uint64_t pd[2], cq[2];
        for (int d = 0; d < 2; ++d) {
            const uint64_t ctx = call(kCreateContext, uint64_t(d + 1)).identity;
            pd[d] = call(kCreatePd, ctx).identity;
            cq[d] = call(kCreateCq, ctx, 64).identity;
        }
        struct Live {
            uint64_t id;
            uint32_t qpn;
            bool connected;
        };
        std::vector<Live> qps;
        for (int op = 0; op < 60; ++op) {
            const uint32_t what = rng() % 3;
            if (what == 0 || qps.size() < 2) {  // create (and move to INIT) on a random engine
                const int d = int(rng() % 2);
                std::vector<std::byte> o;
                ByteWriter w(&o);
                w.be(cq[d]).be(cq[d]).be(uint32_t(8)).be(uint32_t(8)).be(uint32_t(1)).be(uint32_t(1));
                w.be(uint32_t(UGDR_QPT_RC)).be(uint32_t(0));
                Response q = call(kCreateQp, pd[d], 0, 0, std::move(o));
                CHECK_EQ(q.status, 0);
                std::vector<std::byte> m;
                ByteWriter mw(&m);
                mw.be(uint32_t(UGDR_QPS_INIT)).be(uint32_t(0)).be(uint32_t(UGDR_ACCESS_REMOTE_WRITE));
                mw.be(uint8_t(14)).be(uint8_t(7)).be(uint8_t(7)).be(uint8_t(12));
                CHECK_EQ(call(kModifyQp, q.identity, 0, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, std::move(m)).status, 0);
                qps.push_back({q.identity, qpn_of(q), false});
            } else if (what == 1) {  // connect an unconnected QP to any live QP
                Live &x = qps[rng() % qps.size()];
                const Live &y = qps[rng() % qps.size()];
                if (x.connected) continue;
                std::vector<std::byte> o;
                ByteWriter w(&o);
                w.be(y.qpn).be(uint32_t(0)).be(uint32_t(0)).be(uint32_t(0)).be(uint8_t(14)).be(uint8_t(7));
                w.be(uint8_t(7)).be(uint8_t(1));
                const int rc = call(kConnectQp, x.id, 0,
                                    UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER,
                                    std::move(o))
                                   .status;
                if (rc == 0) x.connected = true;
            } else {  // destroy a random QP
                const size_t i = rng() % qps.size();
                CHECK_EQ(call(kDestroyQp, qps[i].id).status, 0);
                qps.erase(qps.begin() + long(i));
            }
            CHECK_EQ(e1.depth, 0);
            CHECK_EQ(e2.depth, 0);
        }
        CHECK_EQ(b.violations, 0);
        if (b.violations != 0) std::fprintf(stderr, "    seed %u: %d violations\n", seed, b.violations);
    }
}
