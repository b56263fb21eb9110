#include "engine/cpu_engine.hpp"

#include "control/service.hpp"
#include "engine/semantics.hpp"
#include "queue/layout.hpp"

#include <chrono>
#include <cstring>
#include <time.h>

namespace ugdr::engine {
namespace {

uint64_t now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return uint64_t(ts.tv_sec) * 1000000000ull + uint64_t(ts.tv_nsec);
}

inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

// Payload copy.  Short segments (descriptor-sized WRs, gathers of a few bytes each) skip the
// library call: up to 16 bytes move as two possibly overlapping 8-byte words, or bytewise.
inline void copy_bytes(uint8_t *dst, const uint8_t *src, uint32_t n) {
    if (n >= 8 && n <= 16) {
        uint64_t a, b;
        std::memcpy(&a, src, 8);
        std::memcpy(&b, src + n - 8, 8);
        std::memcpy(dst, &a, 8);
        std::memcpy(dst + n - 8, &b, 8);
    } else if (n < 8) {
        for (uint32_t i = 0; i < n; ++i) dst[i] = src[i];
    } else {
        std::memcpy(dst, src, n);
    }
}

struct Seg {
    uint8_t *local;
    uint32_t length;
};

}  // namespace

CpuEngine::CpuEngine(std::mutex &objects_mu, bool start_thread) : objects_mu_(objects_mu) {
    if (start_thread) worker_ = std::thread([this] { run(); });
}

CpuEngine::~CpuEngine() {
    stop_.store(true);
    if (worker_.joinable()) worker_.join();
}

control::DeviceInfo CpuEngine::info() const {
    control::DeviceInfo d;
    d.name = "ugdr_cpu0";
    d.kind = control::DeviceKind::cpu;
    return d;
}

int CpuEngine::attach_mr(control::Mr &mr) {
    MrView v;
    if (mr.mem.gpu == -1 && !mr.mem.multicast) v.base = static_cast<uint8_t *>(mr.mem.address);  // host only
    v.client_base = mr.client_address;
    v.length = mr.length;
    v.access = mr.access;
    v.pd_num = mr.pd_num;
    v.lkey = mr.lkey;
    v.rkey = mr.rkey;
    mrs_[mr.table_slot] = v;
    return 0;
}

void CpuEngine::detach_mr(control::Mr &mr) noexcept {
    mrs_.erase(mr.table_slot);
    for (QpView &v : qps_) v.lm = v.rm = nullptr;
}

int CpuEngine::attach_cq(control::Cq &) { return 0; }
void CpuEngine::detach_cq(control::Cq &) noexcept {}

int CpuEngine::attach_qp(control::Qp &qp) {
    QpView v;
    v.qp = &qp;
    qps_.push_back(v);
    return 0;
}

void CpuEngine::update_qp(control::Qp &qp) {
    for (QpView &v : qps_)
        if (v.qp == &qp) v.rnr_attempts = 0;
}

void CpuEngine::detach_qp(control::Qp &qp) noexcept {
    for (size_t i = 0; i < qps_.size(); ++i) {
        if (qps_[i].qp == &qp) {
            qps_[i] = qps_.back();
            qps_.pop_back();
            return;
        }
    }
}

int CpuEngine::stats(control::EngineStats *out, bool reset) {
    *out = stats_;
    if (reset) stats_ = control::EngineStats{};
    return 0;
}

int CpuEngine::qp_counters(control::Qp &qp, control::QpCounters *out) {
    for (const QpView &v : qps_) {
        if (v.qp == &qp) {
            *out = v.c;
            return 0;
        }
    }
    return ENOENT;
}

int CpuEngine::hold(bool on) {
    held_.store(on);
    return 0;
}

const CpuEngine::MrView *CpuEngine::find(uint32_t key, bool remote) const {
    auto it = mrs_.find(control::key_slot(key));
    if (it == mrs_.end()) return nullptr;
    if ((remote ? it->second.rkey : it->second.lkey) != key) return nullptr;
    return &it->second;
}

const CpuEngine::MrView *CpuEngine::find_cached(QpView &v, uint32_t key, bool remote) const {
    const MrView *&slot = remote ? v.rm : v.lm;
    uint32_t &cached = remote ? v.rkey : v.lkey;
    if (slot != nullptr && cached == key) return slot;
    const MrView *m = find(key, remote);
    if (m != nullptr) {
        slot = m;
        cached = key;
    }
    return m;
}

bool CpuEngine::produce(control::Cq *cq, const void *cqe) {
    queue::SlotRun run = cq->ring.reserve(1);
    if (run.count() == 0) return false;
    std::memcpy(run.first, cqe, sizeof(queue::Cqe));
    cq->ring.publish(1);
    return true;
}

void CpuEngine::enter_error(control::Qp &qp) {
    qp.state = UGDR_QPS_ERR;
    qp.sq.set_error_word(UGDR_QPS_ERR);
}

uint8_t *CpuEngine::resolve(const MrView *m, uint64_t addr, uint64_t len) {
    if (m == nullptr || m->base == nullptr || addr < m->client_base || len > m->length ||
        addr - m->client_base > m->length - len)
        return nullptr;
    return m->base + (addr - m->client_base);
}

size_t CpuEngine::progress_qp(QpView &v) {
    control::Qp &qp = *v.qp;
    size_t retired = 0;
    if (qp.state == UGDR_QPS_ERR) {
        // Flush: one FLUSH_ERR per outstanding SQ and RQ WR, signaled or not.
        for (;;) {
            queue::SlotRun run = qp.sq.peek(1);
            if (run.count() == 0) break;
            queue::SendWqe h;
            std::memcpy(&h, run.first, sizeof(h));
            queue::Cqe c{h.wr_id, UGDR_WC_WR_FLUSH_ERR, wc_opcode(h.opcode), 0, 0, qp.qpn, 0};
            if (qp.send_cq->ring.reserve(1).count() == 0) break;
            qp.sq.release(1);  // the slot is free before its completion is visible
            produce(qp.send_cq, &c);
            stats_.error_completions += 1;
            v.c.error_completions += 1;
            ++retired;
        }
        for (;;) {
            queue::SlotRun run = qp.rq.peek(1);
            if (run.count() == 0) break;
            queue::RecvWqe h;
            std::memcpy(&h, run.first, sizeof(h));
            queue::Cqe c{h.wr_id, UGDR_WC_WR_FLUSH_ERR, UGDR_WC_RECV_RDMA_WITH_IMM, 0, 0, qp.qpn, 0};
            if (qp.recv_cq->ring.reserve(1).count() == 0) break;
            qp.rq.release(1);
            produce(qp.recv_cq, &c);
            stats_.error_completions += 1;
            v.c.error_completions += 1;
        }
        return retired;
    }
    if (qp.state != UGDR_QPS_RTS) return 0;

    // One batch per pass: the SQ slots are peeked together, send-CQ slots reserved together, and
    // both cursors move once at the end (SQ head first, then the CQ tail), so the client's
    // polled cache lines are written once per batch instead of once per WR.
    const queue::SlotRun run = qp.sq.peek(64);
    const uint32_t k = run.count();
    if (k == 0) return 0;
    const uint32_t sq_stride = qp.sq.geometry().stride;
    queue::Ring &scq = qp.send_cq->ring;
    const uint32_t cq_stride = scq.geometry().stride;
    queue::SlotRun cq_run = scq.reserve(k);
    uint32_t consumed = 0, ncqe = 0;
    auto cq_slot = [&](uint32_t j) {
        return j < cq_run.first_count ? cq_run.first + j * cq_stride : cq_run.second + (j - cq_run.first_count) * cq_stride;
    };
    auto finish = [&]() {  // SQ slots back before their completions become visible
        qp.sq.release(consumed);
        scq.publish(ncqe);
        ncqe = 0;
    };
    for (uint32_t i = 0; i < k; ++i) {
        const uint8_t *slot = i < run.first_count ? run.first + i * sq_stride : run.second + (i - run.first_count) * sq_stride;
        queue::SendWqe h;
        std::memcpy(&h, slot, sizeof(h));
        const uint32_t op = h.opcode;
        const bool signaled = qp.sq_sig_all || (h.send_flags & UGDR_SEND_SIGNALED) != 0;
        uint32_t status = UGDR_WC_SUCCESS;
        uint64_t total = 0;
        Seg segs[32];
        uint32_t nseg = 0;

        if (!op_known(op) || h.sge_count > qp.caps.max_send_sge || h.sge_count > 32 ||
            (op_atomic(op) && h.sge_count != 1))
            status = UGDR_WC_LOC_QP_OP_ERR;
        for (uint32_t i = 0; status == UGDR_WC_SUCCESS && i < h.sge_count; ++i) {
            queue::Sge sg;
            std::memcpy(&sg, slot + queue::kSendSgeOffset + i * sizeof(queue::Sge), sizeof(sg));
            total += sg.length;
            if (total > 0xffffffffull) {  // byte_len is 32 bits: up to 4 GiB - 1 per WR
                status = UGDR_WC_LOC_LEN_ERR;
                break;
            }
            if (sg.length == 0) continue;
            const MrView *m = find_cached(v, sg.lkey, false);
            uint8_t *p = (m != nullptr && m->pd_num == qp.pd_num) ? resolve(m, sg.address, sg.length)
                                                                   : nullptr;
            if (p == nullptr || (local_written(op) && (m->access & UGDR_ACCESS_LOCAL_WRITE) == 0)) {
                status = UGDR_WC_LOC_PROT_ERR;
                break;
            }
            segs[nseg++] = Seg{p, sg.length};
        }
        if (status == UGDR_WC_SUCCESS && op_atomic(op) && total != 8) status = UGDR_WC_LOC_LEN_ERR;
        if (status == UGDR_WC_SUCCESS && op_sum(op) && h.sge_count > 0) {
            // Every SGE has the same even length L; the WR moves L bytes.
            queue::Sge first;
            std::memcpy(&first, slot + queue::kSendSgeOffset, sizeof(first));
            for (uint32_t i = 0; i < h.sge_count && status == UGDR_WC_SUCCESS; ++i) {
                queue::Sge sg;
                std::memcpy(&sg, slot + queue::kSendSgeOffset + i * sizeof(queue::Sge), sizeof(sg));
                if (sg.length != first.length || (sg.length & 1u) != 0) status = UGDR_WC_LOC_LEN_ERR;
                else if ((sg.address & 1u) != 0) status = UGDR_WC_LOC_PROT_ERR;
            }
            total = first.length;
        }

        control::Qp *peer = qp.peer;
        uint8_t *remote = nullptr;
        if (status == UGDR_WC_SUCCESS) {
            if (peer == nullptr || qp.peer_lost || peer->state == UGDR_QPS_RESET) {
                status = UGDR_WC_RETRY_EXC_ERR;
            } else if (peer->state == UGDR_QPS_ERR) {
                status = UGDR_WC_REM_OP_ERR;
            } else {
                const uint32_t need = remote_access_for(op);
                const MrView *m = find_cached(v, h.rkey, true);
                if (total != 0 || op_atomic(op)) {
                    remote = (m != nullptr && m->pd_num == peer->pd_num && (m->access & need) != 0 &&
                              (peer->access & need) != 0)
                                 ? resolve(m, h.remote_address, op_atomic(op) ? 8 : total)
                                 : nullptr;
                    if (remote == nullptr) status = UGDR_WC_REM_ACCESS_ERR;
                } else if ((peer->access & need) == 0) {
                    status = UGDR_WC_REM_ACCESS_ERR;
                }
                if (status == UGDR_WC_SUCCESS && op_atomic(op) && (h.remote_address & 7) != 0)
                    status = UGDR_WC_REM_INV_REQ_ERR;
                if (status == UGDR_WC_SUCCESS && op_sum(op) && (h.remote_address & 1) != 0)
                    status = UGDR_WC_REM_INV_REQ_ERR;
            }
        }

        // Responder resources for WRITE_WITH_IMM: one RQ WR and one recv-CQ slot.
        uint64_t recv_wr_id = 0;
        if (status == UGDR_WC_SUCCESS && op == UGDR_WR_RDMA_WRITE_WITH_IMM) {
            queue::SlotRun rq = peer->rq.peek(1);
            if (rq.count() == 0) {
                if (!v.rnr_waiting) {
                    v.rnr_waiting = true;
                    v.c.rnr_waits += 1;
                }
                if (qp.rnr_retry == kInfiniteRnrRetry) break;  // wait for a receive
                const uint64_t now = now_ns();
                if (v.rnr_next_ns == 0 || now >= v.rnr_next_ns) {
                    if (v.rnr_next_ns != 0) v.rnr_attempts += 1;
                    if (v.rnr_attempts >= qp.rnr_retry) {
                        status = UGDR_WC_RNR_RETRY_EXC_ERR;
                    } else {
                        v.rnr_next_ns = now + rnr_timer_ns(peer->min_rnr_timer);
                        break;
                    }
                } else {
                    break;
                }
            } else {
                queue::RecvWqe rh;
                std::memcpy(&rh, rq.first, sizeof(rh));
                recv_wr_id = rh.wr_id;
                // The receive CQ may be this batch's send CQ: publish what the batch has so far
                // (earlier WRs complete first), then check the responder's slot afresh.
                if (ncqe > 0) {
                    scq.publish(ncqe);
                    ncqe = 0;
                    cq_run = scq.reserve(k - i);
                }
                if (peer->recv_cq->ring.reserve(1).count() == 0) break;  // responder CQ full: wait
            }
        }
        // Requester CQ slot (signaled successes and every error).
        const bool need_cqe = signaled || status != UGDR_WC_SUCCESS;
        if (need_cqe && ncqe >= cq_run.count()) break;

        if (status == UGDR_WC_SUCCESS) {
            if (op_sum(op)) {
                // Element by element: every input element is read before its output is written,
                // so the remote range may be one of the SGEs.
                for (uint64_t e = 0; e < total / 2; ++e) {
                    float acc = 0.f;
                    for (uint32_t i = 0; i < nseg; ++i) {
                        uint16_t x;
                        std::memcpy(&x, segs[i].local + 2 * e, 2);
                        acc += bf16_to_f32(x);
                    }
                    const uint16_t r = bf16_rne(acc);
                    std::memcpy(remote + 2 * e, &r, 2);
                }
            } else if (op == UGDR_WR_RDMA_WRITE || op == UGDR_WR_RDMA_WRITE_WITH_IMM) {
                uint64_t off = 0;
                for (uint32_t i = 0; i < nseg; ++i) {
                    copy_bytes(remote + off, segs[i].local, segs[i].length);
                    off += segs[i].length;
                }
            } else if (op == UGDR_WR_RDMA_READ) {
                uint64_t off = 0;
                for (uint32_t i = 0; i < nseg; ++i) {
                    copy_bytes(segs[i].local, remote + off, segs[i].length);
                    off += segs[i].length;
                }
            } else {
                uint64_t compare_add = 0;
                std::memcpy(&compare_add, slot + queue::kAtomicCompareOffset, 8);
                const uint64_t swap = (uint64_t(h.reserved) << 32) | h.immediate_data;
                auto *target = reinterpret_cast<uint64_t *>(remote);
                uint64_t old;
                if (op == UGDR_WR_ATOMIC_FETCH_AND_ADD) {
                    old = __atomic_fetch_add(target, compare_add, __ATOMIC_ACQ_REL);
                } else {
                    old = compare_add;
                    __atomic_compare_exchange_n(target, &old, swap, false, __ATOMIC_ACQ_REL,
                                                __ATOMIC_ACQUIRE);
                }
                std::memcpy(segs[0].local, &old, 8);
            }
            std::atomic_thread_fence(std::memory_order_release);
            if (op == UGDR_WR_RDMA_WRITE_WITH_IMM) {
                peer->rq.peek(1);
                peer->rq.release(1);
                queue::Cqe rc{recv_wr_id, UGDR_WC_SUCCESS, UGDR_WC_RECV_RDMA_WITH_IMM,
                              uint32_t(total), h.immediate_data, peer->qpn, UGDR_WC_WITH_IMM};
                produce(peer->recv_cq, &rc);
                if (peer->recv_cq == qp.send_cq) cq_run = scq.reserve(k - i);  // produce() used the ring
            }
            v.rnr_attempts = 0;
            v.rnr_next_ns = 0;
            v.rnr_waiting = false;
            stats_.bytes_moved += op_atomic(op) ? 8 : total;
            v.c.bytes += op_atomic(op) ? 8 : total;
        }
        // The SQ slot is returned before the completion is visible (finish() releases first): a
        // client that sees the CQE may post into that slot at once (an HCA retires the WQE before
        // it reports it).
        ++consumed;
        if (need_cqe) {
            queue::Cqe c{h.wr_id, status, wc_opcode(op), uint32_t(total), 0, qp.qpn, 0};
            if (status != UGDR_WC_SUCCESS) c.byte_length = 0;
            std::memcpy(cq_slot(ncqe), &c, sizeof(c));
            ++ncqe;
        }
        ++retired;
        stats_.wrs_completed += 1;
        if (status != UGDR_WC_SUCCESS) {
            stats_.error_completions += 1;
            v.c.error_completions += 1;
            v.rnr_attempts = 0;
            v.rnr_next_ns = 0;
            finish();
            enter_error(qp);
            return retired + progress_qp(v);  // flush what remains
        }
    }
    finish();
    return retired;
}

size_t CpuEngine::progress_locked() {
    size_t n = 0;
    for (QpView &v : qps_) n += progress_qp(v);
    return n;
}

// Idle policy: spin (with a pause hint) for the first 50 us without work, then yield the CPU
// between passes for up to 2 ms, then sleep 50 us per pass.  Yielding keeps the engine
// responsive while letting a client that shares its core run; a sleep costs tens of
// microseconds however short it is asked to be.
void CpuEngine::run() {
    uint64_t idle_since = 0;
    while (!stop_.load(std::memory_order_relaxed)) {
        size_t n = 0;
        if (!held_.load(std::memory_order_relaxed)) {
            std::lock_guard<std::mutex> lk(objects_mu_);
            n = progress_locked();
        }
        if (n != 0) {
            idle_since = 0;
            continue;
        }
        const uint64_t now = now_ns();
        if (idle_since == 0) idle_since = now;
        const uint64_t idle = now - idle_since;
        if (idle < 50000) {
            for (int i = 0; i < 16; ++i) cpu_relax();
        } else if (idle < 2000000) {
            std::this_thread::yield();
        } else {
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
}

}  // namespace ugdr::engine
