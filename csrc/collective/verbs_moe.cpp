// MoE all-to-all on the verbs: the dispatch and combine permutes are the SGE lists of RDMA WRITE
// and READ work requests that the daemon's executors run.  Client-side code over the public
// verbs calls only (post_recv, post_send, poll_cq).
//
// Dispatch: the per-expert row counts go to every rank as WRITE_WITH_IMM into its count table
// (a registered host buffer); from the full table every rank knows where each (expert, source
// rank) group starts in each owner's receive area.  Then, per owner and expert, WRITEs of up to
// 32 SGEs gather this rank's rows of that expert (one SGE per token row) into the group's
// contiguous range; the last WR to each owner carries an immediate that tells the owner this
// rank's rows have all landed (the owner's QP retires WRs in order).  The packed form takes the
// rows already grouped by expert (ugdr_x_moe_pack_grouped on the GPU) and sends each
// (owner, expert) group as one contiguous WRITE.
// Combine: per owner and expert, READs of up to 32 SGEs bring the group back and scatter it
// (one SGE per row) into (token, k) order.
//
// No counterpart in the reference (it has no collectives); the immediate-signalled WRITE is its
// WRITE_WITH_IMM receive completion (src/worker/worker.cpp:174-203).
#include "ugdr/verbs_collective.h"

#include <cerrno>
#include <chrono>
#include <cstring>
#include <vector>

namespace {

constexpr int kSgePerWr = 32;
constexpr uint64_t kTagLast = 2ull << 60;
constexpr int kPhaseCounts = 5, kPhaseRows = 6;

uint32_t imm_of(uint32_t epoch, int phase, int sender) {
    return ((epoch & 0xffu) << 24) | (uint32_t(phase) << 16) | uint32_t(sender);
}

// The WRs of one call on one QP, posted as far as its send queue allows and re-posted from the
// first refused one as slots free up.
struct Chain {
    ugdr_qp *qp = nullptr;
    std::vector<ugdr_send_wr> wr;
    std::vector<ugdr_sge> sge;
    size_t next = 0;
    void link() {
        for (size_t i = 0; i + 1 < wr.size(); ++i) wr[i].next = &wr[i + 1];
        if (!wr.empty()) wr.back().next = nullptr;
    }
    int post() {
        if (next >= wr.size()) return 0;
        ugdr_send_wr *bad = nullptr;
        const int rc = ugdr_post_send(qp, &wr[next], &bad);
        if (rc == 0) {
            next = wr.size();
        } else if (rc == ENOMEM && bad != nullptr) {
            next = size_t(bad - wr.data());
        } else {
            return rc;
        }
        return 0;
    }
    bool done() const { return next >= wr.size(); }
};

// Rows of this rank by expert in position order: flat (token, k) row index of position p of
// expert e is at order[start[e] + p].
struct Buckets {
    std::vector<uint64_t> start;
    std::vector<uint32_t> order;
};

int bucket(const ugdr_x_vmoe *m, const int32_t *ids, const int32_t *pos, const int32_t *counts, Buckets *b) {
    const uint64_t rows = uint64_t(m->tokens) * uint64_t(m->topk);
    b->start.assign(size_t(m->nexp) + 1, 0);
    for (int e = 0; e < m->nexp; ++e) {
        if (counts[e] < 0) return EINVAL;
        b->start[e + 1] = b->start[e] + uint64_t(counts[e]);
    }
    if (b->start[m->nexp] != rows) return EINVAL;
    b->order.assign(rows, 0);
    for (uint64_t i = 0; i < rows; ++i) {
        const int32_t e = ids[i], p = pos[i];
        if (e < 0 || e >= m->nexp || p < 0 || p >= counts[e]) return EINVAL;
        b->order[b->start[e] + uint64_t(p)] = uint32_t(i);
    }
    return 0;
}

bool valid(const ugdr_x_vgroup *g, const ugdr_x_vmoe *m) {
    if (g == nullptr || m == nullptr || g->n < 1 || g->n > UGDR_X_VGROUP_MAX_RANKS || g->rank < 0 ||
        g->rank >= g->n || g->cq == nullptr || g->self_to == nullptr)
        return false;
    if (m->tokens <= 0 || m->topk <= 0 || m->nexp <= 0 || m->nexp % g->n != 0 || m->row_bytes == 0 ||
        m->table == nullptr || m->base == nullptr)
        return false;
    for (int q = 0; q < g->n; ++q)
        if (q != g->rank && (g->peer[q].to == nullptr || g->peer[q].from == nullptr)) return false;
    return true;
}

ugdr_qp *qp_to(const ugdr_x_vgroup *g, int q) { return q == g->rank ? g->self_to : g->peer[q].to; }

// Poll until `done()`, re-posting refused chains and handing each completion to `on`.
template <typename Done, typename On>
int drive(ugdr_x_vgroup *g, std::vector<Chain> &chains, uint64_t timeout_ns, Done done, On on) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(timeout_ns);
    ugdr_wc wc[64];
    uint32_t idle = 0;
    for (;;) {
        bool all_posted = true;
        for (Chain &c : chains) {
            if (int rc = c.post(); rc != 0) return rc;
            all_posted &= c.done();
        }
        if (all_posted && done()) return 0;
        const int k = ugdr_poll_cq(g->cq, 64, wc);
        if (k < 0) return -k;
        if (k == 0) {
            if ((++idle & 1023) == 0 && std::chrono::steady_clock::now() > deadline) return ETIMEDOUT;
            continue;
        }
        idle = 0;
        for (int i = 0; i < k; ++i) {
            if (wc[i].status != UGDR_WC_SUCCESS) return EIO;
            if (int rc = on(wc[i]); rc != 0) return rc;
        }
    }
}

}  // namespace

extern "C" uint32_t ugdr_x_verbs_moe_wrs(uint64_t rows_per_rank, int nexp, int n) noexcept {
    if (n < 1 || nexp < 1) return 0;
    // Every expert group of one owner starts a new WR: at most ceil(rows / 32) + experts-per-owner.
    return uint32_t((rows_per_rank + kSgePerWr - 1) / kSgePerWr + uint64_t(nexp / n) + 2);
}

namespace {

// Both dispatch forms.  Gathered (`ids` / `pos` given): per owner and expert, WRs of up to 32
// row SGEs straight from x.  Packed (`ids` null): `back` already holds this rank's rows grouped
// by expert, and each (owner, expert) group leaves as ONE contiguous WRITE, so the executors
// chunk it over all their warps instead of staging one 32-SGE WR per pass.
int dispatch(ugdr_x_vgroup *g, ugdr_x_vmoe *m, const int32_t *ids, const int32_t *pos, const int32_t *counts,
             uint64_t timeout_ns) {
    const int n = g->n, r = g->rank, E = m->nexp, epr = E / n;
    const bool packed = ids == nullptr;
    Buckets b;
    if (packed) {
        b.start.assign(size_t(E) + 1, 0);
        for (int e = 0; e < E; ++e) {
            if (counts[e] < 0) return EINVAL;
            b.start[e + 1] = b.start[e] + uint64_t(counts[e]);
        }
        if (b.start[E] != uint64_t(m->tokens) * uint64_t(m->topk)) return EINVAL;
        if (m->back_addr == 0) return EINVAL;
    } else if (int rc = bucket(m, ids, pos, counts, &b); rc != 0) {
        return rc;
    }
    const uint32_t epoch = g->epoch++;

    // Receives: one count-table write and one rows-landed immediate from every peer.
    for (int q = 0; q < n; ++q) {
        if (q == r) continue;
        ugdr_recv_wr rw[2] = {};
        rw[0].wr_id = uint64_t(q);
        rw[0].next = &rw[1];
        rw[1].wr_id = uint64_t(q);
        ugdr_recv_wr *bad = nullptr;
        if (int rc = ugdr_post_recv(g->peer[q].from, rw, &bad); rc != 0) return rc;
    }

    // 1. Counts to every rank's table.
    std::memcpy(m->table + size_t(r) * size_t(E), counts, size_t(E) * 4);
    std::vector<Chain> chains(static_cast<size_t>(n));
    for (int q = 0; q < n; ++q) {
        if (q == r) continue;
        Chain &c = chains[q];
        c.qp = g->peer[q].to;
        c.sge.push_back(ugdr_sge{uint64_t(reinterpret_cast<uintptr_t>(m->table + size_t(r) * size_t(E))),
                                 uint32_t(E * 4), m->table_lkey});
        ugdr_send_wr w{};
        w.sg_list = c.sge.data();
        w.num_sge = 1;
        w.opcode = UGDR_WR_RDMA_WRITE_WITH_IMM;
        w.imm_data = imm_of(epoch, kPhaseCounts, r);
        w.wr.rdma.remote_addr = m->peer_table_addr[q] + uint64_t(r) * uint64_t(E) * 4;
        w.wr.rdma.rkey = m->peer_table_rkey[q];
        c.wr.push_back(w);
        c.link();
    }
    int counts_in = 0, rows_in = 0, lasts = 0;
    auto on = [&](const ugdr_wc &wc) -> int {
        if (wc.opcode == UGDR_WC_RECV_RDMA_WITH_IMM) {
            const uint32_t imm = wc.imm_data;
            const int phase = int((imm >> 16) & 0xffu);
            if ((imm >> 24) != (epoch & 0xffu)) return EIO;
            if (phase == kPhaseCounts) ++counts_in;
            else if (phase == kPhaseRows) ++rows_in;
            else return EIO;
        } else if (wc.wr_id & kTagLast) {
            ++lasts;
        }
        return 0;
    };
    if (int rc = drive(g, chains, timeout_ns, [&] { return counts_in == n - 1; }, on); rc != 0) return rc;

    // 2. Group bases at every owner: experts in order, inside an expert the source ranks in order.
    uint64_t mine = 0;
    for (int q = 0; q < n; ++q) {
        uint64_t off = 0;
        for (int e = q * epr; e < (q + 1) * epr; ++e)
            for (int s = 0; s < n; ++s) {
                m->base[size_t(e) * size_t(n) + size_t(s)] = off;
                off += uint64_t(m->table[size_t(s) * size_t(E) + size_t(e)]);
            }
        if (q == r) mine = off;
    }
    if (mine > m->recv_rows) return ENOSPC;
    m->received = mine;

    // 3. Rows: per owner, per expert, WRs of up to 32 row SGEs into the group's range.
    const uint64_t rb = m->row_bytes;
    for (int k = 0; k < n; ++k) {
        const int q = (r + 1 + k) % n;  // owners in turn, this rank last
        Chain &c = chains[q];
        c = Chain{};
        c.qp = qp_to(g, q);
        const uint64_t dst0 = q == r ? m->recv_addr : m->peer_recv_addr[q];
        const uint32_t rkey = q == r ? m->recv_rkey : m->peer_recv_rkey[q];
        uint64_t nrows = 0;
        for (int e = q * epr; e < (q + 1) * epr; ++e) nrows += uint64_t(counts[e]);
        c.sge.reserve(size_t(nrows));
        c.wr.reserve(size_t(nrows / kSgePerWr + epr + 2));
        for (int e = q * epr; e < (q + 1) * epr; ++e) {
            const uint64_t ce = uint64_t(counts[e]);
            if (packed) {
                // One WRITE per group, split only where an SGE's 32-bit length would overflow.
                const uint64_t per = 0xffffffffull / rb;  // >= 1: row_bytes is 32-bit
                for (uint64_t j = 0; j < ce; j += per) {
                    const uint64_t take = ce - j < per ? ce - j : per;
                    c.sge.push_back(ugdr_sge{m->back_addr + (b.start[e] + j) * rb, uint32_t(take * rb), m->back_lkey});
                    ugdr_send_wr w{};
                    w.num_sge = 1;
                    w.opcode = UGDR_WR_RDMA_WRITE;
                    w.wr.rdma.remote_addr = dst0 + (m->base[size_t(e) * size_t(n) + size_t(r)] + j) * rb;
                    w.wr.rdma.rkey = rkey;
                    c.wr.push_back(w);
                }
                continue;
            }
            for (uint64_t j = 0; j < ce; j += kSgePerWr) {
                const uint64_t take = ce - j < uint64_t(kSgePerWr) ? ce - j : uint64_t(kSgePerWr);
                const size_t first = c.sge.size();
                for (uint64_t p = j; p < j + take; ++p) {
                    const uint64_t tok = b.order[b.start[e] + p] / uint64_t(m->topk);
                    c.sge.push_back(ugdr_sge{m->x_addr + tok * rb, uint32_t(rb), m->x_lkey});
                }
                ugdr_send_wr w{};
                w.sg_list = &c.sge[first];
                w.num_sge = int(take);
                w.opcode = UGDR_WR_RDMA_WRITE;
                w.wr.rdma.remote_addr = dst0 + (m->base[size_t(e) * size_t(n) + size_t(r)] + j) * rb;
                w.wr.rdma.rkey = rkey;
                c.wr.push_back(w);
            }
        }
        // The owner learns that every row has landed from the immediate of the last WR (a QP's
        // WRs retire in order); toward this rank itself a signalled WRITE is enough.
        ugdr_send_wr w{};
        w.wr_id = kTagLast | uint64_t(q);
        w.send_flags = UGDR_SEND_SIGNALED;
        if (q != r) {
            w.opcode = UGDR_WR_RDMA_WRITE_WITH_IMM;
            w.imm_data = imm_of(epoch, kPhaseRows, r);
            w.wr.rdma.remote_addr = dst0;
            w.wr.rdma.rkey = rkey;
        } else {
            w.opcode = UGDR_WR_RDMA_WRITE;
            w.wr.rdma.remote_addr = dst0;
            w.wr.rdma.rkey = rkey;
        }
        c.wr.push_back(w);
        if (packed)  // sg_list of WR i is SGE i (the closing WR has none)
            for (size_t i = 0; i + 1 < c.wr.size(); ++i) c.wr[i].sg_list = &c.sge[i];
        c.link();
    }
    return drive(g, chains, timeout_ns, [&] { return rows_in == n - 1 && lasts == n; }, on);
}

}  // namespace

extern "C" int ugdr_x_verbs_moe_dispatch(ugdr_x_vgroup *g, ugdr_x_vmoe *m, const int32_t *ids, const int32_t *pos,
                                         const int32_t *counts, uint64_t timeout_ns) noexcept {
    if (!valid(g, m) || ids == nullptr || pos == nullptr || counts == nullptr) return EINVAL;
    return dispatch(g, m, ids, pos, counts, timeout_ns);
}

extern "C" int ugdr_x_verbs_moe_dispatch_packed(ugdr_x_vgroup *g, ugdr_x_vmoe *m, const int32_t *counts,
                                                uint64_t timeout_ns) noexcept {
    if (!valid(g, m) || counts == nullptr) return EINVAL;
    return dispatch(g, m, nullptr, nullptr, counts, timeout_ns);
}

extern "C" int ugdr_x_verbs_moe_combine(ugdr_x_vgroup *g, ugdr_x_vmoe *m, uint64_t timeout_ns) noexcept {
    if (!valid(g, m)) return EINVAL;
    const int n = g->n, r = g->rank, E = m->nexp, epr = E / n;
    const int32_t *counts = m->table + size_t(r) * size_t(E);
    const uint64_t rb = m->row_bytes;
    // `back` holds this rank's rows grouped by expert (expert e's rows from row start(e) on, in
    // position order), the same order dispatch read them in, so every (owner, expert) group
    // comes back with ONE contiguous READ; the unpermute to (token, k) order is done by the
    // weighted sum that consumes them (ugdr_x_moe_weighted_sum_grouped).
    std::vector<uint64_t> start(size_t(E) + 1, 0);
    for (int e = 0; e < E; ++e) {
        if (counts[e] < 0) return EINVAL;
        start[e + 1] = start[e] + uint64_t(counts[e]);
    }
    if (start[E] != uint64_t(m->tokens) * uint64_t(m->topk)) return EINVAL;
    std::vector<Chain> chains(static_cast<size_t>(n));
    for (int k = 0; k < n; ++k) {
        const int q = (r + 1 + k) % n;
        Chain &c = chains[q];
        c.qp = qp_to(g, q);
        const uint64_t src0 = q == r ? m->recv_addr : m->peer_recv_addr[q];
        const uint32_t rkey = q == r ? m->recv_rkey : m->peer_recv_rkey[q];
        c.sge.reserve(size_t(epr));
        c.wr.reserve(size_t(epr + 1));
        for (int e = q * epr; e < (q + 1) * epr; ++e) {
            const uint64_t ce = uint64_t(counts[e]);
            if (ce == 0) continue;
            if (ce * rb > 0xffffffffull) return EINVAL;  // one SGE per group
            c.sge.push_back(ugdr_sge{m->back_addr + start[e] * rb, uint32_t(ce * rb), m->back_lkey});
            ugdr_send_wr w{};
            w.sg_list = &c.sge.back();
            w.num_sge = 1;
            w.opcode = UGDR_WR_RDMA_READ;
            w.wr.rdma.remote_addr = src0 + m->base[size_t(e) * size_t(n) + size_t(r)] * rb;
            w.wr.rdma.rkey = rkey;
            c.wr.push_back(w);
        }
        // A zero-length signalled READ closes the QP's list (its WRs retire in order).
        ugdr_send_wr w{};
        w.wr_id = kTagLast | uint64_t(q);
        w.send_flags = UGDR_SEND_SIGNALED;
        w.opcode = UGDR_WR_RDMA_READ;
        w.wr.rdma.remote_addr = src0;
        w.wr.rdma.rkey = rkey;
        c.wr.push_back(w);
        c.link();
    }
    int lasts = 0;
    return drive(g, chains, timeout_ns, [&] { return lasts == n; }, [&](const ugdr_wc &wc) -> int {
        if (wc.opcode == UGDR_WC_RECV_RDMA_WITH_IMM) return EIO;  // nothing signals this rank in combine
        if (wc.wr_id & kTagLast) ++lasts;
        return 0;
    });
}
