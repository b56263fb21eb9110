// bf16 allreduce on the verbs: a reduce-scatter and an all-gather of RDMA WRITE work requests,
// with the sum done by the executor as it runs a UGDR_X_WR_RDMA_WRITE_SUM_BF16 WR.  This is
// client-side code: it calls only the public verbs entry points (post_recv, post_send,
// poll_cq), so it runs the same on the host engine and on the GPU executors.
//
// No counterpart in the reference (it has no collectives).  The primitive it builds on is the
// reference's WRITE_WITH_IMM receive completion (src/worker/worker.cpp:174-203): a rank learns
// that a peer's piece has landed from the immediate of the WR that carried it.
#include "ugdr/verbs_collective.h"

#include <cerrno>
#include <chrono>
#include <cstring>
#include <vector>

namespace {

constexpr int kMaxPieces = 64;
constexpr uint64_t kTagSum = 1ull << 60;
constexpr uint64_t kTagLast = 2ull << 60;

// Element ranges: shard s is [lo(s), hi(s)); its piece m is [plo, phi).  Boundaries sit on
// 8-element (16-byte) multiples so vector copies stay aligned; the last shard and the last piece
// of a shard take the remainders.
struct Geometry {
    uint64_t count;
    int n, pieces;
    uint64_t S;  // shard step
    uint64_t lo(int s) const { return S * uint64_t(s); }
    uint64_t hi(int s) const { return s == n - 1 ? count : S * uint64_t(s + 1); }
    uint64_t plo(int s, int m) const {
        const uint64_t P = (hi(s) - lo(s)) / uint64_t(pieces) / 8 * 8;
        return lo(s) + P * uint64_t(m);
    }
    uint64_t phi(int s, int m) const { return m == pieces - 1 ? hi(s) : plo(s, m + 1); }
    uint64_t shard_max() const { return count - S * uint64_t(n - 1); }
};

Geometry geometry(uint64_t count, int n, int pieces) {
    return Geometry{count, n, pieces, count / uint64_t(n) / 8 * 8};
}

uint32_t imm_of(uint32_t epoch, int phase, int piece, int sender) {
    return ((epoch & 0xffu) << 24) | (uint32_t(phase) << 16) | (uint32_t(piece) << 8) | uint32_t(sender);
}

}  // namespace

extern "C" uint64_t ugdr_x_verbs_allreduce_stage_bytes(uint64_t count, int n) noexcept {
    if (n < 1 || n > UGDR_X_VGROUP_MAX_RANKS) return 0;
    return uint64_t(n) * geometry(count, n, 1).shard_max() * 2;
}

extern "C" int ugdr_x_verbs_allreduce_bf16(ugdr_x_vgroup *g, uint64_t count, int pieces,
                                           uint64_t timeout_ns) noexcept {
    if (g == nullptr || g->n < 1 || g->n > UGDR_X_VGROUP_MAX_RANKS || g->rank < 0 || g->rank >= g->n ||
        pieces < 1 || pieces > kMaxPieces)
        return EINVAL;
    const int n = g->n, r = g->rank;
    if (n == 1) return 0;
    if (g->cq == nullptr || g->self_to == nullptr) return EINVAL;
    for (int q = 0; q < n; ++q)
        if (q != r && (g->peer[q].to == nullptr || g->peer[q].from == nullptr)) return EINVAL;
    const Geometry G = geometry(count, n, pieces);
    const uint64_t smax = G.shard_max();
    if (g->stage_bytes < uint64_t(n) * smax * 2) return EINVAL;
    const uint32_t epoch = g->epoch++;

    // Receives for this call: every peer sends `pieces` immediates per phase.
    std::vector<ugdr_recv_wr> rw(static_cast<size_t>(2 * pieces));
    for (int q = 0; q < n; ++q) {
        if (q == r) continue;
        for (int i = 0; i < 2 * pieces; ++i) {
            rw[i] = ugdr_recv_wr{};
            rw[i].wr_id = (uint64_t(q) << 16) | uint64_t(i);
            rw[i].next = i + 1 < 2 * pieces ? &rw[i + 1] : nullptr;
        }
        ugdr_recv_wr *bad = nullptr;
        if (int rc = ugdr_post_recv(g->peer[q].from, rw.data(), &bad); rc != 0) return rc;
    }

    auto bytes = [](uint64_t elems) { return elems * 2; };
    // Phase 1: piece m of shard q to rank q's staging slot r, as one chain per peer.
    {
        std::vector<ugdr_send_wr> w(static_cast<size_t>(pieces));
        std::vector<ugdr_sge> sg(static_cast<size_t>(pieces));
        for (int k = 1; k < n; ++k) {
            const int q = (r + k) % n;  // peers in turn, so ranks do not all start on rank 0
            for (int m = 0; m < pieces; ++m) {
                const uint64_t a = G.plo(q, m), b = G.phi(q, m);
                sg[m] = ugdr_sge{g->buf_addr + bytes(a), uint32_t(bytes(b - a)), g->buf_lkey};
                w[m] = ugdr_send_wr{};
                w[m].wr_id = uint64_t(m);
                w[m].sg_list = &sg[m];
                w[m].num_sge = 1;
                w[m].opcode = UGDR_WR_RDMA_WRITE_WITH_IMM;
                w[m].imm_data = imm_of(epoch, 1, m, r);
                w[m].wr.rdma.remote_addr = g->peer[q].stage_addr + bytes(uint64_t(r) * smax + (a - G.lo(q)));
                w[m].wr.rdma.rkey = g->peer[q].stage_rkey;
                w[m].next = m + 1 < pieces ? &w[m + 1] : nullptr;
            }
            ugdr_send_wr *bad = nullptr;
            if (int rc = ugdr_post_send(g->peer[q].to, w.data(), &bad); rc != 0) return rc;
        }
    }

    auto post_sum = [&](int m) -> int {
        const uint64_t a = G.plo(r, m), b = G.phi(r, m);
        // SGEs in rank order (this rank's own piece at position r), so every element of the
        // result is the fp32 sum x_0 + x_1 + ... + x_{n-1} rounded once, whichever rank owns it.
        ugdr_sge sg[UGDR_X_VGROUP_MAX_RANKS];
        int k = 0;
        for (int q = 0; q < n; ++q)
            sg[k++] = q == r ? ugdr_sge{g->buf_addr + bytes(a), uint32_t(bytes(b - a)), g->buf_lkey}
                             : ugdr_sge{g->stage_addr + bytes(uint64_t(q) * smax + (a - G.lo(r))),
                                        uint32_t(bytes(b - a)), g->stage_lkey};
        ugdr_send_wr w{};
        w.wr_id = kTagSum | uint64_t(m);
        w.sg_list = sg;
        w.num_sge = k;
        w.opcode = UGDR_X_WR_RDMA_WRITE_SUM_BF16;
        w.send_flags = UGDR_SEND_SIGNALED;
        w.wr.rdma.remote_addr = g->buf_addr + bytes(a);
        w.wr.rdma.rkey = g->buf_rkey;
        ugdr_send_wr *bad = nullptr;
        return ugdr_post_send(g->self_to, &w, &bad);
    };
    auto post_gather = [&](int m) -> int {
        const uint64_t a = G.plo(r, m), b = G.phi(r, m);
        for (int k = 1; k < n; ++k) {
            const int q = (r + k) % n;
            ugdr_sge sg{g->buf_addr + bytes(a), uint32_t(bytes(b - a)), g->buf_lkey};
            ugdr_send_wr w{};
            w.wr_id = (m == pieces - 1 ? kTagLast : 0) | uint64_t(q);
            w.sg_list = &sg;
            w.num_sge = 1;
            w.opcode = UGDR_WR_RDMA_WRITE_WITH_IMM;
            w.send_flags = m == pieces - 1 ? UGDR_SEND_SIGNALED : 0;  // the QP's last WR of the call
            w.imm_data = imm_of(epoch, 3, m, r);
            w.wr.rdma.remote_addr = g->peer[q].buf_addr + bytes(a);
            w.wr.rdma.rkey = g->peer[q].buf_rkey;
            ugdr_send_wr *bad = nullptr;
            if (int rc = ugdr_post_send(g->peer[q].to, &w, &bad); rc != 0) return rc;
        }
        return 0;
    };

    int arrived1[kMaxPieces] = {};
    int arrived3 = 0, sums = 0, lasts = 0;
    const int want3 = (n - 1) * pieces;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(timeout_ns);
    ugdr_wc wc[64];
    uint32_t idle = 0;
    while (arrived3 < want3 || sums < pieces || lasts < n - 1) {
        const int k = ugdr_poll_cq(g->cq, 64, wc);
        if (k < 0) return -k;
        if (k == 0) {
            if ((++idle & 1023) == 0 && std::chrono::steady_clock::now() > deadline) return ETIMEDOUT;
            continue;
        }
        idle = 0;
        for (int i = 0; i < k; ++i) {
            if (wc[i].status != UGDR_WC_SUCCESS) return EIO;
            if (wc[i].opcode == UGDR_WC_RECV_RDMA_WITH_IMM) {
                const uint32_t imm = wc[i].imm_data;
                const int phase = int((imm >> 16) & 0xffu), m = int((imm >> 8) & 0xffu);
                if ((imm >> 24) != (epoch & 0xffu) || m >= pieces || (phase != 1 && phase != 3)) return EIO;
                if (phase == 3) {
                    ++arrived3;
                } else if (++arrived1[m] == n - 1) {
                    if (int rc = post_sum(m); rc != 0) return rc;
                }
            } else if (wc[i].wr_id & kTagSum) {
                ++sums;
                if (int rc = post_gather(int(wc[i].wr_id & 0xffffu)); rc != 0) return rc;
            } else if (wc[i].wr_id & kTagLast) {
                ++lasts;
            }
        }
    }
    return 0;
}

extern "C" int ugdr_x_verbs_allreduce_bf16_mc(ugdr_x_vgroup *g, uint64_t mc_addr, uint32_t mc_lkey, uint32_t mc_rkey,
                                              uint64_t count, uint64_t timeout_ns) noexcept {
    if (g == nullptr || g->n < 1 || g->n > UGDR_X_VGROUP_MAX_RANKS || g->rank < 0 || g->rank >= g->n ||
        g->cq == nullptr || g->self_to == nullptr || mc_addr == 0 || (mc_addr & 15) != 0 || count % 8 != 0)
        return EINVAL;
    const int n = g->n, r = g->rank;
    for (int q = 0; q < n; ++q)
        if (q != r && (g->peer[q].to == nullptr || g->peer[q].from == nullptr)) return EINVAL;
    const Geometry G = geometry(count, n, 1);
    const uint32_t epoch = g->epoch++;
    constexpr int kReady = 7, kDone = 8;

    for (int q = 0; q < n; ++q) {
        if (q == r) continue;
        ugdr_recv_wr rw[2] = {};
        rw[0].next = &rw[1];
        ugdr_recv_wr *bad = nullptr;
        if (int rc = ugdr_post_recv(g->peer[q].from, rw, &bad); rc != 0) return rc;
    }
    // A zero-length WRITE_WITH_IMM to every peer; with `signal`, its retirement (after every
    // earlier WR of the QP) is reported here too.
    auto notify = [&](int phase, bool signal) -> int {
        for (int k = 1; k < n; ++k) {
            const int q = (r + k) % n;
            ugdr_send_wr w{};
            w.wr_id = signal ? (kTagLast | uint64_t(q)) : 0;
            w.opcode = UGDR_WR_RDMA_WRITE_WITH_IMM;
            w.send_flags = signal ? UGDR_SEND_SIGNALED : 0;
            w.imm_data = imm_of(epoch, phase, 0, r);
            w.wr.rdma.remote_addr = g->peer[q].buf_addr;
            w.wr.rdma.rkey = g->peer[q].buf_rkey;
            ugdr_send_wr *bad = nullptr;
            if (int rc = ugdr_post_send(g->peer[q].to, &w, &bad); rc != 0) return rc;
        }
        return 0;
    };
    int ready = 0, done = 0, lasts = 0, sums = 0;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(timeout_ns);
    auto wait = [&](auto until) -> int {
        ugdr_wc wc[64];
        uint32_t idle = 0;
        while (!until()) {
            const int k = ugdr_poll_cq(g->cq, 64, wc);
            if (k < 0) return -k;
            if (k == 0) {
                if ((++idle & 1023) == 0 && std::chrono::steady_clock::now() > deadline) return ETIMEDOUT;
                continue;
            }
            idle = 0;
            for (int i = 0; i < k; ++i) {
                if (wc[i].status != UGDR_WC_SUCCESS) return EIO;
                if (wc[i].opcode == UGDR_WC_RECV_RDMA_WITH_IMM) {
                    const uint32_t imm = wc[i].imm_data;
                    const int phase = int((imm >> 16) & 0xffu);
                    if ((imm >> 24) != (epoch & 0xffu)) return EIO;
                    if (phase == kReady) ++ready;
                    else if (phase == kDone) ++done;
                    else return EIO;
                } else if (wc[i].wr_id & kTagSum) {
                    ++sums;
                } else if (wc[i].wr_id & kTagLast) {
                    ++lasts;
                }
            }
        }
        return 0;
    };
    // 1. Every rank's input is in place.
    if (int rc = notify(kReady, false); rc != 0) return rc;
    if (int rc = wait([&] { return ready == n - 1; }); rc != 0) return rc;
    // 2. This rank's shard: one WRITE_SUM_BF16 from the multicast view (the NVSwitch sums every
    //    GPU's copy) to the multicast view (every GPU receives the sum).
    {
        const uint64_t a = G.lo(r), b = G.hi(r);
        ugdr_sge sg{mc_addr + a * 2, uint32_t((b - a) * 2), mc_lkey};
        ugdr_send_wr w{};
        w.wr_id = kTagSum;
        w.sg_list = &sg;
        w.num_sge = 1;
        w.opcode = UGDR_X_WR_RDMA_WRITE_SUM_BF16;
        w.send_flags = UGDR_SEND_SIGNALED;
        w.wr.rdma.remote_addr = mc_addr + a * 2;
        w.wr.rdma.rkey = mc_rkey;
        ugdr_send_wr *bad = nullptr;
        if (int rc = ugdr_post_send(g->self_to, &w, &bad); rc != 0) return rc;
    }
    if (int rc = wait([&] { return sums == 1; }); rc != 0) return rc;
    // 3. Tell every peer this shard is everywhere; done when every shard is.
    if (int rc = notify(kDone, true); rc != 0) return rc;
    return wait([&] { return done == n - 1 && lasts == n - 1; });
}
