// Concurrent use of the public API from one client process (reference suite semantics: the
// per-QP posting and per-CQ polling locks of src/api/api.cpp, exercised here from threads; under
// the TSan build this is the client library's race check).
//
// Four worker threads each create their own QP pair on one shared PD and CQ, then post signaled
// 64-byte WRITEs into their own slice of a shared host MR, keeping at most 32 in flight.  Two
// poller threads drain the shared CQ concurrently and credit each completion to the thread that
// posted it (wr_id high bits).  At the end every slice must hold its worker's pattern, every WR
// must have completed exactly once, and every object must destroy cleanly.
#include "harness.hpp"

#include "daemon_proc.hpp"
#include "ugdr/api.hpp"

#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int kWorkers = 4;
constexpr int kPollers = 2;
constexpr uint64_t kWrsPerWorker = 3000;
constexpr uint64_t kWindow = 32;
constexpr uint32_t kBytes = 64;
constexpr size_t kSlice = 1 << 16;

struct Shared {
    ugdr_pd *pd = nullptr;
    ugdr_cq *cq = nullptr;
    ugdr_mr *mr = nullptr;
    uint8_t *buf = nullptr;
    std::atomic<uint64_t> done[kWorkers] = {};
    std::atomic<uint64_t> bad_status{0}, bad_id{0}, worker_errors{0};
    std::atomic<bool> stop{false};
};

bool connect_pair(ugdr_qp *a, ugdr_qp *b) {
    ugdr_qp_attr at{};
    at.qp_state = UGDR_QPS_INIT;
    at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE;
    if (ugdr_modify_qp(a, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS) != 0 ||
        ugdr_modify_qp(b, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS) != 0)
        return false;
    ugdr_qp_conn_info ca{}, cb{};
    if (ugdr_query_qp_conn_info(a, &ca) != 0 || ugdr_query_qp_conn_info(b, &cb) != 0) return false;
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    const int m = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    return ugdr_connect_qp(a, &cb, &c, m) == 0 && ugdr_connect_qp(b, &ca, &c, m) == 0;
}

void worker(Shared *s, int t) {
    ugdr_qp_init_attr ia{s->cq, s->cq, 64, 16, 1, 1, UGDR_QPT_RC, 0};
    ugdr_qp *a = ugdr_create_qp(s->pd, &ia), *b = ugdr_create_qp(s->pd, &ia);
    if (a == nullptr || b == nullptr || !connect_pair(a, b)) {
        s->worker_errors.fetch_add(1);
        return;
    }
    // Source: the first half of this worker's slice; destination: the second half.
    uint8_t *src = s->buf + size_t(t) * kSlice;
    for (size_t i = 0; i < kSlice / 2; ++i) src[i] = uint8_t(i * 7 + t * 31 + 1);
    ugdr_sge sg{0, kBytes, s->mr->lkey};
    ugdr_send_wr wr{};
    wr.sg_list = &sg;
    wr.num_sge = 1;
    wr.opcode = UGDR_WR_RDMA_WRITE;
    wr.send_flags = UGDR_SEND_SIGNALED;
    wr.wr.rdma.rkey = s->mr->rkey;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    for (uint64_t i = 0; i < kWrsPerWorker;) {
        if (i - s->done[t].load(std::memory_order_acquire) >= kWindow) {
            if (std::chrono::steady_clock::now() > deadline) {
                s->worker_errors.fetch_add(1);
                break;
            }
            std::this_thread::yield();
            continue;
        }
        const uint64_t off = (i * kBytes) % (kSlice / 2);
        sg.addr = reinterpret_cast<uint64_t>(src + off);
        wr.wr.rdma.remote_addr = reinterpret_cast<uint64_t>(src + kSlice / 2 + off);
        wr.wr_id = (uint64_t(t) << 32) | i;
        ugdr_send_wr *bad = nullptr;
        if (ugdr_post_send(a, &wr, &bad) != 0) {
            s->worker_errors.fetch_add(1);
            break;
        }
        ++i;
    }
    while (s->done[t].load(std::memory_order_acquire) < kWrsPerWorker &&
           std::chrono::steady_clock::now() < deadline)
        std::this_thread::yield();
    if (ugdr_destroy_qp(a) != 0 || ugdr_destroy_qp(b) != 0) s->worker_errors.fetch_add(1);
}

void poller(Shared *s) {
    ugdr_wc wc[16];
    while (!s->stop.load(std::memory_order_acquire)) {
        const int n = ugdr_poll_cq(s->cq, 16, wc);
        if (n < 0) {
            s->bad_status.fetch_add(1);
            return;
        }
        for (int i = 0; i < n; ++i) {
            const uint64_t t = wc[i].wr_id >> 32;
            if (wc[i].status != UGDR_WC_SUCCESS) s->bad_status.fetch_add(1);
            if (t >= uint64_t(kWorkers)) {
                s->bad_id.fetch_add(1);
                continue;
            }
            s->done[t].fetch_add(1, std::memory_order_acq_rel);
        }
        if (n == 0) std::this_thread::yield();
    }
}

}  // namespace

TEST(api_threads_post_and_poll_concurrently) {
    th::DaemonProc d;
    if (!d.start()) {
        std::fprintf(stderr, "  (skipped: ugdr_daemon not found next to the test binary)\n");
        return;
    }
    ::setenv("UGDR_DAEMON_SOCKET", d.sock.c_str(), 1);
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    CHECK(list != nullptr);
    if (list == nullptr) return;
    ugdr_device *cpu = nullptr;
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0 && info.kind == 0) cpu = list[i];
    }
    CHECK(cpu != nullptr);
    if (cpu == nullptr) return;
    ugdr_context *ctx = ugdr_open_device(cpu);
    Shared s;
    s.pd = ugdr_alloc_pd(ctx);
    s.cq = ugdr_create_cq(ctx, 1024, nullptr, nullptr, 0);
    const size_t bytes = kSlice * kWorkers;
    s.buf = static_cast<uint8_t *>(ugdr_x_alloc_host(bytes));
    CHECK(ctx && s.pd && s.cq && s.buf);
    if (!(ctx && s.pd && s.cq && s.buf)) return;
    std::memset(s.buf, 0, bytes);
    s.mr = ugdr_reg_mr(s.pd, s.buf, bytes, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE);
    CHECK(s.mr != nullptr);
    if (s.mr == nullptr) return;

    std::vector<std::thread> pollers, workers;
    for (int i = 0; i < kPollers; ++i) pollers.emplace_back(poller, &s);
    for (int t = 0; t < kWorkers; ++t) workers.emplace_back(worker, &s, t);
    for (auto &w : workers) w.join();
    s.stop.store(true, std::memory_order_release);
    for (auto &p : pollers) p.join();

    CHECK_EQ(s.worker_errors.load(), 0ull);
    CHECK_EQ(s.bad_status.load(), 0ull);
    CHECK_EQ(s.bad_id.load(), 0ull);
    for (int t = 0; t < kWorkers; ++t) {
        CHECK_EQ(s.done[t].load(), kWrsPerWorker);
        const uint8_t *slice = s.buf + size_t(t) * kSlice;
        // Every 64-byte block of the source half was written at least once (3000 x 64 B > 32 KiB).
        CHECK(std::memcmp(slice + kSlice / 2, slice, kSlice / 2) == 0);
    }
    ugdr_wc extra[4];
    CHECK_EQ(ugdr_poll_cq(s.cq, 4, extra), 0);
    CHECK_EQ(ugdr_dereg_mr(s.mr), 0);
    CHECK_EQ(ugdr_x_free_host(s.buf), 0);
    CHECK_EQ(ugdr_destroy_cq(s.cq), 0);
    CHECK_EQ(ugdr_dealloc_pd(s.pd), 0);
    CHECK_EQ(ugdr_close_device(ctx), 0);
    ugdr_free_device_list(list);
}
