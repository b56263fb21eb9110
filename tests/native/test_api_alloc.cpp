// Hot-path allocation check through the public API (reference suite semantics:
// tests/integration/queue_api_client_server_test.cpp counts global operator new calls and
// asserts none happen in a warmed post_send / poll_cq window).
//
// The test starts the real ugdr_daemon (found next to this binary, or at $UGDR_DAEMON_BIN) on a
// private socket with the host-memory device only, sets up one QP pair over host buffers, warms
// up, then counts operator new calls while it posts signaled 8-byte WRITEs and polls their
// completions.
#include "harness.hpp"

#include "daemon_proc.hpp"
#include "ugdr/api.hpp"

#include <signal.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <sys/wait.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <thread>

namespace {
std::atomic<bool> g_counting{false};
std::atomic<unsigned long long> g_news{0};

void *counted(std::size_t n) {
    if (g_counting.load(std::memory_order_relaxed)) g_news.fetch_add(1, std::memory_order_relaxed);
    void *p = std::malloc(n ? n : 1);
    if (p == nullptr) throw std::bad_alloc();
    return p;
}
void *counted_aligned(std::size_t n, std::align_val_t a) {
    if (g_counting.load(std::memory_order_relaxed)) g_news.fetch_add(1, std::memory_order_relaxed);
    const std::size_t al = static_cast<std::size_t>(a);
    void *p = std::aligned_alloc(al, (n + al - 1) / al * al);
    if (p == nullptr) throw std::bad_alloc();
    return p;
}
}  // namespace

void *operator new(std::size_t n) { return counted(n); }
void *operator new[](std::size_t n) { return counted(n); }
void *operator new(std::size_t n, std::align_val_t a) { return counted_aligned(n, a); }
void *operator new[](std::size_t n, std::align_val_t a) { return counted_aligned(n, a); }
void operator delete(void *p) noexcept { std::free(p); }
void operator delete[](void *p) noexcept { std::free(p); }
void operator delete(void *p, std::size_t) noexcept { std::free(p); }
void operator delete[](void *p, std::size_t) noexcept { std::free(p); }
void operator delete(void *p, std::align_val_t) noexcept { std::free(p); }
void operator delete[](void *p, std::align_val_t) noexcept { std::free(p); }
void operator delete(void *p, std::size_t, std::align_val_t) noexcept { std::free(p); }
void operator delete[](void *p, std::size_t, std::align_val_t) noexcept { std::free(p); }

namespace {

}  // namespace

TEST(api_post_poll_hot_path_does_not_allocate) {
    th::DaemonProc d;
    if (!d.start()) {
        std::fprintf(stderr, "  (skipped: ugdr_daemon not found next to the test binary)\n");
        return;
    }
    ::setenv("UGDR_DAEMON_SOCKET", d.sock.c_str(), 1);
    int n = 0;
    // The counter sees the library's allocations (this binary's operator new interposes it).
    g_news.store(0);
    g_counting.store(true);
    ugdr_device **list = ugdr_get_device_list(&n);
    g_counting.store(false);
    CHECK(g_news.load() > 0);
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
    ugdr_pd *pd = ugdr_alloc_pd(ctx);
    ugdr_cq *cq = ugdr_create_cq(ctx, 256, nullptr, nullptr, 0);
    void *buf = ugdr_x_alloc_host(1 << 16);
    ugdr_mr *mr = ugdr_reg_mr(pd, buf, 1 << 16, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE);
    ugdr_qp_init_attr ia{cq, cq, 64, 16, 1, 1, UGDR_QPT_RC, 0};
    ugdr_qp *a = ugdr_create_qp(pd, &ia), *b = ugdr_create_qp(pd, &ia);
    CHECK(ctx && pd && cq && buf && mr && a && b);
    if (!(ctx && pd && cq && buf && mr && a && b)) return;
    ugdr_qp_attr at{};
    at.qp_state = UGDR_QPS_INIT;
    at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE;
    CHECK_EQ(ugdr_modify_qp(a, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS), 0);
    CHECK_EQ(ugdr_modify_qp(b, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS), 0);
    ugdr_qp_conn_info ca{}, cb{};
    ugdr_query_qp_conn_info(a, &ca);
    ugdr_query_qp_conn_info(b, &cb);
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    const int cm = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    CHECK_EQ(ugdr_connect_qp(a, &cb, &c, cm), 0);
    CHECK_EQ(ugdr_connect_qp(b, &ca, &c, cm), 0);

    ugdr_sge sg{reinterpret_cast<uint64_t>(buf), 8, mr->lkey};
    ugdr_send_wr wr{};
    wr.sg_list = &sg;
    wr.num_sge = 1;
    wr.opcode = UGDR_WR_RDMA_WRITE;
    wr.send_flags = UGDR_SEND_SIGNALED;
    wr.wr.rdma.remote_addr = reinterpret_cast<uint64_t>(buf) + 4096;
    wr.wr.rdma.rkey = mr->rkey;
    ugdr_wc wc[4];
    auto one = [&](uint64_t id) {
        wr.wr_id = id;
        ugdr_send_wr *bad = nullptr;
        if (ugdr_post_send(a, &wr, &bad) != 0) return false;
        const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(10);
        for (;;) {
            const int k = ugdr_poll_cq(cq, 4, wc);
            if (k == 1) return wc[0].status == UGDR_WC_SUCCESS && wc[0].wr_id == id;
            if (k != 0 || std::chrono::steady_clock::now() > deadline) return false;
        }
    };
    bool ok = true;
    for (uint64_t i = 0; i < 64 && ok; ++i) ok = one(i);  // warm-up
    CHECK(ok);
    g_news.store(0);
    g_counting.store(true);
    for (uint64_t i = 64; i < 1064 && ok; ++i) ok = one(i);
    g_counting.store(false);
    CHECK(ok);
    CHECK_EQ(g_news.load(), 0ull);

    ugdr_destroy_qp(a);
    ugdr_destroy_qp(b);
    ugdr_dereg_mr(mr);
    ugdr_x_free_host(buf);
    ugdr_destroy_cq(cq);
    ugdr_dealloc_pd(pd);
    ugdr_close_device(ctx);
    ugdr_free_device_list(list);
}
