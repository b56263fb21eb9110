// ugdr_perf: verbs-level benchmarks through the public C API (the point-to-point sweep and the WR
// posting rate).  Needs a running ugdr_daemon (UGDR_DAEMON_SOCKET).
//
//   ugdr_perf latency  --src-gpu A --dst-gpu B --bytes N --iters K        QD1 post_send -> poll_cq
//   ugdr_perf bw       --src-gpu A --dst-gpu B --op write|read --min 8 --max 1G --qd 64 --bytes-per-size T
//                      [--trace-size S --trace-out PATH]   device trace of the executor at WR size S
//   ugdr_perf posting  --batch B --wrs N                                    post_send into the SQ ring
//   ugdr_perf ring     --batch B --wrs N                                    shared SPSC ring alone (2 threads)
//   ugdr_perf postcore --batch B --wrs N                                    WR encode + publish path alone
//   ugdr_perf plumbing --wrs 10000                                          CPU-only plumbing (host engine)
//   ugdr_perf control  --src-gpu A|-1 --iters N                             control-plane op latencies
//   ugdr_perf stress   --src-gpu A --dst-gpu B --qps 64 --depth 128 --sges 16 --rounds R
//                      verbs-feature stress: per QP an interleave of
//                      16-SGE WRITE and WRITE_WITH_IMM (SGE sizes log-uniform in 64 B..64 KiB,
//                      gathered into a contiguous remote range), FETCH_ADD and CMP_AND_SWP on a
//                      4096-entry uint64 counter array; checks every byte, immediate, and
//                      atomic result; reports posting and completion rates.
//
// Output: one key=value line per measurement (reference style, benchmarks/*.cpp) and a JSON
// line with the same fields.  Payload: uniform uint8 from a seed; every size's destination is
// compared byte-for-byte with the source once.
#include "api/posting.hpp"
#include "queue/layout.hpp"
#include "queue/ring.hpp"
#include "ugdr/api.hpp"

#include <cuda_runtime_api.h>

#include <dirent.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

namespace {

using Clock = std::chrono::steady_clock;

struct Opts {
    std::string mode = "latency";
    int src_gpu = 0, dst_gpu = 0;
    uint64_t bytes = 8, iters = 20000, warmup = 2000;
    std::string op = "write";
    uint64_t min_bytes = 8, max_bytes = 1ull << 30, qd = 64, bytes_per_size = 8ull << 30;
    uint64_t batch = 32, wrs = 4000000;
    uint64_t qps = 64, depth = 128, sges = 16, rounds = 3, seed = 7;
    uint64_t trace_size = 0;  // bw: keep a device trace of the executor at this WR size
    std::string trace_out;    // ... written here (Chrome trace JSON)
    std::string sync_dir;  // stress: start / finish barrier shared by concurrent clients
    uint64_t sync_n = 0;
};

[[noreturn]] void die(const char *what, int rc) {
    std::fprintf(stderr, "ugdr_perf: %s failed (%d: %s)\n", what, rc, std::strerror(rc > 0 ? rc : -rc));
    std::exit(1);
}

uint64_t parse_size(const char *s) {
    char *end = nullptr;
    double v = std::strtod(s, &end);
    if (end && (*end == 'k' || *end == 'K')) v *= 1024;
    if (end && (*end == 'm' || *end == 'M')) v *= 1024 * 1024;
    if (end && (*end == 'g' || *end == 'G')) v *= 1024.0 * 1024 * 1024;
    return uint64_t(v);
}

struct Side {
    ugdr_context *ctx = nullptr;
    ugdr_pd *pd = nullptr;
    ugdr_cq *cq = nullptr;
    ugdr_qp *qp = nullptr;
    ugdr_mr *mr = nullptr;
    void *buf = nullptr;
};

// `gpu` < 0 selects the host-memory device (buffers from ugdr_x_alloc_host).
ugdr_device *gpu_device(ugdr_device **list, int n, int gpu) {
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (gpu < 0 && ugdr_x_query_device(list[i], &info) == 0 && info.kind == 0) return list[i];
    }
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0 && info.kind == 1 && info.gpu_ordinal == gpu) return list[i];
    }
    std::fprintf(stderr, "ugdr_perf: daemon has no GPU %d\n", gpu);
    std::exit(1);
}

// Requester on src_gpu, responder on dst_gpu, each with an MR of `bytes`.
void setup(const Opts &o, uint64_t bytes, uint32_t depth, Side *a, Side *b) {
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (!list) die("ugdr_get_device_list", errno);
    Side *sides[2] = {a, b};
    const int gpus[2] = {o.src_gpu, o.dst_gpu};
    for (int i = 0; i < 2; ++i) {
        Side &s = *sides[i];
        s.ctx = ugdr_open_device(gpu_device(list, n, gpus[i]));
        if (!s.ctx) die("ugdr_open_device", errno);
        s.pd = ugdr_alloc_pd(s.ctx);
        s.cq = ugdr_create_cq(s.ctx, int(depth * 2 + 16), nullptr, nullptr, 0);
        if (!s.pd || !s.cq) die("pd/cq", errno);
        if (gpus[i] < 0) {
            s.buf = ugdr_x_alloc_host(bytes);
            if (!s.buf) die("ugdr_x_alloc_host", ENOMEM);
        } else {
            cudaSetDevice(gpus[i]);
            if (cudaMalloc(&s.buf, bytes) != cudaSuccess) die("cudaMalloc", ENOMEM);
        }
        s.mr = ugdr_reg_mr(s.pd, s.buf, bytes,
                           UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ);
        if (!s.mr) die("ugdr_reg_mr", errno);
        ugdr_qp_init_attr ia{s.cq, s.cq, depth, depth, 1, 1, UGDR_QPT_RC, 0};
        s.qp = ugdr_create_qp(s.pd, &ia);
        if (!s.qp) die("ugdr_create_qp", errno);
        ugdr_qp_attr at{};
        at.qp_state = UGDR_QPS_INIT;
        at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ;
        if (int rc = ugdr_modify_qp(s.qp, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS)) die("modify INIT", rc);
    }
    ugdr_qp_conn_info ca{}, cb{};
    ugdr_query_qp_conn_info(a->qp, &ca);
    ugdr_query_qp_conn_info(b->qp, &cb);
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    const int mask = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    if (int rc = ugdr_connect_qp(a->qp, &cb, &c, mask)) die("connect a", rc);
    if (int rc = ugdr_connect_qp(b->qp, &ca, &c, mask)) die("connect b", rc);
}

void fill(void *dev, uint64_t bytes, uint64_t seed, int gpu) {
    std::vector<uint8_t> h(std::min<uint64_t>(bytes, 64ull << 20));
    std::mt19937_64 rng(seed);
    for (auto &x : h) x = uint8_t(rng());
    if (gpu >= 0) cudaSetDevice(gpu);
    for (uint64_t off = 0; off < bytes; off += h.size()) {
        const uint64_t k = std::min<uint64_t>(h.size(), bytes - off);
        if (gpu < 0)
            std::memcpy(static_cast<uint8_t *>(dev) + off, h.data(), k);
        else
            cudaMemcpy(static_cast<uint8_t *>(dev) + off, h.data(), k, cudaMemcpyHostToDevice);
    }
}

bool same(const void *a, int ga, const void *b, int gb, uint64_t bytes) {
    const uint64_t n = std::min<uint64_t>(bytes, 16ull << 20);
    std::vector<uint8_t> x(n), y(n);
    auto get = [](std::vector<uint8_t> &out, const void *p, int g, uint64_t k) {
        if (g < 0) {
            std::memcpy(out.data(), p, k);
        } else {
            cudaSetDevice(g);
            cudaMemcpy(out.data(), p, k, cudaMemcpyDeviceToHost);
        }
    };
    get(x, a, ga, n);
    get(y, b, gb, n);
    return x == y;
}

void wait_cq(ugdr_cq *cq, uint64_t want) {
    ugdr_wc wc[64];
    uint64_t got = 0;
    const auto deadline = Clock::now() + std::chrono::seconds(60);
    while (got < want) {
        const int n = ugdr_poll_cq(cq, int(std::min<uint64_t>(64, want - got)), wc);
        if (n < 0) die("ugdr_poll_cq", -n);
        for (int i = 0; i < n; ++i)
            if (wc[i].status != UGDR_WC_SUCCESS) die("work completion", int(wc[i].status));
        got += uint64_t(n);
        if (n == 0 && Clock::now() > deadline) die("completion timeout", ETIMEDOUT);
    }
}

void post(ugdr_qp *qp, int op, void *local, uint32_t lkey, uint64_t bytes, void *remote, uint32_t rkey,
          uint64_t wr_id) {
    ugdr_sge sg{reinterpret_cast<uint64_t>(local), uint32_t(bytes), lkey};
    ugdr_send_wr wr{};
    wr.wr_id = wr_id;
    wr.sg_list = &sg;
    wr.num_sge = 1;
    wr.opcode = ugdr_wr_opcode(op);
    wr.send_flags = UGDR_SEND_SIGNALED;
    wr.wr.rdma.remote_addr = reinterpret_cast<uint64_t>(remote);
    wr.wr.rdma.rkey = rkey;
    ugdr_send_wr *bad = nullptr;
    int rc;
    while ((rc = ugdr_post_send(qp, &wr, &bad)) == ENOMEM) std::this_thread::yield();
    if (rc) die("ugdr_post_send", rc);
}

double pct(std::vector<double> v, double p) {
    std::sort(v.begin(), v.end());
    return v[std::min<size_t>(v.size() - 1, size_t(p * (v.size() - 1) + 0.5))];
}

int run_latency(const Opts &o) {
    Side a, b;
    setup(o, std::max<uint64_t>(o.bytes, 4096), 16, &a, &b);
    fill(a.buf, o.bytes, 1, o.src_gpu);
    std::vector<double> us;
    us.reserve(o.iters);
    ugdr_x_engine_stats es{};
    for (uint64_t i = 0; i < o.warmup + o.iters; ++i) {
        if (i == o.warmup) ugdr_x_query_engine_stats(a.ctx, &es, 1);
        const auto t0 = Clock::now();
        post(a.qp, UGDR_WR_RDMA_WRITE, a.buf, a.mr->lkey, o.bytes, b.buf, b.mr->rkey, i);
        wait_cq(a.cq, 1);
        const double dt = std::chrono::duration<double, std::micro>(Clock::now() - t0).count();
        if (i >= o.warmup) us.push_back(dt);
    }
    const bool ok = same(a.buf, o.src_gpu, b.buf, o.dst_gpu, o.bytes);
    std::printf("benchmark=ugdr_latency op=write bytes=%llu src_gpu=%d dst_gpu=%d iters=%llu p50_us=%.3f "
                "p99_us=%.3f p999_us=%.3f min_us=%.3f correct=%d\n",
                (unsigned long long)o.bytes, o.src_gpu, o.dst_gpu, (unsigned long long)o.iters, pct(us, 0.5),
                pct(us, 0.99), pct(us, 0.999), pct(us, 0.0), int(ok));
    // Executor side of the same WRs (GPU contexts): mean time per fast batch in each phase.
    if (ugdr_x_query_engine_stats(a.ctx, &es, 0) == 0 && es.fast_batches > 0) {
        const double nb = double(es.fast_batches) * 1e3;
        std::printf("executor: batches=%llu fetch_us=%.3f exec_us=%.3f reserve_us=%.3f publish_us=%.3f\n",
                    (unsigned long long)es.fast_batches, es.fast_fetch_ns / nb, es.fast_exec_ns / nb,
                    es.fast_reserve_ns / nb, es.fast_publish_ns / nb);
    }
    std::printf("{\"benchmark\": \"ugdr_latency\", \"bytes\": %llu, \"src_gpu\": %d, \"dst_gpu\": %d, "
                "\"p50_us\": %.3f, \"p99_us\": %.3f, \"correct\": %s}\n",
                (unsigned long long)o.bytes, o.src_gpu, o.dst_gpu, pct(us, 0.5), pct(us, 0.99),
                ok ? "true" : "false");
    return ok ? 0 : 2;
}

int run_bw(const Opts &o) {
    Side a, b;
    const uint32_t qd = uint32_t(o.qd);
    setup(o, o.max_bytes, qd + 4, &a, &b);
    fill(a.buf, o.max_bytes, 2, o.src_gpu);
    fill(b.buf, o.max_bytes, 3, o.dst_gpu);
    const int op = o.op == "read" ? UGDR_WR_RDMA_READ : UGDR_WR_RDMA_WRITE;
    int status = 0;
    for (uint64_t sz = o.min_bytes; sz <= o.max_bytes; sz *= 2) {
        uint64_t wrs = std::max<uint64_t>(qd * 4, o.bytes_per_size / sz);
        wrs = std::min<uint64_t>(wrs, 200000);
        // Warm-up: one window.
        for (uint64_t i = 0; i < qd; ++i) post(a.qp, op, a.buf, a.mr->lkey, sz, b.buf, b.mr->rkey, i);
        wait_cq(a.cq, qd);
        uint64_t posted = 0, done = 0;
        ugdr_wc wc[64];
        std::vector<ugdr_send_wr> chain(qd);
        std::vector<ugdr_sge> chain_sge(qd);
        ugdr_x_engine_stats es{};
        ugdr_x_query_engine_stats(a.ctx, &es, 1);
        const bool tracing = o.trace_size == sz && !o.trace_out.empty();
        if (tracing && ugdr_x_engine_trace(a.ctx, 16384) != 0) die("ugdr_x_engine_trace", EINVAL);
        const auto t0 = Clock::now();
        while (done < wrs) {
            // Bound each size to ~2 s: stop posting and drain what is in flight.
            if (posted < wrs && (posted & 255) == 0 && Clock::now() - t0 > std::chrono::seconds(2)) wrs = posted;
            // Post every free window slot as one chain (one ugdr_post_send call), as the
            // reference's client benchmark does with its post chains.
            uint32_t nchain = 0;
            while (posted + nchain < wrs && posted + nchain - done < qd) {
                // WRs rotate over the buffer's sz-byte slices.  A QP's WRs take effect in posting
                // order, so two in flight on the same slice would run one after the other; with
                // at least 32 slices (the executor's per-QP window) none ever waits for another.
                const uint64_t w = posted + nchain;
                const uint64_t nslices = std::max<uint64_t>(1, o.max_bytes / sz);
                const uint64_t off = (w % nslices) * sz;
                chain_sge[nchain] = ugdr_sge{reinterpret_cast<uint64_t>(static_cast<uint8_t *>(a.buf) + off),
                                             uint32_t(sz), a.mr->lkey};
                ugdr_send_wr &wr = chain[nchain];
                wr = ugdr_send_wr{};
                wr.wr_id = w;
                wr.sg_list = &chain_sge[nchain];
                wr.num_sge = 1;
                wr.opcode = ugdr_wr_opcode(op);
                wr.send_flags = UGDR_SEND_SIGNALED;
                wr.wr.rdma.remote_addr = reinterpret_cast<uint64_t>(static_cast<uint8_t *>(b.buf) + off);
                wr.wr.rdma.rkey = b.mr->rkey;
                if (nchain > 0) chain[nchain - 1].next = &wr;
                ++nchain;
            }
            if (nchain > 0) {
                ugdr_send_wr *bad = nullptr;
                const int rc = ugdr_post_send(a.qp, chain.data(), &bad);
                if (rc != 0 && rc != ENOMEM) die("ugdr_post_send", rc);
                uint32_t accepted = nchain;
                if (rc == ENOMEM) {
                    accepted = 0;
                    for (ugdr_send_wr *x = chain.data(); x != bad; x = x->next) ++accepted;
                }
                posted += accepted;
            }
            const int n = ugdr_poll_cq(a.cq, 64, wc);
            if (n < 0) die("ugdr_poll_cq", -n);
            for (int i = 0; i < n; ++i)
                if (wc[i].status != UGDR_WC_SUCCESS) die("work completion", int(wc[i].status));
            done += uint64_t(n);
        }
        const double s = std::chrono::duration<double>(Clock::now() - t0).count();
        const double gbps = double(wrs) * double(sz) / s / 1e9;
        if (tracing) {
            uint64_t kept = 0, dropped = 0;
            if (ugdr_x_engine_trace_dump(a.ctx, o.trace_out.c_str(), &kept, &dropped) != 0)
                die("ugdr_x_engine_trace_dump", EIO);
            ugdr_x_engine_trace(a.ctx, 0);
            std::fprintf(stderr, "trace: %llu events kept, %llu dropped -> %s\n", (unsigned long long)kept,
                         (unsigned long long)dropped, o.trace_out.c_str());
        }
        const bool ok = op == UGDR_WR_RDMA_WRITE ? same(a.buf, o.src_gpu, b.buf, o.dst_gpu, sz)
                                                 : same(b.buf, o.dst_gpu, a.buf, o.src_gpu, sz);
        if (!ok) status = 2;
        if (ugdr_x_query_engine_stats(a.ctx, &es, 0) == 0)
            std::printf("engine bytes=%llu wrs=%llu jobs=%llu chunks=%llu claim_misses=%llu busy_us=%.1f "
                        "fast_batches=%llu slow_wrs=%llu publish_waits=%llu order_waits=%llu slot_misses=%llu overlap_issues=%llu\n",
                        (unsigned long long)sz, (unsigned long long)es.wrs_completed,
                        (unsigned long long)es.jobs_published, (unsigned long long)es.chunks_run,
                        (unsigned long long)es.claim_misses, double(es.busy_ns) / 1e3,
                        (unsigned long long)es.fast_batches, (unsigned long long)es.slow_wrs,
                        (unsigned long long)es.publish_waits, (unsigned long long)es.order_waits, (unsigned long long)es.job_slot_misses,
                        (unsigned long long)es.overlap_issues);
        std::printf("benchmark=ugdr_bw op=%s bytes=%llu qd=%u src_gpu=%d dst_gpu=%d wrs=%llu seconds=%.6f "
                    "GB_per_s=%.3f MWR_per_s=%.4f correct=%d\n",
                    o.op.c_str(), (unsigned long long)sz, qd, o.src_gpu, o.dst_gpu, (unsigned long long)wrs, s,
                    gbps, double(wrs) / s / 1e6, int(ok));
        std::printf("{\"benchmark\": \"ugdr_bw\", \"op\": \"%s\", \"bytes\": %llu, \"qd\": %u, \"GBps\": %.3f, "
                    "\"MWRps\": %.4f, \"correct\": %s}\n",
                    o.op.c_str(), (unsigned long long)sz, qd, gbps, double(wrs) / s / 1e6, ok ? "true" : "false");
        std::fflush(stdout);
    }
    return status;
}

// Posting rate: the client path alone (validate, encode into the shared SQ ring, publish).  The
// host engine is held while a 16 Ki-slot SQ is filled with 8-byte RDMA WRITEs in chains of
// `batch`; only the ugdr_post_send calls are timed.  Then the engine is released and drains the
// ring (a signaled last WR marks the end) before the next fill.  This is the reference's
// "posting + consume" measurement (benchmarks/queue_metadata_benchmark.cpp) without its consumer
// on the critical path.
int run_posting(const Opts &o) {
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (!list) die("ugdr_get_device_list", errno);
    ugdr_device *cpu = nullptr;
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0 && info.kind == 0) cpu = list[i];
    }
    if (!cpu) die("no host device", ENODEV);
    constexpr uint32_t kDepth = 16384;
    ugdr_context *ctx = ugdr_open_device(cpu);
    ugdr_pd *pd = ugdr_alloc_pd(ctx);
    ugdr_cq *cq = ugdr_create_cq(ctx, 1024, nullptr, nullptr, 0);
    void *buf = ugdr_x_alloc_host(1 << 20);
    ugdr_mr *mr = ugdr_reg_mr(pd, buf, 1 << 20, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE);
    ugdr_qp_init_attr ia{cq, cq, kDepth, 16, 1, 1, UGDR_QPT_RC, 0};
    ugdr_qp *qp = ugdr_create_qp(pd, &ia), *peer = ugdr_create_qp(pd, &ia);
    if (!qp || !peer || !mr) die("posting setup", errno);
    ugdr_qp_attr at{};
    at.qp_state = UGDR_QPS_INIT;
    at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE;
    ugdr_modify_qp(qp, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_modify_qp(peer, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_qp_conn_info ci{};
    ugdr_query_qp_conn_info(peer, &ci);
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    if (int rc = ugdr_connect_qp(qp, &ci, &c, UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY |
                                                UGDR_QP_MIN_RNR_TIMER))
        die("connect", rc);
    const uint32_t batch = uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(o.batch, kDepth)));
    std::vector<ugdr_sge> sg(batch, ugdr_sge{reinterpret_cast<uint64_t>(buf), 8, mr->lkey});
    std::vector<ugdr_send_wr> wr(batch);
    for (uint32_t i = 0; i < batch; ++i) {
        wr[i] = ugdr_send_wr{};
        wr[i].wr_id = i;
        wr[i].sg_list = &sg[i];
        wr[i].num_sge = 1;
        wr[i].opcode = UGDR_WR_RDMA_WRITE;
        wr[i].wr.rdma.remote_addr = reinterpret_cast<uint64_t>(buf) + 64;
        wr[i].wr.rdma.rkey = mr->rkey;
        wr[i].next = i + 1 < batch ? &wr[i + 1] : nullptr;
    }
    ugdr_send_wr last = wr[0];
    last.next = nullptr;
    last.send_flags = UGDR_SEND_SIGNALED;
    uint64_t accepted = 0;
    double posting_s = 0;
    while (accepted < o.wrs) {
        ugdr_x_engine_hold(ctx, 1);
        // Fill all but one slot in chains of `batch` (the last slot takes the signaled marker).
        uint64_t in_ring = 0;
        const auto t0 = Clock::now();
        while (in_ring + batch <= kDepth - 1 && accepted + in_ring < o.wrs) {
            ugdr_send_wr *bad = nullptr;
            const int rc = ugdr_post_send(qp, wr.data(), &bad);
            if (rc != 0) die("ugdr_post_send", rc);
            in_ring += batch;
        }
        posting_s += std::chrono::duration<double>(Clock::now() - t0).count();
        accepted += in_ring;
        ugdr_send_wr *bad = nullptr;
        if (int rc = ugdr_post_send(qp, &last, &bad)) die("ugdr_post_send", rc);
        ugdr_x_engine_hold(ctx, 0);
        wait_cq(cq, 1);
    }
    std::printf("benchmark=ugdr_posting batch=%u wrs=%llu posting_seconds=%.6f MWR_per_s=%.3f ns_per_wr=%.2f\n", batch,
                (unsigned long long)accepted, posting_s, double(accepted) / posting_s / 1e6,
                posting_s * 1e9 / double(accepted));
    std::printf("{\"benchmark\": \"ugdr_posting\", \"batch\": %u, \"MWRps\": %.3f, \"ns_per_wr\": %.2f}\n", batch,
                double(accepted) / posting_s / 1e6, posting_s * 1e9 / double(accepted));
    return 0;
}

// ---- verbs-feature stress ------------------------------------------------------------------------

constexpr uint64_t kCounters = 4096;
constexpr uint64_t kFaaCounters = 2048;  // [0, 2048): fetch-add from every QP
                                          // [2048, 4096): compare-swap chains, owned per QP

struct StressSide {
    ugdr_context *ctx = nullptr;
    ugdr_pd *pd = nullptr;
    ugdr_cq *cq = nullptr;
};

ugdr_device *any_device(ugdr_device **list, int n, int gpu) {
    if (gpu >= 0) return gpu_device(list, n, gpu);
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0 && info.kind == 0) return list[i];
    }
    std::fprintf(stderr, "ugdr_perf: daemon has no host-memory device\n");
    std::exit(1);
}

// Memory of one side: device memory of GPU `gpu`, or (gpu < 0) a ugdr host buffer served by the
// daemon's CPU engine.
void *mem_alloc(int gpu, uint64_t bytes) {
    void *p = nullptr;
    if (gpu < 0) {
        p = ugdr_x_alloc_host(bytes);
        if (!p) die("ugdr_x_alloc_host", errno);
        std::memset(p, 0, bytes);
        return p;
    }
    cudaSetDevice(gpu);
    if (cudaMalloc(&p, bytes) != cudaSuccess) die("cudaMalloc", ENOMEM);
    cudaMemset(p, 0, bytes);
    return p;
}
void mem_zero(int gpu, void *p, uint64_t bytes) {
    if (gpu < 0) {
        std::memset(p, 0, bytes);
        return;
    }
    cudaSetDevice(gpu);
    cudaMemset(p, 0, bytes);
    cudaDeviceSynchronize();
}
void mem_read(int gpu, void *host, const void *p, uint64_t bytes) {
    if (gpu < 0) {
        std::memcpy(host, p, bytes);
        return;
    }
    cudaSetDevice(gpu);
    cudaMemcpy(host, p, bytes, cudaMemcpyDeviceToHost);
}
void mem_write(int gpu, void *p, const void *host, uint64_t bytes) {
    if (gpu < 0) {
        std::memcpy(p, host, bytes);
        return;
    }
    cudaSetDevice(gpu);
    cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice);
}

// Cross-process start / finish barrier for concurrent stress clients: every process creates
// <dir>/<phase>.<pid> and waits (bounded) until `n` such files exist.
void sync_phase(const std::string &dir, uint64_t n, const char *phase) {
    if (dir.empty() || n <= 1) return;
    const std::string mine = dir + "/" + phase + "." + std::to_string(getpid());
    if (FILE *f = std::fopen(mine.c_str(), "w")) std::fclose(f);
    const auto deadline = Clock::now() + std::chrono::seconds(600);
    for (;;) {
        uint64_t seen = 0;
        if (DIR *d = opendir(dir.c_str())) {
            const size_t pl = std::strlen(phase);
            while (dirent *e = readdir(d))
                if (std::strncmp(e->d_name, phase, pl) == 0 && e->d_name[pl] == '.') ++seen;
            closedir(d);
        }
        if (seen >= n) return;
        if (Clock::now() > deadline) die("stress sync barrier", ETIMEDOUT);
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
}

StressSide open_side(ugdr_device **list, int n, int gpu, int cqe) {
    StressSide s;
    s.ctx = ugdr_open_device(any_device(list, n, gpu));
    if (!s.ctx) die("ugdr_open_device", errno);
    s.pd = ugdr_alloc_pd(s.ctx);
    s.cq = ugdr_create_cq(s.ctx, cqe, nullptr, nullptr, 0);
    if (!s.pd || !s.cq) die("pd/cq", errno);
    return s;
}

ugdr_mr *dev_mr(ugdr_pd *pd, int gpu, uint64_t bytes, int access, void **buf) {
    *buf = mem_alloc(gpu, bytes);
    ugdr_mr *mr = ugdr_reg_mr(pd, *buf, bytes, access);
    if (!mr) die("ugdr_reg_mr", errno);
    return mr;
}

// ---- shared ring alone -------------------------------------------------------------------------

// Descriptor rate of the shared SPSC ring with no daemon: a producer thread reserves up to `batch`
// slots, writes the first 16 bytes of each 64-byte slot and publishes them; a consumer thread
// peeks up to `batch` slots, reads and releases them.  As in the reference counterpart
// (benchmarks/shared_ring_benchmark.cpp: its reserve and peek return what is there, EAGAIN only
// when that is nothing), a shorter run is taken as it is rather than waited for.
int run_ring(const Opts &o) {
    // Each side's ring view (its private cursor copies) on its own cache lines, as in real use
    // where producer and consumer are different processes.
    struct alignas(128) Side {
        ugdr::queue::Ring r;
    };
    Side ps, cs;
    ugdr::queue::Ring &prod = ps.r, &cons = cs.r;
    const ugdr::queue::RingGeometry g{ugdr::queue::kSendRing, 4096, 64};
    if (int rc = ugdr::queue::Ring::create(g, &prod)) die("ring create", rc);
    if (int rc = ugdr::queue::Ring::attach(::dup(prod.fd()), g, &cons)) die("ring attach", rc);
    const uint32_t batch = uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(o.batch, 4096)));
    const uint64_t total = o.wrs;
    std::atomic<uint64_t> checksum{0};
    const auto t0 = Clock::now();
    std::thread consumer([&] {
        uint64_t got = 0, sum = 0;
        while (got < total) {
            const uint32_t want = uint32_t(std::min<uint64_t>(batch, total - got));
            ugdr::queue::SlotRun r = cons.peek(want);
            const uint32_t n = r.count();
            if (n == 0) continue;
            for (uint32_t i = 0; i < n; ++i) {
                const uint8_t *slot = i < r.first_count ? r.first + uint64_t(i) * 64 : r.second + uint64_t(i - r.first_count) * 64;
                uint64_t v;
                std::memcpy(&v, slot, 8);
                sum += v;
            }
            cons.release(n);
            got += n;
        }
        checksum.store(sum);
    });
    uint64_t sent = 0;
    while (sent < total) {
        const uint32_t want = uint32_t(std::min<uint64_t>(batch, total - sent));
        ugdr::queue::SlotRun r = prod.reserve(want);
        const uint32_t n = r.count();
        if (n == 0) continue;
        for (uint32_t i = 0; i < n; ++i) {
            uint8_t *slot = i < r.first_count ? r.first + uint64_t(i) * 64 : r.second + uint64_t(i - r.first_count) * 64;
            const uint64_t v = sent + i;
            std::memcpy(slot, &v, 8);
            std::memcpy(slot + 8, &v, 8);
        }
        prod.publish(n);
        sent += n;
    }
    consumer.join();
    const double sec = std::chrono::duration<double>(Clock::now() - t0).count();
    const bool ok = checksum.load() == total * (total - 1) / 2;
    std::printf("benchmark=ugdr_ring batch=%u descriptors=%llu seconds=%.6f M_per_s=%.3f correct=%d\n", batch,
                (unsigned long long)total, sec, double(total) / sec / 1e6, int(ok));
    std::printf("{\"benchmark\": \"ugdr_ring\", \"batch\": %u, \"M_per_s\": %.3f, \"correct\": %s}\n", batch,
                double(total) / sec / 1e6, ok ? "true" : "false");
    return ok ? 0 : 2;
}

// Posting core without the public API's per-call checks: chains of `batch` zero-SGE RDMA WRITEs
// encoded by the library's posting routine into a 64-slot send ring, consumed in the same thread
// right after each chain (the ring stays in L1).  Same setup as the reference's
// benchmarks/wr_posting_benchmark.cpp, so the two numbers compare directly.
int run_postcore(const Opts &o) {
    ugdr::queue::Ring prod, cons;
    const ugdr::queue::RingGeometry g{ugdr::queue::kSendRing, 64, ugdr::queue::send_stride(1)};
    if (int rc = ugdr::queue::Ring::create(g, &prod)) die("ring create", rc);
    if (int rc = ugdr::queue::Ring::attach(::dup(prod.fd()), g, &cons)) die("ring attach", rc);
    const uint32_t batch = uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(o.batch, 64)));
    std::vector<ugdr_send_wr> wr(batch);
    for (uint32_t i = 0; i < batch; ++i) {
        wr[i] = ugdr_send_wr{};
        wr[i].wr_id = i;
        wr[i].opcode = UGDR_WR_RDMA_WRITE;
        wr[i].next = i + 1 < batch ? &wr[i + 1] : nullptr;
    }
    const uint64_t iters = std::max<uint64_t>(1, o.wrs / batch);
    const auto t0 = Clock::now();
    for (uint64_t it = 0; it < iters; ++it) {
        ugdr_send_wr *bad = nullptr;
        if (ugdr::api::post_send_chain(prod, 1, wr.data(), &bad) != 0) die("post_send_chain", EIO);
        if (cons.peek(batch).count() != batch) die("ring peek", EIO);
        cons.release(batch);
    }
    const double sec = std::chrono::duration<double>(Clock::now() - t0).count();
    const double rate = double(iters * batch) / sec / 1e6;
    std::printf("benchmark=ugdr_postcore batch=%u wrs=%llu seconds=%.6f MWR_per_s=%.3f\n", batch,
                (unsigned long long)(iters * batch), sec, rate);
    std::printf("{\"benchmark\": \"ugdr_postcore\", \"batch\": %u, \"MWRps\": %.3f}\n", batch, rate);
    return 0;
}

// ---- control-plane operation costs ------------------------------------------------------------

// Round trips of the object life cycle through the public API on one device (`--src-gpu`, -1 for
// the host-memory device): CQ create / destroy, QP create / destroy, RESET->INIT->RTS (modify +
// connect of a pair), MR register / deregister of a 64 KiB range, query_qp.  Each is timed
// per call over `iters` repetitions after a warm-up; p50 / p99 in microseconds.
int run_control(const Opts &o) {
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (!list) die("ugdr_get_device_list", errno);
    ugdr_context *ctx = ugdr_open_device(any_device(list, n, o.src_gpu));
    ugdr_pd *pd = ugdr_alloc_pd(ctx);
    ugdr_cq *cq = ugdr_create_cq(ctx, 256, nullptr, nullptr, 0);
    const size_t bytes = 1 << 16;
    void *buf = nullptr;
    if (o.src_gpu < 0) {
        buf = ugdr_x_alloc_host(bytes);
    } else if (cudaSetDevice(o.src_gpu) != cudaSuccess || cudaMalloc(&buf, bytes) != cudaSuccess) {
        buf = nullptr;
    }
    if (!ctx || !pd || !cq || !buf) die("control setup", errno);
    const uint64_t iters = o.iters > 0 ? o.iters : 2000;
    using Op = std::pair<const char *, std::vector<double>>;
    std::vector<Op> ops = {{"cq_create", {}}, {"cq_destroy", {}}, {"qp_create", {}}, {"qp_destroy", {}},
                           {"qp_connect_pair", {}}, {"mr_register", {}}, {"mr_deregister", {}}, {"query_qp", {}}};
    auto timed = [](std::vector<double> &v, auto &&fn) {
        const auto t0 = Clock::now();
        fn();
        v.push_back(std::chrono::duration<double, std::micro>(Clock::now() - t0).count());
    };
    const uint64_t warm = iters / 10 + 10;
    for (uint64_t i = 0; i < warm + iters; ++i) {
        const bool keep = i >= warm;
        std::vector<double> sink;
        auto sel = [&](size_t k) -> std::vector<double> & { return keep ? ops[k].second : sink; };
        ugdr_cq *c = nullptr;
        timed(sel(0), [&] { c = ugdr_create_cq(ctx, 256, nullptr, nullptr, 0); });
        if (!c) die("ugdr_create_cq", errno);
        timed(sel(1), [&] { ugdr_destroy_cq(c); });
        ugdr_qp_init_attr ia{cq, cq, 128, 128, 1, 1, UGDR_QPT_RC, 0};
        ugdr_qp *a = nullptr, *b = nullptr;
        timed(sel(2), [&] { a = ugdr_create_qp(pd, &ia); });
        b = ugdr_create_qp(pd, &ia);
        if (!a || !b) die("ugdr_create_qp", errno);
        timed(sel(4), [&] {
            ugdr_qp_attr at{};
            at.qp_state = UGDR_QPS_INIT;
            at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE;
            ugdr_modify_qp(a, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
            ugdr_modify_qp(b, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
            ugdr_qp_conn_info ca{}, cb{};
            ugdr_query_qp_conn_info(a, &ca);
            ugdr_query_qp_conn_info(b, &cb);
            ugdr_qp_attr c2{};
            c2.timeout = 14;
            c2.retry_cnt = 7;
            c2.rnr_retry = 7;
            c2.min_rnr_timer = 1;
            const int cm = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
            if (ugdr_connect_qp(a, &cb, &c2, cm) != 0 || ugdr_connect_qp(b, &ca, &c2, cm) != 0) die("connect", EINVAL);
        });
        timed(sel(7), [&] {
            ugdr_qp_attr qa{};
            ugdr_qp_init_attr qi{};
            ugdr_query_qp(a, &qa, UGDR_QP_STATE, &qi);
        });
        timed(sel(3), [&] { ugdr_destroy_qp(a); });
        ugdr_destroy_qp(b);
        ugdr_mr *m = nullptr;
        timed(sel(5), [&] { m = ugdr_reg_mr(pd, buf, bytes, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE); });
        if (!m) die("ugdr_reg_mr", errno);
        timed(sel(6), [&] { ugdr_dereg_mr(m); });
    }
    std::printf("{\"benchmark\": \"ugdr_control\", \"device\": %d, \"iters\": %llu", o.src_gpu,
                (unsigned long long)iters);
    for (auto &op : ops) {
        std::sort(op.second.begin(), op.second.end());
        const double p50 = op.second[op.second.size() / 2], p99 = op.second[op.second.size() * 99 / 100];
        std::printf(", \"%s_p50_us\": %.2f, \"%s_p99_us\": %.2f", op.first, p50, op.first, p99);
    }
    std::printf("}\n");
    ugdr_destroy_cq(cq);
    ugdr_dealloc_pd(pd);
    ugdr_close_device(ctx);
    ugdr_free_device_list(list);
    return 0;
}

// ---- CPU-only plumbing workload -------------------------------------------------------

// One client and the daemon's host-memory engine: 1 PD, two 1 MiB host MRs, one QP of depth
// 128, one CQ; `wrs` RDMA_WRITEs of one 4 KiB SGE at seeded random 4 KiB-aligned offsets, with
// payload bytes uniform from seed 0; the CQ is polled until every completion arrives and the
// destination is checked against a host model of the same writes.
int run_plumbing(const Opts &o) {
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (!list) die("ugdr_get_device_list", errno);
    ugdr_context *ctx = ugdr_open_device(any_device(list, n, -1));
    ugdr_pd *pd = ugdr_alloc_pd(ctx);
    ugdr_cq *cq = ugdr_create_cq(ctx, 256, nullptr, nullptr, 0);
    constexpr uint64_t kMr = 1 << 20, kWr = 4096;
    uint8_t *src = static_cast<uint8_t *>(ugdr_x_alloc_host(kMr));
    uint8_t *dst = static_cast<uint8_t *>(ugdr_x_alloc_host(kMr));
    if (!ctx || !pd || !cq || !src || !dst) die("plumbing setup", errno);
    std::mt19937_64 rng(0);
    for (uint64_t i = 0; i < kMr; ++i) src[i] = uint8_t(rng());
    std::memset(dst, 0, kMr);
    ugdr_mr *smr = ugdr_reg_mr(pd, src, kMr, UGDR_ACCESS_LOCAL_WRITE);
    ugdr_mr *dmr = ugdr_reg_mr(pd, dst, kMr, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE);
    ugdr_qp_init_attr ia{cq, cq, 128, 16, 1, 1, UGDR_QPT_RC, 0};
    ugdr_qp *qp = ugdr_create_qp(pd, &ia), *peer = ugdr_create_qp(pd, &ia);
    if (!smr || !dmr || !qp || !peer) die("plumbing setup", errno);
    ugdr_qp_attr at{};
    at.qp_state = UGDR_QPS_INIT;
    at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE;
    ugdr_modify_qp(qp, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_modify_qp(peer, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_qp_conn_info ci{}, cj{};
    ugdr_query_qp_conn_info(peer, &ci);
    ugdr_query_qp_conn_info(qp, &cj);
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    const int cm = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    if (ugdr_connect_qp(qp, &ci, &c, cm) || ugdr_connect_qp(peer, &cj, &c, cm)) die("connect", EINVAL);
    const uint64_t total = o.wrs;
    std::vector<uint64_t> soff(total), doff(total);
    std::vector<uint8_t> model(kMr, 0);
    std::mt19937_64 pick(1);
    for (uint64_t i = 0; i < total; ++i) {
        soff[i] = (pick() % (kMr / kWr)) * kWr;
        doff[i] = (pick() % (kMr / kWr)) * kWr;
        std::memcpy(model.data() + doff[i], src + soff[i], kWr);
    }
    uint64_t posted = 0, done = 0;
    ugdr_wc wc[64];
    const auto t0 = Clock::now();
    while (done < total) {
        while (posted < total && posted - done < 128) {
            post(qp, UGDR_WR_RDMA_WRITE, src + soff[posted], smr->lkey, kWr, dst + doff[posted], dmr->rkey, posted);
            ++posted;
        }
        const int k = ugdr_poll_cq(cq, 64, wc);
        if (k < 0) die("ugdr_poll_cq", -k);
        for (int i = 0; i < k; ++i)
            if (wc[i].status != UGDR_WC_SUCCESS) die("work completion", int(wc[i].status));
        done += uint64_t(k);
    }
    const double sec = std::chrono::duration<double>(Clock::now() - t0).count();
    const bool ok = std::memcmp(model.data(), dst, kMr) == 0;
    std::printf("benchmark=ugdr_plumbing wrs=%llu wr_bytes=4096 qd=128 seconds=%.6f MWR_per_s=%.4f GB_per_s=%.3f "
                "correct=%d\n", (unsigned long long)total, sec, double(total) / sec / 1e6,
                double(total) * kWr / sec / 1e9, int(ok));
    std::printf("{\"benchmark\": \"ugdr_plumbing\", \"wrs\": %llu, \"MWRps\": %.4f, \"GBps\": %.3f, "
                "\"correct\": %s}\n", (unsigned long long)total, double(total) / sec / 1e6,
                double(total) * kWr / sec / 1e9, ok ? "true" : "false");
    return ok ? 0 : 2;
}

int run_stress(const Opts &o) {
    const uint32_t nq = uint32_t(o.qps), depth = uint32_t(o.depth), nsge = uint32_t(o.sges);
    if (nq == 0 || nq > 64 || depth == 0 || nsge == 0 || nsge > 32) die("stress options", EINVAL);
    const uint64_t per_round = uint64_t(nq) * depth;
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (!list) die("ugdr_get_device_list", errno);
    StressSide rq = open_side(list, n, o.src_gpu, int(per_round + 64));
    StressSide rs = open_side(list, n, o.dst_gpu, int(per_round + 64));
    // Requester memory: gather source (seeded bytes) and atomic results.
    const uint64_t src_bytes = 64ull << 20;
    void *src = nullptr, *res = nullptr, *dst = nullptr, *ctr = nullptr;
    ugdr_mr *src_mr = dev_mr(rq.pd, o.src_gpu, src_bytes, UGDR_ACCESS_LOCAL_WRITE, &src);
    ugdr_mr *res_mr = dev_mr(rq.pd, o.src_gpu, per_round * 8, UGDR_ACCESS_LOCAL_WRITE, &res);
    std::vector<uint8_t> host_src(src_bytes);
    {
        std::mt19937_64 fr(o.seed);
        for (auto &x : host_src) x = uint8_t(fr());
    }
    mem_write(o.src_gpu, src, host_src.data(), src_bytes);
    // Responder memory: gather destination (sized for the largest possible round) and counters.
    const uint64_t dst_bytes = per_round * nsge * 65536ull / 2 + (1 << 20);
    ugdr_mr *dst_mr = dev_mr(rs.pd, o.dst_gpu, dst_bytes, UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE, &dst);
    ugdr_mr *ctr_mr = dev_mr(rs.pd, o.dst_gpu, kCounters * 8,
                             UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_ATOMIC, &ctr);
    // QP pairs.
    std::vector<ugdr_qp *> req(nq), rsp(nq);
    ugdr_qp_attr c{};
    c.timeout = 14;
    c.retry_cnt = 7;
    c.rnr_retry = 7;
    c.min_rnr_timer = 1;
    const int cmask = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    for (uint32_t q = 0; q < nq; ++q) {
        ugdr_qp_init_attr a{rq.cq, rq.cq, depth, 4, nsge, 1, UGDR_QPT_RC, 0};
        ugdr_qp_init_attr b{rs.cq, rs.cq, 4, depth, 1, 1, UGDR_QPT_RC, 0};
        req[q] = ugdr_create_qp(rq.pd, &a);
        rsp[q] = ugdr_create_qp(rs.pd, &b);
        if (!req[q] || !rsp[q]) die("ugdr_create_qp", errno);
        ugdr_qp_attr at{};
        at.qp_state = UGDR_QPS_INIT;
        at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_ATOMIC;
        if (int rc = ugdr_modify_qp(req[q], &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS)) die("modify", rc);
        if (int rc = ugdr_modify_qp(rsp[q], &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS)) die("modify", rc);
        ugdr_qp_conn_info ia{}, ib{};
        ugdr_query_qp_conn_info(req[q], &ia);
        ugdr_query_qp_conn_info(rsp[q], &ib);
        if (int rc = ugdr_connect_qp(req[q], &ib, &c, cmask)) die("connect", rc);
        if (int rc = ugdr_connect_qp(rsp[q], &ia, &c, cmask)) die("connect", rc);
    }

    ugdr_x_engine_stats es{};
    ugdr_x_query_engine_stats(rq.ctx, &es, 1);  // reset the requester engine's counters
    std::mt19937_64 rng(o.seed * 1000003ull + 17);
    auto log_uniform = [&](uint64_t lo, uint64_t hi) {
        const double u = std::uniform_real_distribution<double>(std::log(double(lo)), std::log(double(hi) + 1))(rng);
        return std::min<uint64_t>(hi, std::max<uint64_t>(lo, uint64_t(std::exp(u))));
    };
    std::vector<uint64_t> faa_expect(kCounters, 0), cas_seen(kCounters, 0);
    bool ok = true;
    uint64_t bad_bytes = 0, bad_imm = 0, bad_cas = 0, bad_wc = 0, total_wrs = 0, total_bytes = 0;
    double post_s = 0, run_s = 0;
    std::vector<ugdr_sge> sges(per_round * nsge);
    std::vector<ugdr_send_wr> wrs(per_round);
    std::vector<ugdr_recv_wr> rwrs(per_round);
    std::vector<uint64_t> cas_expect(per_round, ~0ull);
    std::vector<uint8_t> expect;
    for (uint64_t round = 0; round < o.rounds; ++round) {
        // ---- build the round ----
        uint64_t dst_off = 0;
        expect.clear();
        struct Span { uint64_t dst, len; };
        std::vector<Span> spans;
        std::vector<uint64_t> imm_of(per_round, 0);
        uint64_t nimm = 0;
        for (uint32_t q = 0; q < nq; ++q) {
            for (uint32_t i = 0; i < depth; ++i) {
                const uint64_t w = uint64_t(q) * depth + i;
                ugdr_send_wr &wr = wrs[w];
                wr = ugdr_send_wr{};
                wr.wr_id = (round << 40) | w;
                wr.send_flags = UGDR_SEND_SIGNALED;
                wr.next = i + 1 < depth ? &wrs[w + 1] : nullptr;
                ugdr_sge *sg = &sges[w * nsge];
                const uint32_t kind = (q + i) % 4;
                if (kind <= 1) {  // 16-SGE gather: WRITE, or WRITE_WITH_IMM
                    const uint64_t start = dst_off;
                    for (uint32_t k = 0; k < nsge; ++k) {
                        const uint64_t len = log_uniform(64, 65536);
                        const uint64_t off = std::uniform_int_distribution<uint64_t>(0, src_bytes - len)(rng);
                        sg[k] = ugdr_sge{reinterpret_cast<uint64_t>(src) + off, uint32_t(len), src_mr->lkey};
                        expect.insert(expect.end(), host_src.begin() + off, host_src.begin() + off + len);
                        dst_off += len;
                    }
                    spans.push_back({start, dst_off - start});
                    dst_off = (dst_off + 63) & ~63ull;  // next WR's range starts on a fresh line
                    expect.resize(dst_off, 0);
                    wr.sg_list = sg;
                    wr.num_sge = int(nsge);
                    wr.opcode = kind == 0 ? UGDR_WR_RDMA_WRITE : UGDR_WR_RDMA_WRITE_WITH_IMM;
                    wr.wr.rdma.remote_addr = reinterpret_cast<uint64_t>(dst) + start;
                    wr.wr.rdma.rkey = dst_mr->rkey;
                    if (kind == 1) {
                        wr.imm_data = uint32_t(rng());
                        imm_of[w] = wr.imm_data | (1ull << 32);
                        ++nimm;
                    }
                    total_bytes += dst_off - start;
                } else {
                    sg[0] = ugdr_sge{reinterpret_cast<uint64_t>(res) + w * 8, 8, res_mr->lkey};
                    wr.sg_list = sg;
                    wr.num_sge = 1;
                    uint64_t idx;
                    if (kind == 2) {
                        idx = rng() % kFaaCounters;
                        const uint64_t add = 1 + rng() % 7;
                        faa_expect[idx] += add;
                        wr.opcode = UGDR_WR_ATOMIC_FETCH_AND_ADD;
                        wr.wr.atomic.compare_add = add;
                    } else {
                        // QP q owns counters [2048 + 32 q, 2048 + 32 q + 32): its CAS chain on each
                        // is in posting order, so every old value is known in advance.
                        idx = kFaaCounters + (uint64_t(q) * 32 + rng() % 32) % (kCounters - kFaaCounters);
                        wr.opcode = UGDR_WR_ATOMIC_CMP_AND_SWP;
                        wr.wr.atomic.compare_add = cas_seen[idx];
                        wr.wr.atomic.swap = cas_seen[idx] + 1;
                        cas_expect[w] = cas_seen[idx];
                        cas_seen[idx] += 1;
                    }
                    wr.wr.atomic.remote_addr = reinterpret_cast<uint64_t>(ctr) + idx * 8;
                    wr.wr.atomic.rkey = ctr_mr->rkey;
                }
            }
        }
        if (dst_off > dst_bytes) die("stress destination too small", ENOMEM);
        // Receive WRs for the immediates (no SGE: WRITE_WITH_IMM lands at its remote address).
        for (uint32_t q = 0; q < nq; ++q) {
            uint32_t k = 0;
            for (uint32_t i = 0; i < depth; ++i)
                if ((q + i) % 4 == 1) {
                    ugdr_recv_wr &r = rwrs[uint64_t(q) * depth + k];
                    r = ugdr_recv_wr{};
                    r.wr_id = (round << 40) | (uint64_t(q) * depth + i);
                    r.num_sge = 0;
                    r.next = nullptr;
                    if (k > 0) rwrs[uint64_t(q) * depth + k - 1].next = &r;
                    ++k;
                }
            ugdr_recv_wr *bad = nullptr;
            if (k > 0)
                if (int rc = ugdr_post_recv(rsp[q], &rwrs[uint64_t(q) * depth], &bad)) die("ugdr_post_recv", rc);
        }
        mem_zero(o.dst_gpu, dst, dst_off);
        if (round == 0) sync_phase(o.sync_dir, o.sync_n, "ready");
        // ---- post (timed: the posting rate) and complete (timed: the completion rate) ----
        const auto t0 = Clock::now();
        for (uint32_t q = 0; q < nq; ++q) {
            ugdr_send_wr *bad = nullptr;
            if (int rc = ugdr_post_send(req[q], &wrs[uint64_t(q) * depth], &bad)) die("ugdr_post_send", rc);
        }
        const auto t1 = Clock::now();
        ugdr_wc wc[64];
        uint64_t got = 0, got_recv = 0;
        const auto deadline = t1 + std::chrono::seconds(120);
        while (got < per_round || got_recv < nimm) {
            int k = ugdr_poll_cq(rq.cq, 64, wc);
            if (k < 0) die("ugdr_poll_cq", -k);
            for (int j = 0; j < k; ++j) {
                if (wc[j].status != UGDR_WC_SUCCESS) ++bad_wc;
            }
            got += uint64_t(k);
            k = ugdr_poll_cq(rs.cq, 64, wc);
            if (k < 0) die("ugdr_poll_cq", -k);
            for (int j = 0; j < k; ++j) {
                const uint64_t w = wc[j].wr_id & ((1ull << 40) - 1);
                if (wc[j].status != UGDR_WC_SUCCESS || wc[j].opcode != UGDR_WC_RECV_RDMA_WITH_IMM ||
                    !(wc[j].wc_flags & UGDR_WC_WITH_IMM) || w >= per_round || imm_of[w] != (wc[j].imm_data | (1ull << 32)))
                    ++bad_imm;
            }
            got_recv += uint64_t(k);
            if (Clock::now() > deadline) {
                std::fprintf(stderr, "ugdr_perf: stress round %llu: %llu of %llu send and %llu of %llu receive "
                             "completions\n", (unsigned long long)round, (unsigned long long)got,
                             (unsigned long long)per_round, (unsigned long long)got_recv, (unsigned long long)nimm);
                die("stress completion timeout", ETIMEDOUT);
            }
        }
        const auto t2 = Clock::now();
        post_s += std::chrono::duration<double>(t1 - t0).count();
        run_s += std::chrono::duration<double>(t2 - t0).count();
        total_wrs += per_round;
        // Compare-swap results: each old value is the chain position known at build time.
        std::vector<uint64_t> olds(per_round);
        mem_read(o.src_gpu, olds.data(), res, per_round * 8);
        for (uint64_t w = 0; w < per_round; ++w)
            if (cas_expect[w] != ~0ull && olds[w] != cas_expect[w]) ++bad_cas;
        std::fill(cas_expect.begin(), cas_expect.end(), ~0ull);
        // ---- verify every gathered byte ----
        std::vector<uint8_t> got_dst(dst_off);
        mem_read(o.dst_gpu, got_dst.data(), dst, dst_off);
        for (const Span &sp : spans)
            if (std::memcmp(got_dst.data() + sp.dst, expect.data() + sp.dst, sp.len) != 0) bad_bytes += 1;
    }
    // Counters: fetch-add sums and compare-swap chain lengths.
    std::vector<uint64_t> ctr_host(kCounters);
    mem_read(o.dst_gpu, ctr_host.data(), ctr, kCounters * 8);
    uint64_t bad_ctr = 0;
    for (uint64_t i = 0; i < kCounters; ++i)
        if (ctr_host[i] != (i < kFaaCounters ? faa_expect[i] : cas_seen[i])) ++bad_ctr;
    ok = bad_bytes == 0 && bad_imm == 0 && bad_cas == 0 && bad_wc == 0 && bad_ctr == 0;
    if (ugdr_x_query_engine_stats(rq.ctx, &es, 0) == 0)
        std::printf("engine src_gpu=%d wrs=%llu jobs=%llu chunks=%llu claim_misses=%llu inline=%llu slow_wrs=%llu "
                    "slow_issue_us_avg=%.3f job_slot_misses=%llu publish_waits=%llu publish_wait_us_avg=%.3f "
                    "launches=%llu wait_timeouts=%llu\n",
                    o.src_gpu, (unsigned long long)es.wrs_completed, (unsigned long long)es.jobs_published,
                    (unsigned long long)es.chunks_run, (unsigned long long)es.claim_misses,
                    (unsigned long long)es.inline_runs, (unsigned long long)es.slow_wrs,
                    es.slow_wrs ? double(es.slow_issue_ns) / es.slow_wrs / 1e3 : 0.0,
                    (unsigned long long)es.job_slot_misses, (unsigned long long)es.publish_waits,
                    es.publish_waits ? double(es.publish_wait_ns) / es.publish_waits / 1e3 : 0.0,
                    (unsigned long long)es.launches, (unsigned long long)es.wait_timeouts);
    const double post_mops = double(total_wrs) / post_s / 1e6, run_mops = double(total_wrs) / run_s / 1e6;
    std::printf("benchmark=ugdr_stress src_gpu=%d dst_gpu=%d qps=%u depth=%u sges=%u rounds=%llu wrs=%llu "
                "post_MWR_per_s=%.3f complete_MWR_per_s=%.3f GB_per_s=%.3f bad_wrs=%llu bad_imm=%llu bad_cas=%llu "
                "bad_counters=%llu bad_wc=%llu correct=%d\n",
                o.src_gpu, o.dst_gpu, nq, depth, nsge, (unsigned long long)o.rounds, (unsigned long long)total_wrs,
                post_mops, run_mops, double(total_bytes) / run_s / 1e9, (unsigned long long)bad_bytes,
                (unsigned long long)bad_imm, (unsigned long long)bad_cas, (unsigned long long)bad_ctr,
                (unsigned long long)bad_wc, int(ok));
    std::printf("{\"benchmark\": \"ugdr_stress\", \"src_gpu\": %d, \"dst_gpu\": %d, \"qps\": %u, \"depth\": %u, "
                "\"sges\": %u, \"wrs\": %llu, \"post_MWRps\": %.3f, \"complete_MWRps\": %.3f, \"GBps\": %.3f, "
                "\"correct\": %s}\n",
                o.src_gpu, o.dst_gpu, nq, depth, nsge, (unsigned long long)total_wrs, post_mops, run_mops,
                double(total_bytes) / run_s / 1e9, ok ? "true" : "false");
    std::fflush(stdout);
    sync_phase(o.sync_dir, o.sync_n, "done");  // nobody tears down while others still run
    return ok ? 0 : 2;
}

}  // namespace

int main(int argc, char **argv) {
    Opts o;
    if (argc < 2) {
        std::fprintf(stderr, "usage: ugdr_perf latency|bw|posting [options]\n");
        return 2;
    }
    o.mode = argv[1];
    for (int i = 2; i + 1 < argc; i += 2) {
        const std::string k = argv[i];
        const char *v = argv[i + 1];
        if (k == "--src-gpu") o.src_gpu = std::atoi(v);
        else if (k == "--dst-gpu") o.dst_gpu = std::atoi(v);
        else if (k == "--bytes") o.bytes = parse_size(v);
        else if (k == "--iters") o.iters = parse_size(v);
        else if (k == "--warmup") o.warmup = parse_size(v);
        else if (k == "--op") o.op = v;
        else if (k == "--min") o.min_bytes = parse_size(v);
        else if (k == "--max") o.max_bytes = parse_size(v);
        else if (k == "--qd") o.qd = parse_size(v);
        else if (k == "--bytes-per-size") o.bytes_per_size = parse_size(v);
        else if (k == "--trace-size") o.trace_size = parse_size(v);
        else if (k == "--trace-out") o.trace_out = v;
        else if (k == "--batch") o.batch = parse_size(v);
        else if (k == "--wrs") o.wrs = parse_size(v);
        else if (k == "--qps") o.qps = parse_size(v);
        else if (k == "--depth") o.depth = parse_size(v);
        else if (k == "--sges") o.sges = parse_size(v);
        else if (k == "--rounds") o.rounds = parse_size(v);
        else if (k == "--seed") o.seed = parse_size(v);
        else if (k == "--sync-dir") o.sync_dir = v;
        else if (k == "--sync-n") o.sync_n = parse_size(v);
        else {
            std::fprintf(stderr, "ugdr_perf: unknown option %s\n", k.c_str());
            return 2;
        }
    }
    if (o.mode == "latency") return run_latency(o);
    if (o.mode == "bw") return run_bw(o);
    if (o.mode == "posting") return run_posting(o);
    if (o.mode == "stress") return run_stress(o);
    if (o.mode == "plumbing") return run_plumbing(o);
    if (o.mode == "control") return run_control(o);
    if (o.mode == "ring") return run_ring(o);
    if (o.mode == "postcore") return run_postcore(o);
    std::fprintf(stderr, "ugdr_perf: unknown mode %s\n", o.mode.c_str());
    return 2;
}
