// ugdr_engine_bench: the host engine driven in one thread, without a daemon or sockets.  It
// covers the reference's two in-process benchmarks, with this build's engine in the worker's
// place:
//
//   ugdr_engine_bench metadata   post_send chain -> engine pass -> poll CQ, per batch
//                                (--pass-lock 0: no object lock around the pass, as the
//                                reference's lock-free mock worker)
//                                (reference: benchmarks/queue_metadata_benchmark.cpp:70-176;
//                                batch 1/32 x SGEs 1/4 x signal every WR / every 32nd WR).
//   ugdr_engine_bench payload    up to `depth` WRs in flight on one QP, completion seen at the
//                                SQ consumer cursor, latency post -> retire per WR
//                                (reference: benchmarks/loop_worker_payload_benchmark.cpp:296-452;
//                                its four cases: 4 KiB x 1 SGE depth 32 every WR signaled,
//                                64 KiB x 1 and x 4 SGEs depth 64 every 32nd, 64 KiB x 4 unsignaled).
//
// Unlike the reference's mock workers, the engine here moves every payload byte (memcpy between
// two registered host ranges), so the figures include the copies.  `--wr-bytes` changes the
// metadata benchmark's WR size (8 isolates the descriptor path).
//
// Output: one key=value line per case, in the reference's style.
#include "api/posting.hpp"
#include "common/bytes.hpp"
#include "common/shm.hpp"
#include "control/service.hpp"
#include "engine/cpu_engine.hpp"
#include "queue/layout.hpp"
#include "queue/ring.hpp"
#include "ugdr/api.hpp"

#include <unistd.h>
#if defined(__x86_64__)
#include <x86intrin.h>
#endif

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

using namespace ugdr;
using namespace ugdr::control;

namespace {

using Clock = std::chrono::steady_clock;

uint64_t cycles() {
#if defined(__x86_64__)
    return __rdtsc();
#else
    return uint64_t(Clock::now().time_since_epoch().count());
#endif
}

[[noreturn]] void die(const char *what, int rc) {
    std::fprintf(stderr, "ugdr_engine_bench: %s failed (%d: %s)\n", what, rc, std::strerror(rc));
    std::exit(1);
}

// Host MRs only: maps the memfd the registration carries, as the daemon does.
class HostBackend : public MemoryBackend {
  public:
    int open(MemoryDescriptor &d, uint64_t, OpenedMemory *out) override {
        if (d.kind != MemKind::host) return EOPNOTSUPP;
        if (int rc = map_shared_fd(d.region_fd.release(), 0, &out->host); rc != 0) return rc;
        out->address = static_cast<uint8_t *>(out->host.address) + d.region_offset;
        out->gpu = -1;
        return 0;
    }
    void close(OpenedMemory &m) noexcept override { m.host.unmap(); }
};

constexpr uint32_t kAccess = UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ;

// One connected QP pair on one PD, one CQ, and one host region holding the source range (first
// half) and the target range (second half).  The requester's SQ and the CQ are attached here
// exactly as a client library attaches them.
struct Rig {
    std::mutex mu;
    engine::CpuEngine eng{mu, false};
    HostBackend mem;
    ControlPlane cp{{&eng}, mem};
    SharedMapping region;
    queue::Ring sq, cq;
    uint32_t lkey = 0, rkey = 0, max_sge = 0;
    uint8_t *src = nullptr, *dst = nullptr;
    uint64_t half = 0;

    Response call(uint32_t method, uint64_t id, uint64_t length = 0, uint32_t access = 0,
                  std::vector<std::byte> opaque = {}, std::vector<Fd> fds = {}) {
        Request r;
        r.method = method;
        r.identity = id;
        r.length = length;
        r.access = access;
        r.opaque = std::move(opaque);
        r.fds = std::move(fds);
        Response resp = cp.dispatch(1, std::move(r));
        if (resp.status != 0) die("control call", resp.status);
        return resp;
    }

    Rig(uint32_t depth, uint32_t sges, uint32_t cq_depth, uint64_t bytes) : max_sge(sges), half(bytes) {
        const uint64_t ctx = call(kCreateContext, 1).identity;
        const uint64_t pd = call(kCreatePd, ctx).identity;
        Response c = call(kCreateCq, ctx, cq_depth);
        uint32_t cap = 0, stride = 0;
        ByteReader crd(c.opaque);
        crd.be(&cap);
        crd.be(&stride);
        if (int rc = queue::Ring::attach(c.fds[0].release(), {queue::kCompletionRing, cap, stride}, &cq); rc != 0)
            die("attach CQ", rc);
        uint64_t qp[2];
        uint32_t qpn[2];
        for (int i = 0; i < 2; ++i) {
            std::vector<std::byte> o;
            ByteWriter w(&o);
            w.be(c.identity).be(c.identity).be(depth).be(depth).be(sges).be(sges).be(uint32_t(UGDR_QPT_RC));
            w.be(uint32_t(0));
            Response q = call(kCreateQp, pd, 0, 0, std::move(o));
            ByteReader rd(q.opaque);
            uint32_t v[9] = {};
            for (uint32_t &x : v) rd.be(&x);
            qp[i] = q.identity;
            qpn[i] = v[0];
            if (i == 0) {
                if (int rc = queue::Ring::attach(q.fds[0].release(), {queue::kSendRing, v[5], v[6]}, &sq); rc != 0)
                    die("attach SQ", rc);
            }
            std::vector<std::byte> m;
            ByteWriter mw(&m);
            mw.be(uint32_t(UGDR_QPS_INIT)).be(uint32_t(0)).be(uint32_t(UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ));
            mw.be(uint8_t(14)).be(uint8_t(7)).be(uint8_t(7)).be(uint8_t(12));
            call(kModifyQp, qp[i], 0, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS, std::move(m));
        }
        for (int i = 0; i < 2; ++i) {
            std::vector<std::byte> o;
            ByteWriter w(&o);
            w.be(qpn[1 - i]).be(uint32_t(0)).be(uint32_t(0)).be(uint32_t(0)).be(uint8_t(14)).be(uint8_t(7));
            w.be(uint8_t(7)).be(uint8_t(1));
            call(kConnectQp, qp[i], 0, UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER,
                 std::move(o));
        }
        if (int rc = create_shared_mapping("engine-bench", 2 * bytes, &region); rc != 0) die("region", rc);
        src = static_cast<uint8_t *>(region.address);
        dst = src + bytes;
        for (uint64_t i = 0; i < 2 * bytes; ++i) src[i] = uint8_t(i * 131 + 7);
        std::vector<std::byte> o;
        ByteWriter w(&o);
        const uint8_t pad[3] = {0, 0, 0};
        w.be(uint8_t(MemKind::host)).raw(pad, 3).be(uint64_t(reinterpret_cast<uintptr_t>(src)));
        w.be(uint64_t(region.bytes)).be(uint64_t(0));
        std::vector<Fd> fds;
        fds.emplace_back(::dup(region.fd.get()));
        Response mr = call(kRegisterMr, pd, 2 * bytes, kAccess, std::move(o), std::move(fds));
        ByteReader rd(mr.opaque);
        uint64_t a = 0, l = 0;
        rd.be(&a);
        rd.be(&l);
        rd.be(&lkey);
        rd.be(&rkey);
    }

    uint64_t addr(const uint8_t *p) const { return reinterpret_cast<uintptr_t>(p); }

    // With `pass_lock` each engine pass takes the control plane's object lock, as the daemon's
    // engine thread does; without it this single thread holds no lock (nothing else runs here),
    // which is the reference's mock-worker setting.
    bool pass_lock = true;
    size_t progress() {
        if (!pass_lock) return eng.progress_locked();
        std::lock_guard<std::mutex> lk(mu);
        return eng.progress_locked();
    }

    // Polls everything in the CQ; returns the number of completions (statuses checked).
    int drain() {
        int n = 0;
        for (;;) {
            queue::SlotRun run = cq.peek(64);
            const uint32_t k = run.count();
            if (k == 0) return n;
            for (uint32_t i = 0; i < k; ++i) {
                const uint8_t *s = i < run.first_count ? run.first + i * 64u : run.second + (i - run.first_count) * 64u;
                queue::Cqe e;
                std::memcpy(&e, s, sizeof(e));
                ugdr_wc wc;
                api::cqe_to_wc(e, &wc);
                if (wc.status != UGDR_WC_SUCCESS) die("completion status", int(wc.status));
            }
            cq.release(k);
            n += int(k);
        }
    }
};

double pct(std::vector<double> &v, double q) {
    if (v.empty()) return 0;
    std::sort(v.begin(), v.end());
    return v[size_t(q * double(v.size() - 1))];
}

// Split `bytes` over `n` SGEs the way the reference's payload benchmark does (remainder first).
void fill_sges(ugdr_sge *sg, uint32_t n, uint64_t base, uint32_t bytes, uint32_t lkey) {
    const uint32_t each = bytes / n, rem = bytes % n;
    uint64_t off = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t len = each + (i < rem ? 1 : 0);
        sg[i] = {base + off, len, lkey};
        off += len;
    }
}

bool g_pass_lock = true;

void metadata_case(uint32_t batch, uint32_t nsge, bool every, uint32_t wr_bytes) {
    constexpr uint32_t kCap = 256;
    constexpr uint64_t kWrs = 262144;
    Rig r(kCap, nsge, kCap, uint64_t(wr_bytes) * batch);
    r.pass_lock = g_pass_lock;
    std::vector<ugdr_send_wr> wr(batch);
    std::vector<ugdr_sge> sg(size_t(batch) * nsge);
    for (uint32_t i = 0; i < batch; ++i) {
        wr[i] = {};
        wr[i].next = i + 1 < batch ? &wr[i + 1] : nullptr;
        wr[i].sg_list = &sg[size_t(i) * nsge];
        wr[i].num_sge = int(nsge);
        wr[i].opcode = UGDR_WR_RDMA_WRITE;
        wr[i].wr.rdma.remote_addr = r.addr(r.dst) + uint64_t(i) * wr_bytes;
        wr[i].wr.rdma.rkey = r.rkey;
        fill_sges(wr[i].sg_list, nsge, r.addr(r.src) + uint64_t(i) * wr_bytes, wr_bytes, r.lkey);
    }
    uint64_t seq = 0, wc = 0;
    auto iteration = [&]() {
        int expect = 0;
        for (uint32_t i = 0; i < batch; ++i, ++seq) {
            wr[i].wr_id = seq + 1;
            const bool sig = every || seq % 32 == 31;
            wr[i].send_flags = sig ? UGDR_SEND_SIGNALED : 0;
            expect += sig ? 1 : 0;
        }
        ugdr_send_wr *bad = nullptr;
        if (int rc = api::post_send_chain(r.sq, r.max_sge, wr.data(), &bad); rc != 0) die("post_send_chain", rc);
        size_t done = 0;
        while (done < batch) done += r.progress();
        int got = 0;
        while (got < expect) got += r.drain();
        wc += uint64_t(got);
    };
    for (int i = 0; i < 128; ++i) iteration();
    wc = 0;
    const uint64_t iters = kWrs / batch;
    std::vector<double> lat(iters);
    const uint64_t c0 = cycles();
    const auto t0 = Clock::now();
    for (uint64_t i = 0; i < iters; ++i) {
        const auto s = Clock::now();
        iteration();
        lat[i] = std::chrono::duration<double, std::nano>(Clock::now() - s).count();
    }
    const double secs = std::chrono::duration<double>(Clock::now() - t0).count();
    const uint64_t c1 = cycles();
    const double wrs = double(iters * batch);
    if (std::memcmp(r.dst, r.src, size_t(wr_bytes) * batch) != 0) die("payload check", EIO);
    std::printf("benchmark=engine_metadata pass_lock=%d batch=%u num_sge=%u signaling=%s wr_bytes=%u completed_wr=%llu wc=%llu "
                "MWR_per_s=%.3f cycles_per_wr=%.1f latency_sample=batch p50_ns=%.0f p99_ns=%.0f\n",
                int(g_pass_lock), batch, nsge, every ? "every_wr" : "every_32_wr", wr_bytes, (unsigned long long)(iters * batch),
                (unsigned long long)wc, wrs / secs / 1e6, double(c1 - c0) / wrs, pct(lat, 0.5), pct(lat, 0.99));
}

void payload_case(uint32_t wr_bytes, uint32_t nsge, uint32_t depth, uint32_t interval, uint64_t iters) {
    const uint64_t warm = 1000;
    Rig r(depth, nsge, 2 * depth, wr_bytes);
    std::vector<ugdr_sge> sg(nsge);
    ugdr_send_wr wr{};
    wr.sg_list = sg.data();
    wr.num_sge = int(nsge);
    wr.opcode = UGDR_WR_RDMA_WRITE;
    wr.wr.rdma.remote_addr = r.addr(r.dst);
    wr.wr.rdma.rkey = r.rkey;
    fill_sges(sg.data(), nsge, r.addr(r.src), wr_bytes, r.lkey);
    std::vector<Clock::time_point> posted_at(depth);
    std::vector<double> lat;
    lat.reserve(iters);
    uint64_t next_id = 0;
    auto phase = [&](uint64_t n, bool record) {
        const uint64_t base = r.sq.head();  // WRs retired before this phase
        uint64_t posted = 0, done = 0;
        while (done < n) {
            while (posted < n && posted - done < depth) {
                const uint64_t id = next_id++;
                wr.wr_id = id;
                wr.send_flags = interval != 0 && id % interval == 0 ? UGDR_SEND_SIGNALED : 0;
                posted_at[(base + posted) % depth] = Clock::now();
                ugdr_send_wr *bad = nullptr;
                if (int rc = api::post_send_chain(r.sq, r.max_sge, &wr, &bad); rc != 0) die("post_send_chain", rc);
                ++posted;
            }
            r.progress();
            r.drain();
            const uint64_t now_done = r.sq.head() - base;
            if (record) {
                const auto t = Clock::now();
                for (uint64_t k = done; k < now_done; ++k)
                    lat.push_back(std::chrono::duration<double, std::micro>(t - posted_at[(base + k) % depth]).count());
            }
            done = now_done;
        }
        while (r.drain() > 0) {
        }
    };
    phase(warm, false);
    const auto t0 = Clock::now();
    phase(iters, true);
    const double secs = std::chrono::duration<double>(Clock::now() - t0).count();
    if (std::memcmp(r.dst, r.src, wr_bytes) != 0) die("payload check", EIO);
    std::printf("benchmark=engine_payload wr_bytes=%u sge_count=%u queue_depth=%u signaling_interval=%u warmup=%llu "
                "iterations=%llu parent_MWR_per_s=%.6f logical_payload_GB_per_s=%.6f wr_p50_us=%.3f wr_p99_us=%.3f\n",
                wr_bytes, nsge, depth, interval, (unsigned long long)warm, (unsigned long long)iters,
                double(iters) / secs / 1e6, double(iters) * wr_bytes / secs / 1e9, pct(lat, 0.5), pct(lat, 0.99));
}

}  // namespace

int main(int argc, char **argv) {
    std::string mode = argc > 1 ? argv[1] : "metadata";
    uint32_t wr_bytes = 4096;
    uint64_t iters = 10000;
    for (int i = 2; i + 1 < argc; i += 2) {
        const std::string k = argv[i];
        if (k == "--wr-bytes") wr_bytes = uint32_t(std::strtoul(argv[i + 1], nullptr, 0));
        else if (k == "--iters") iters = std::strtoull(argv[i + 1], nullptr, 0);
        else if (k == "--pass-lock") g_pass_lock = std::strtoul(argv[i + 1], nullptr, 0) != 0;
        else die("unknown option", EINVAL);
    }
    if (mode == "metadata") {
        for (uint32_t batch : {1u, 32u})
            for (uint32_t nsge : {1u, 4u})
                for (bool every : {true, false}) metadata_case(batch, nsge, every, wr_bytes);
    } else if (mode == "payload") {
        payload_case(4096, 1, 32, 1, iters);
        payload_case(65536, 1, 64, 32, iters);
        payload_case(65536, 4, 64, 32, iters);
        payload_case(65536, 4, 64, 0, iters);
    } else {
        die("mode (metadata | payload)", EINVAL);
    }
    return 0;
}
