// Chrome-trace writer of the executor's device trace, on synthetic records (no GPU needed).
#include "harness.hpp"

#include "gpu/trace_writer.hpp"

#include <unistd.h>

#include <cerrno>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

using namespace ugdr::gpu;

namespace {

size_t count_of(const std::string &s, const std::string &needle) {
    size_t n = 0;
    for (size_t p = s.find(needle); p != std::string::npos; p = s.find(needle, p + 1)) ++n;
    return n;
}

TraceRec rec(uint64_t t0, uint64_t t1, uint32_t ev, uint32_t warp, uint32_t qp, uint32_t value, uint32_t cta) {
    TraceRec r{};
    r.t0 = t0;
    r.t1 = t1;
    r.event = (ev << 16) | warp;
    r.qp = qp;
    r.value = value;
    r.cta = cta;
    return r;
}

}  // namespace

TEST(trace_writer_keeps_segments_counts_drops_and_clamps) {
    // Two CTAs, three records each; CTA 0 recorded 2 events, CTA 1 tried 5 (2 dropped).
    const uint32_t cap = 3;
    std::vector<TraceRec> recs(2 * cap);
    recs[0] = rec(5000, 7000, kTraceFastBatch, 3, 12, 16, 0);
    recs[1] = rec(9000, 8000, kTraceRetire, 3, 12, 4, 0);  // t1 < t0: duration clamps to 0
    recs[3] = rec(6000, 6500, kTraceChunk, 20, 0xffffffffu, 65536, 1);
    recs[4] = rec(6100, 6600, kTraceChunk, 21, 0xffffffffu, 65536, 1);
    recs[5] = rec(6200, 6300, kTraceError, 22, 0xffffffffu, 1, 1);
    const std::vector<unsigned int> counts = {2, 5};
    char path[] = "/tmp/ugdr-trace-XXXXXX";
    const int fd = ::mkstemp(path);
    CHECK(fd >= 0);
    ::close(fd);
    uint64_t kept = 0, dropped = 0;
    CHECK_EQ(write_chrome_trace(path, recs, counts, cap, 3, &kept, &dropped), 0);
    CHECK_EQ(kept, 5ull);
    CHECK_EQ(dropped, 2ull);
    std::ifstream in(path);
    std::stringstream ss;
    ss << in.rdbuf();
    const std::string doc = ss.str();
    ::unlink(path);
    CHECK_EQ(count_of(doc, "\"ph\": \"X\""), size_t(5));
    CHECK_EQ(count_of(doc, "\"name\": \"chunk\""), size_t(2));
    CHECK_EQ(count_of(doc, "\"name\": \"error\""), size_t(1));
    CHECK(doc.find("\"ts\": 0.000") != std::string::npos);       // earliest record starts the clock
    CHECK(doc.find("\"ts\": 4.000, \"dur\": 0.000") != std::string::npos);  // clamped span
    CHECK(doc.find("\"qp\": -1") != std::string::npos);
    CHECK(doc.find("\"dropped\": 2") != std::string::npos && doc.find("\"gpu\": 3") != std::string::npos);
    // Too few records for the segments claimed: refused.
    CHECK_EQ(write_chrome_trace("/tmp/unused", std::vector<TraceRec>(2), counts, cap, 0, &kept, &dropped), EINVAL);
}
