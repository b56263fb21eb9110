#include "gpu/trace_writer.hpp"

#include <algorithm>
#include <cerrno>
#include <cstdio>

namespace ugdr::gpu {

int write_chrome_trace(const std::string &path, const std::vector<TraceRec> &recs,
                       const std::vector<unsigned int> &counts, uint32_t cap, int gpu, uint64_t *kept,
                       uint64_t *dropped) {
    if (recs.size() < counts.size() * size_t(cap)) return EINVAL;
    static const char *names[] = {"?", "fast_batch", "retire", "chunk", "error", "issue"};
    uint64_t t_min = ~0ull, n_kept = 0, n_drop = 0;
    for (size_t c = 0; c < counts.size(); ++c) {
        const uint32_t k = std::min<uint32_t>(counts[c], cap);
        n_kept += k;
        n_drop += counts[c] - k;
        for (uint32_t i = 0; i < k; ++i) t_min = std::min<uint64_t>(t_min, recs[c * cap + i].t0);
    }
    FILE *f = std::fopen(path.c_str(), "w");
    if (f == nullptr) return errno != 0 ? errno : EIO;
    std::fprintf(f, "{\"traceEvents\": [");
    bool first = true;
    for (size_t c = 0; c < counts.size(); ++c) {
        const uint32_t k = std::min<uint32_t>(counts[c], cap);
        for (uint32_t i = 0; i < k; ++i) {
            const TraceRec &r = recs[c * cap + i];
            const uint32_t ev = r.event >> 16;
            // t1 < t0 cannot come from one warp's clock; clamp rather than print a negative span.
            const uint64_t dur = r.t1 > r.t0 ? r.t1 - r.t0 : 0;
            std::fprintf(f,
                         "%s\n{\"name\": \"%s\", \"ph\": \"X\", \"pid\": %u, \"tid\": %u, \"ts\": %.3f, "
                         "\"dur\": %.3f, \"args\": {\"qp\": %d, \"value\": %u}}",
                         first ? "" : ",", ev < 6 ? names[ev] : "?", r.cta, r.event & 0xffffu,
                         double(r.t0 - t_min) / 1000.0, double(dur) / 1000.0,
                         r.qp == 0xffffffffu ? -1 : int(r.qp), r.value);
            first = false;
        }
    }
    std::fprintf(f, "\n], \"displayTimeUnit\": \"ns\", \"otherData\": {\"gpu\": %d, \"dropped\": %llu}}\n", gpu,
                 (unsigned long long)n_drop);
    const bool ok = std::fclose(f) == 0;
    if (kept) *kept = n_kept;
    if (dropped) *dropped = n_drop;
    return ok ? 0 : EIO;
}

}  // namespace ugdr::gpu
