// Chrome trace-event JSON for the executor's device trace (TraceRec records, device_abi.hpp).
#pragma once

#include "gpu/device_abi.hpp"

#include <cstdint>
#include <string>
#include <vector>

namespace ugdr::gpu {

// `recs` holds counts.size() segments of `cap` records (one per CTA); counts[c] is how many
// events CTA c tried to record (those past `cap` were dropped).  Writes "X" (complete) events:
// pid = CTA, tid = global warp, ts / dur in microseconds from the earliest kept record.
// Returns 0 or an errno; *kept / *dropped receive the totals.
int write_chrome_trace(const std::string &path, const std::vector<TraceRec> &recs,
                       const std::vector<unsigned int> &counts, uint32_t cap, int gpu, uint64_t *kept,
                       uint64_t *dropped);

}  // namespace ugdr::gpu
