// NVTX ranges on the host phases of the control plane and the engines.  NVTX v3 is header-only:
// without a tool attached (Nsight Systems, or any NVTX injection library) every call is a
// check of one pointer, so the ranges stay in release builds.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace ugdr {

class TraceRange {
  public:
    explicit TraceRange(const char *name) noexcept { nvtxRangePushA(name); }
    ~TraceRange() { nvtxRangePop(); }
    TraceRange(const TraceRange &) = delete;
    TraceRange &operator=(const TraceRange &) = delete;
};

}  // namespace ugdr
