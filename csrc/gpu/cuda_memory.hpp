// Daemon side of the CUDA-IPC memory-registration model.
//
// Parity: reference src/gpu/cuda_ipc_memory.cu:170-292 (per-UUID device table, open with
// cudaIpcMemLazyEnablePeerAccess, close).  Differences: the daemon enables peer access between
// every pair of GPUs it owns, and opens each handle once in every GPU's context, because an
// IPC mapping exists only in the context that opened it: the executor on GPU a stores into an
// MR on GPU b through GPU a's own mapping (NVLink).  Opened handles are reference-counted, since
// a client may register several ranges of one allocation and a handle opens once per context.
#pragma once

#include "control/objects.hpp"

#include <array>
#include <cstdint>
#include <map>
#include <mutex>
#include <vector>

namespace ugdr::gpu {

struct GpuInventory {
    int count = 0;
    std::vector<std::array<uint8_t, 16>> uuids;
    std::vector<int> sm_count;
};

// Enumerate visible GPUs (count 0 when CUDA is unusable).  `limit` < 0 means all.
GpuInventory probe_gpus(int limit);
// Enable peer access between every ordered pair of the first `n` GPUs.  Returns the number of
// pairs that could not be enabled.
int enable_all_peer_access(int n);

class DaemonMemoryBackend : public control::MemoryBackend {
  public:
    explicit DaemonMemoryBackend(GpuInventory inv) : inv_(std::move(inv)) {}
    int open(control::MemoryDescriptor &desc, uint64_t length, control::OpenedMemory *out) override;
    void close(control::OpenedMemory &mem) noexcept override;

  private:
    struct Mapping {
        std::vector<void *> bases;  // one mapping per daemon GPU (index = CUDA ordinal)
        int gpu = -1;               // owner
        int refs = 0;
    };
    GpuInventory inv_;
    std::mutex mu_;
    std::map<std::vector<uint8_t>, Mapping> open_;  // handle bytes -> mapping
};

}  // namespace ugdr::gpu
