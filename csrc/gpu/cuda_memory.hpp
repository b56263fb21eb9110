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

// Close the IPC mappings on GPU `device` whose last MR went away.  cudaIpcCloseMemHandle waits
// for the kernels running in that GPU's context, and the executor is persistent, so closing at
// deregistration would stall the caller until the executor's idle exit.  Deregistration only
// marks the mapping unused (the MR entry is already invalid and no WR can reach it); each GPU's
// engine calls this while its executor is not running.  A handle registered again before then
// reuses its open mapping.
void reap_ipc_closes(int device) noexcept;

class DaemonMemoryBackend : public control::MemoryBackend {
  public:
    explicit DaemonMemoryBackend(GpuInventory inv);
    ~DaemonMemoryBackend() override;
    int open(control::MemoryDescriptor &desc, uint64_t length, control::OpenedMemory *out) override;
    void close(control::OpenedMemory &mem) noexcept override;

  private:
    struct Mapping {
        std::vector<void *> bases;  // one mapping per daemon GPU (index = CUDA ordinal)
        std::vector<uint8_t> closed;  // per GPU: unused and already closed by reap()
        int gpu = -1;               // owner
        int refs = 0;               // 0: unused, waiting for reap() on every GPU
    };
    friend void reap_ipc_closes(int device) noexcept;
    void reap(int device) noexcept;
    GpuInventory inv_;
    std::mutex mu_;
    std::map<std::vector<uint8_t>, Mapping> open_;  // handle bytes -> mapping
};

}  // namespace ugdr::gpu
