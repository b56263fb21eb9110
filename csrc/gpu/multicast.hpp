// Daemon-side mapping of a client's NVLink multicast object (see multicast.cpp).
#pragma once

#include <cstdint>
#include <vector>

namespace ugdr::gpu {

struct McMapping {
    void *address = nullptr;      // multicast view in the daemon's address space
    uint64_t bytes = 0;
    uint64_t handle = 0;          // imported object
    std::vector<bool> reachable;  // per daemon GPU: access granted (member of the object's team)
};

// Import `fd` (a POSIX shareable handle of the object), map `bytes` from offset 0 and enable
// access for every GPU of the team among the daemon's `gpus`.  Returns 0 or an errno.
int map_multicast(int fd, uint64_t bytes, int gpus, McMapping *out);
void unmap_multicast(McMapping &m) noexcept;

}  // namespace ugdr::gpu
