// Client-side description of memory handed to ugdr_reg_mr.
//
// Two kinds of memory can be registered: ranges inside a cudaMalloc allocation (exported as a
// CUDA IPC handle of the allocation base plus an offset and the owning GPU's UUID, as in the
// reference src/gpu/cuda_ipc_memory.cu:104-168), and ranges inside a ugdr host buffer from
// ugdr_x_alloc_host (exported as its memfd).  Anything else is EOPNOTSUPP.
#pragma once

#include "common/fd.hpp"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace ugdr::api {

// Build the register-MR opaque (and the fd list) for [addr, addr + len).
int export_memory(void *addr, size_t len, std::vector<std::byte> *opaque, std::vector<Fd> *fds);

// The register-MR opaque for an NVLink multicast object: `fd` is its POSIX shareable handle
// (duplicated here), `client_addr` the caller's own multicast mapping of it and `len` the bytes
// registered from offset 0.
int export_multicast(int fd, uint64_t client_addr, size_t len, std::vector<std::byte> *opaque,
                     std::vector<Fd> *fds);

// Host buffers.
void *host_alloc(size_t len);
int host_free(void *addr);

}  // namespace ugdr::api
