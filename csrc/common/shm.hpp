// memfd-backed shared mappings: the transport for rings and for registrable host buffers.
#pragma once

#include "common/fd.hpp"

#include <cstddef>

namespace ugdr {

struct SharedMapping {
    void *address = nullptr;
    size_t bytes = 0;
    Fd fd;

    SharedMapping() = default;
    SharedMapping(const SharedMapping &) = delete;
    SharedMapping &operator=(const SharedMapping &) = delete;
    SharedMapping(SharedMapping &&o) noexcept;
    SharedMapping &operator=(SharedMapping &&o) noexcept;
    ~SharedMapping() { unmap(); }
    void unmap() noexcept;
};

size_t page_size() noexcept;
size_t round_up_pages(size_t bytes) noexcept;

// Create a sealed (no grow / shrink) memfd of `bytes` (rounded to pages), zero-filled and
// mapped read/write shared.  Returns 0 or a positive errno.
int create_shared_mapping(const char *name, size_t bytes, SharedMapping *out) noexcept;
// Map an existing memfd (takes ownership of `fd`).  `expected_bytes` of 0 accepts any size.
int map_shared_fd(int fd, size_t expected_bytes, SharedMapping *out) noexcept;

}  // namespace ugdr
