#include "common/shm.hpp"

#include <cstdint>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <utility>

namespace ugdr {

SharedMapping::SharedMapping(SharedMapping &&o) noexcept
    : address(std::exchange(o.address, nullptr)), bytes(std::exchange(o.bytes, 0)),
      fd(std::move(o.fd)) {}

SharedMapping &SharedMapping::operator=(SharedMapping &&o) noexcept {
    if (this != &o) {
        unmap();
        address = std::exchange(o.address, nullptr);
        bytes = std::exchange(o.bytes, 0);
        fd = std::move(o.fd);
    }
    return *this;
}

void SharedMapping::unmap() noexcept {
    if (address != nullptr) ::munmap(address, bytes);
    address = nullptr;
    bytes = 0;
    fd.reset();
}

size_t page_size() noexcept {
    static const size_t p = static_cast<size_t>(::sysconf(_SC_PAGESIZE));
    return p;
}

size_t round_up_pages(size_t bytes) noexcept {
    const size_t p = page_size();
    if (bytes > SIZE_MAX - (p - 1)) return 0;
    return (bytes + p - 1) / p * p;
}

int create_shared_mapping(const char *name, size_t bytes, SharedMapping *out) noexcept {
    if (out == nullptr || bytes == 0) return EINVAL;
    const size_t total = round_up_pages(bytes);
    if (total == 0) return EOVERFLOW;
    Fd fd(::memfd_create(name, MFD_CLOEXEC | MFD_ALLOW_SEALING));
    if (!fd.valid()) return errno;
    if (::ftruncate(fd.get(), static_cast<off_t>(total)) != 0) return errno;
    if (::fcntl(fd.get(), F_ADD_SEALS, F_SEAL_SHRINK | F_SEAL_GROW | F_SEAL_SEAL) != 0) return errno;
    void *addr = ::mmap(nullptr, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd.get(), 0);
    if (addr == MAP_FAILED) return errno;
    out->unmap();
    out->address = addr;
    out->bytes = total;
    out->fd = std::move(fd);
    return 0;
}

int map_shared_fd(int raw_fd, size_t expected_bytes, SharedMapping *out) noexcept {
    Fd fd(raw_fd);
    if (out == nullptr || !fd.valid()) return EINVAL;
    struct stat st {};
    if (::fstat(fd.get(), &st) != 0) return errno;
    if (st.st_size <= 0) return EPROTO;
    const size_t size = static_cast<size_t>(st.st_size);
    if (expected_bytes != 0 && size != expected_bytes) return EPROTO;
    void *addr = ::mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd.get(), 0);
    if (addr == MAP_FAILED) return errno;
    out->unmap();
    out->address = addr;
    out->bytes = size;
    out->fd = std::move(fd);
    return 0;
}

}  // namespace ugdr
