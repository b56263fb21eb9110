#include "api/memory_export.hpp"

#include "common/bytes.hpp"
#include "common/shm.hpp"
#include "control/objects.hpp"

#include <cuda.h>
#include <cuda_runtime_api.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <map>
#include <mutex>

namespace ugdr::api {
namespace {

std::mutex g_host_mu;
std::map<uintptr_t, SharedMapping> g_host;  // base -> mapping

using GetRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

GetRangeFn get_range_fn() {
    static GetRangeFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return GetRangeFn(nullptr);
        return reinterpret_cast<GetRangeFn>(p);
    }();
    return fn;
}

int export_host(const SharedMapping &m, uintptr_t addr, size_t len, std::vector<std::byte> *opaque,
                std::vector<Fd> *fds) {
    const uintptr_t base = reinterpret_cast<uintptr_t>(m.address);
    if (addr + len > base + m.bytes || addr + len < addr) return EINVAL;
    Fd dup_fd(::dup(m.fd.get()));
    if (!dup_fd.valid()) return errno;
    ByteWriter w(opaque);
    const uint8_t pad[3] = {0, 0, 0};
    w.be(uint8_t(control::MemKind::host)).raw(pad, 3).be(uint64_t(addr));
    w.be(uint64_t(m.bytes)).be(uint64_t(addr - base));
    fds->push_back(std::move(dup_fd));
    return 0;
}

}  // namespace

int export_multicast(int fd, uint64_t client_addr, size_t len, std::vector<std::byte> *opaque,
                     std::vector<Fd> *fds) {
    if (fd < 0 || client_addr == 0 || len == 0) return EINVAL;
    Fd dup_fd(::dup(fd));
    if (!dup_fd.valid()) return errno;
    ByteWriter w(opaque);
    const uint8_t pad[3] = {0, 0, 0};
    w.be(uint8_t(control::MemKind::multicast)).raw(pad, 3).be(uint64_t(client_addr));
    w.be(uint64_t(len)).be(uint64_t(0));
    fds->push_back(std::move(dup_fd));
    return 0;
}

void *host_alloc(size_t len) {
    if (len == 0) {
        errno = EINVAL;
        return nullptr;
    }
    SharedMapping m;
    if (int rc = create_shared_mapping("ugdr-host", len, &m); rc != 0) {
        errno = rc;
        return nullptr;
    }
    void *addr = m.address;
    std::lock_guard<std::mutex> lk(g_host_mu);
    g_host.emplace(reinterpret_cast<uintptr_t>(addr), std::move(m));
    return addr;
}

int host_free(void *addr) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    auto it = g_host.find(reinterpret_cast<uintptr_t>(addr));
    if (it == g_host.end()) return EINVAL;
    g_host.erase(it);
    return 0;
}

int export_memory(void *addr, size_t len, std::vector<std::byte> *opaque, std::vector<Fd> *fds) {
    if (addr == nullptr || len == 0) return EINVAL;
    const uintptr_t a = reinterpret_cast<uintptr_t>(addr);
    {
        std::lock_guard<std::mutex> lk(g_host_mu);
        auto it = g_host.upper_bound(a);
        if (it != g_host.begin()) {
            --it;
            const SharedMapping &m = it->second;
            if (a >= it->first && a < it->first + m.bytes) return export_host(m, a, len, opaque, fds);
        }
    }
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, addr) != cudaSuccess) {
        (void)cudaGetLastError();
        return EOPNOTSUPP;
    }
    if (attr.type != cudaMemoryTypeDevice) return EOPNOTSUPP;
    GetRangeFn range = get_range_fn();
    if (range == nullptr) return EOPNOTSUPP;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, attr.device) != cudaSuccess) return EOPNOTSUPP;
    // The range query and the export run in the owning device's context.
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(attr.device);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, CUdeviceptr(a)) != CUDA_SUCCESS) {
        cudaSetDevice(prev);
        return EOPNOTSUPP;
    }
    if (a + len > base + size || a + len < a) {
        cudaSetDevice(prev);
        return EINVAL;
    }
    cudaIpcMemHandle_t h{};
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return EOPNOTSUPP;  // e.g. VMM / pool allocations without IPC support
    }
    ByteWriter w(opaque);
    const uint8_t pad[3] = {0, 0, 0};
    w.be(uint8_t(control::MemKind::cuda)).raw(pad, 3).be(uint64_t(a));
    w.raw(prop.uuid.bytes, 16).be(uint64_t(size)).be(uint64_t(a - base));
    w.be(uint32_t(sizeof(h))).raw(&h, sizeof(h));
    return 0;
}

}  // namespace ugdr::api
