#include "gpu/cuda_memory.hpp"
#include "gpu/multicast.hpp"

#include <cuda_runtime_api.h>

#include <cerrno>
#include <cstring>

namespace ugdr::gpu {

GpuInventory probe_gpus(int limit) {
    GpuInventory inv;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        (void)cudaGetLastError();
        return inv;
    }
    if (limit >= 0 && limit < n) n = limit;
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp p{};
        if (cudaGetDeviceProperties(&p, i) != cudaSuccess) break;
        std::array<uint8_t, 16> u{};
        std::memcpy(u.data(), p.uuid.bytes, 16);
        inv.uuids.push_back(u);
        inv.sm_count.push_back(p.multiProcessorCount);
        inv.count += 1;
    }
    return inv;
}

int enable_all_peer_access(int n) {
    int failures = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    for (int a = 0; a < n; ++a) {
        cudaSetDevice(a);
        for (int b = 0; b < n; ++b) {
            if (a == b) continue;
            int can = 0;
            cudaDeviceCanAccessPeer(&can, a, b);
            if (!can) {
                ++failures;
                continue;
            }
            const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) ++failures;
            (void)cudaGetLastError();
        }
    }
    cudaSetDevice(prev);
    return failures;
}

namespace {
std::mutex g_backend_mu;
DaemonMemoryBackend *g_backend = nullptr;  // the daemon's one backend (reap_ipc_closes)
}  // namespace

DaemonMemoryBackend::DaemonMemoryBackend(GpuInventory inv) : inv_(std::move(inv)) {
    std::lock_guard<std::mutex> lk(g_backend_mu);
    g_backend = this;
}

DaemonMemoryBackend::~DaemonMemoryBackend() {
    {
        std::lock_guard<std::mutex> lk(g_backend_mu);
        if (g_backend == this) g_backend = nullptr;
    }
    for (int d = 0; d < inv_.count; ++d) reap(d);
}

void reap_ipc_closes(int device) noexcept {
    std::lock_guard<std::mutex> lk(g_backend_mu);
    if (g_backend != nullptr) g_backend->reap(device);
}

void DaemonMemoryBackend::reap(int device) noexcept {
    std::lock_guard<std::mutex> lk(mu_);
    if (device < 0 || device >= inv_.count) return;
    int prev = -1;
    for (auto it = open_.begin(); it != open_.end();) {
        Mapping &m = it->second;
        if (m.refs == 0 && m.bases[size_t(device)] != nullptr) {
            if (prev < 0) cudaGetDevice(&prev);
            cudaSetDevice(device);
            cudaIpcCloseMemHandle(m.bases[size_t(device)]);
            m.bases[size_t(device)] = nullptr;
            m.closed[size_t(device)] = 1;
        }
        bool any = false;
        for (void *b : m.bases) any |= b != nullptr;
        if (m.refs == 0 && !any)
            it = open_.erase(it);
        else
            ++it;
    }
    if (prev >= 0) cudaSetDevice(prev);
    (void)cudaGetLastError();
}

int DaemonMemoryBackend::open(control::MemoryDescriptor &desc, uint64_t length,
                              control::OpenedMemory *out) {
    if (desc.kind == control::MemKind::multicast) {
        if (inv_.count <= 0) return EOPNOTSUPP;
        McMapping m;
        const int rc = map_multicast(desc.region_fd.get(), desc.region_bytes, inv_.count, &m);
        desc.region_fd.reset();
        if (rc != 0) return rc;
        out->multicast = true;
        out->mc_handle = m.handle;
        out->mc_bytes = m.bytes;
        out->address = m.address;
        out->gpu = -2;  // no owner: every team GPU reaches it through the same multicast view
        out->device_address.assign(size_t(inv_.count), nullptr);
        for (int g = 0; g < inv_.count; ++g)
            if (m.reachable[size_t(g)]) out->device_address[size_t(g)] = m.address;
        return 0;
    }
    if (desc.kind == control::MemKind::host) {
        if (int rc = map_shared_fd(desc.region_fd.release(), 0, &out->host); rc != 0) return rc;
        if (desc.region_offset > out->host.bytes || length > out->host.bytes - desc.region_offset) {
            out->host.unmap();
            return EINVAL;
        }
        out->address = static_cast<uint8_t *>(out->host.address) + desc.region_offset;
        out->gpu = -1;
        out->device_address.assign(size_t(inv_.count), nullptr);
        if (inv_.count > 0) {
            // Pin and map the whole region once, portable to every GPU the executors run on.
            if (cudaHostRegister(out->host.address, out->host.bytes,
                                 cudaHostRegisterMapped | cudaHostRegisterPortable) == cudaSuccess) {
                void *dev = nullptr;
                if (cudaHostGetDevicePointer(&dev, out->host.address, 0) == cudaSuccess)
                    for (auto &d : out->device_address) d = static_cast<uint8_t *>(dev) + desc.region_offset;
                out->host_registered = out->host.address;
            }
            (void)cudaGetLastError();
        }
        return 0;
    }
    if (desc.ipc_handle.size() != sizeof(cudaIpcMemHandle_t)) return EINVAL;
    int gpu = -1;
    for (int i = 0; i < inv_.count; ++i)
        if (std::memcmp(inv_.uuids[i].data(), desc.uuid.data(), 16) == 0) gpu = i;
    if (gpu < 0) return ENODEV;  // the allocation lives on a GPU this daemon does not own
    std::lock_guard<std::mutex> lk(mu_);
    auto it = open_.find(desc.ipc_handle);
    if (it == open_.end()) {
        // Open the handle in every GPU's context: each executor stores / loads through a mapping
        // of its own (the owner's is local memory, the others reach it over NVLink).
        cudaIpcMemHandle_t h;
        std::memcpy(&h, desc.ipc_handle.data(), sizeof(h));
        int prev = 0;
        cudaGetDevice(&prev);
        Mapping m;
        m.gpu = gpu;
        m.bases.assign(size_t(inv_.count), nullptr);
        m.closed.assign(size_t(inv_.count), 0);
        bool ok = true;
        for (int d = 0; d < inv_.count && ok; ++d) {
            cudaSetDevice(d);
            if (cudaIpcOpenMemHandle(&m.bases[d], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                (void)cudaGetLastError();
                m.bases[d] = nullptr;
                ok = d != gpu;  // a peer that cannot map it only loses access; the owner must
            }
        }
        if (!ok) {
            for (int d = 0; d < inv_.count; ++d) {
                if (m.bases[d] == nullptr) continue;
                cudaSetDevice(d);
                cudaIpcCloseMemHandle(m.bases[d]);
            }
            cudaSetDevice(prev);
            return EACCES;
        }
        cudaSetDevice(prev);
        it = open_.emplace(desc.ipc_handle, std::move(m)).first;
    } else if (it->second.refs == 0) {
        // Unused and partly reaped: map it again on the GPUs that already closed it.
        cudaIpcMemHandle_t h;
        std::memcpy(&h, desc.ipc_handle.data(), sizeof(h));
        int prev = 0;
        cudaGetDevice(&prev);
        for (int d = 0; d < inv_.count; ++d) {
            if (!it->second.closed[size_t(d)]) continue;
            cudaSetDevice(d);
            if (cudaIpcOpenMemHandle(&it->second.bases[size_t(d)], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                (void)cudaGetLastError();
                it->second.bases[size_t(d)] = nullptr;
                if (d == gpu) {
                    cudaSetDevice(prev);
                    return EACCES;
                }
            }
            it->second.closed[size_t(d)] = 0;
        }
        cudaSetDevice(prev);
    }
    it->second.refs += 1;
    out->gpu = gpu;
    out->bases = it->second.bases;
    out->device_address.assign(size_t(inv_.count), nullptr);
    for (int d = 0; d < inv_.count; ++d)
        if (it->second.bases[d] != nullptr)
            out->device_address[d] = static_cast<uint8_t *>(it->second.bases[d]) + desc.allocation_offset;
    out->address = out->device_address[gpu];
    return 0;
}

void DaemonMemoryBackend::close(control::OpenedMemory &mem) noexcept {
    if (mem.multicast) {
        McMapping m;
        m.address = mem.address;
        m.bytes = mem.mc_bytes;
        m.handle = mem.mc_handle;
        unmap_multicast(m);
        mem.address = nullptr;
        mem.device_address.clear();
        mem.multicast = false;
        return;
    }
    if (mem.gpu < 0) {
        if (mem.host_registered != nullptr) cudaHostUnregister(mem.host_registered);
        mem.host_registered = nullptr;
        mem.device_address.clear();
        mem.host.unmap();
        mem.address = nullptr;
        return;
    }
    std::lock_guard<std::mutex> lk(mu_);
    for (auto it = open_.begin(); it != open_.end(); ++it) {
        if (it->second.bases != mem.bases) continue;
        it->second.refs -= 1;  // at 0 the mappings close in reap(), while no executor runs
        break;
    }
    mem.address = nullptr;
    mem.bases.clear();
    mem.device_address.clear();
}

}  // namespace ugdr::gpu
