// Daemon-side mapping of an NVLink multicast object that a client registers as an MR.  The
// client processes created the object, added their GPUs and bound their memory; the daemon only
// imports the object from its POSIX shareable handle, maps it into its own address space and
// enables access for each of its GPUs that belongs to the object's team, so the executors of
// those GPUs can issue multimem loads and stores through it.
//
// Driver entry points come from cudaGetDriverEntryPoint, so libugdr.so still loads where there
// is no driver (the open then fails with EOPNOTSUPP).
#include "gpu/multicast.hpp"

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <cerrno>

namespace ugdr::gpu {
namespace {

struct McDriver {
    CUresult (*import_handle)(CUmemGenericAllocationHandle *, void *, CUmemAllocationHandleType) = nullptr;
    CUresult (*reserve)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
    CUresult (*address_free)(CUdeviceptr, size_t) = nullptr;
    CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
    CUresult (*unmap)(CUdeviceptr, size_t) = nullptr;
    CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t) = nullptr;
    CUresult (*release)(CUmemGenericAllocationHandle) = nullptr;
    bool ok = false;
};

template <typename F> bool entry(const char *name, F *fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    *fn = reinterpret_cast<F>(p);
    return true;
}

const McDriver &drv() {
    static const McDriver d = [] {
        McDriver x;
        x.ok = entry("cuMemImportFromShareableHandle", &x.import_handle) && entry("cuMemAddressReserve", &x.reserve) &&
               entry("cuMemAddressFree", &x.address_free) && entry("cuMemMap", &x.map) &&
               entry("cuMemUnmap", &x.unmap) && entry("cuMemSetAccess", &x.set_access) &&
               entry("cuMemRelease", &x.release);
        return x;
    }();
    return d;
}

}  // namespace

int map_multicast(int fd, uint64_t bytes, int gpus, McMapping *out) {
    *out = McMapping{};
    if (fd < 0 || bytes == 0 || gpus <= 0) return EINVAL;
    const McDriver &d = drv();
    if (!d.ok) return EOPNOTSUPP;
    CUmemGenericAllocationHandle h = 0;
    if (d.import_handle(&h, reinterpret_cast<void *>(uintptr_t(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) !=
        CUDA_SUCCESS)
        return EINVAL;
    CUdeviceptr va = 0;
    if (d.reserve(&va, size_t(bytes), 0, 0, 0) != CUDA_SUCCESS) {
        d.release(h);
        return ENOMEM;
    }
    if (d.map(va, size_t(bytes), 0, h, 0) != CUDA_SUCCESS) {
        d.address_free(va, size_t(bytes));
        d.release(h);
        return EINVAL;
    }
    // Access per GPU: a GPU outside the object's team refuses, and only loses the MR.
    int granted = 0;
    out->reachable.assign(size_t(gpus), false);
    for (int g = 0; g < gpus; ++g) {
        CUmemAccessDesc acc{};
        acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc.location.id = g;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        if (d.set_access(va, size_t(bytes), &acc, 1) == CUDA_SUCCESS) {
            out->reachable[size_t(g)] = true;
            ++granted;
        }
    }
    if (granted == 0) {
        d.unmap(va, size_t(bytes));
        d.address_free(va, size_t(bytes));
        d.release(h);
        return EACCES;
    }
    out->handle = uint64_t(h);
    out->address = reinterpret_cast<void *>(va);
    out->bytes = bytes;
    return 0;
}

void unmap_multicast(McMapping &m) noexcept {
    const McDriver &d = drv();
    if (!d.ok || m.address == nullptr) return;
    const CUdeviceptr va = CUdeviceptr(reinterpret_cast<uintptr_t>(m.address));
    d.unmap(va, size_t(m.bytes));
    d.address_free(va, size_t(m.bytes));
    d.release(CUmemGenericAllocationHandle(m.handle));
    m = McMapping{};
}

}  // namespace ugdr::gpu
