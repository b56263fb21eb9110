// NVLink SHARP (NVLS) multicast memory for the collectives: one multicast object spanning every
// rank's GPU, each rank's physical memory bound to it, mapped twice in every process: a unicast
// view (this GPU's bytes, ordinary loads / stores) and a multicast view that only multimem.*
// instructions use.  A multimem.ld_reduce through the multicast view makes the NVSwitch read the
// same offset from every bound GPU and return the reduction; a multimem.st writes every GPU.
//
// The driver API is reached through cudaGetDriverEntryPoint, so libugdr.so loads (and its
// host-only parts run) on machines without a GPU driver.  The object is shared between the rank
// processes as a POSIX file descriptor (CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR); passing the
// descriptor between processes is the caller's job (SCM_RIGHTS over a Unix socket).
#include "ugdr/collective.h"

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <cerrno>
#include <cstdint>
#include <unistd.h>

namespace {

struct Driver {
    CUresult (*mc_create)(CUmemGenericAllocationHandle *, const CUmulticastObjectProp *) = nullptr;
    CUresult (*mc_granularity)(size_t *, const CUmulticastObjectProp *, CUmulticastGranularity_flags) = nullptr;
    CUresult (*mc_add_device)(CUmemGenericAllocationHandle, CUdevice) = nullptr;
    CUresult (*mc_bind_mem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                            unsigned long long) = nullptr;
    CUresult (*mc_unbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t) = nullptr;
    CUresult (*mem_create)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                           unsigned long long) = nullptr;
    CUresult (*mem_release)(CUmemGenericAllocationHandle) = nullptr;
    CUresult (*mem_granularity)(size_t *, const CUmemAllocationProp *, CUmemAllocationGranularity_flags) = nullptr;
    CUresult (*export_handle)(void *, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                              unsigned long long) = nullptr;
    CUresult (*import_handle)(CUmemGenericAllocationHandle *, void *, CUmemAllocationHandleType) = nullptr;
    CUresult (*reserve)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
    CUresult (*address_free)(CUdeviceptr, size_t) = nullptr;
    CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
    CUresult (*unmap)(CUdeviceptr, size_t) = nullptr;
    CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t) = nullptr;
    CUresult (*attribute)(int *, CUdevice_attribute, CUdevice) = nullptr;
    bool ok = false;
};

template <typename F> bool load(const char *name, F *fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return false;
    *fn = reinterpret_cast<F>(p);
    return true;
}

const Driver &drv() {
    static const Driver d = [] {
        Driver x;
        x.ok = load("cuMulticastCreate", &x.mc_create) && load("cuMulticastGetGranularity", &x.mc_granularity) &&
               load("cuMulticastAddDevice", &x.mc_add_device) && load("cuMulticastBindMem", &x.mc_bind_mem) &&
               load("cuMulticastUnbind", &x.mc_unbind) && load("cuMemCreate", &x.mem_create) &&
               load("cuMemRelease", &x.mem_release) &&
               load("cuMemGetAllocationGranularity", &x.mem_granularity) &&
               load("cuMemExportToShareableHandle", &x.export_handle) &&
               load("cuMemImportFromShareableHandle", &x.import_handle) &&
               load("cuMemAddressReserve", &x.reserve) && load("cuMemAddressFree", &x.address_free) &&
               load("cuMemMap", &x.map) && load("cuMemUnmap", &x.unmap) && load("cuMemSetAccess", &x.set_access) &&
               load("cuDeviceGetAttribute", &x.attribute);
        return x;
    }();
    return d;
}

// CUresult -> this ABI's cudaError_t-valued codes: success 0, anything else the CUresult itself
// (the two enums agree on the common values; callers only test for zero and print the rest).
int rc(CUresult r) { return int(r); }

int current_device(CUdevice *dev) {
    int ord = 0;
    if (cudaGetDevice(&ord) != cudaSuccess) return int(cudaErrorNoDevice);
    *dev = CUdevice(ord);
    return 0;
}

CUmemAllocationProp phys_prop(CUdevice dev) {
    CUmemAllocationProp p{};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = int(dev);
    p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return p;
}

// Multicast and physical granularity for `ndev` GPUs; sizes are rounded up to the larger one.
int granularity(int ndev, uint64_t bytes, CUdevice dev, size_t *gran) {
    const Driver &d = drv();
    CUmulticastObjectProp mp{};
    mp.numDevices = unsigned(ndev);
    mp.size = size_t(bytes);
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t g1 = 0, g2 = 0;
    CUresult r = d.mc_granularity(&g1, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) return rc(r);
    const CUmemAllocationProp pp = phys_prop(dev);
    r = d.mem_granularity(&g2, &pp, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) return rc(r);
    *gran = g1 > g2 ? g1 : g2;
    return 0;
}

uint64_t round_up(uint64_t v, uint64_t g) { return (v + g - 1) / g * g; }

}  // namespace

extern "C" {

int ugdr_x_nvls_supported(int device) {
    const Driver &d = drv();
    if (!d.ok) return 0;
    int v = 0;
    if (d.attribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, CUdevice(device)) != CUDA_SUCCESS) return 0;
    return v != 0;
}

int ugdr_x_nvls_create(int ndev, uint64_t bytes, ugdr_x_nvls *h, int *fd) {
    if (h == nullptr || fd == nullptr || ndev < 1 || ndev > UGDR_X_MAX_RANKS || bytes == 0)
        return int(cudaErrorInvalidValue);
    const Driver &d = drv();
    if (!d.ok) return int(cudaErrorNotSupported);
    *h = ugdr_x_nvls{};
    CUdevice dev;
    int e = current_device(&dev);
    if (e) return e;
    size_t g = 0;
    if ((e = granularity(ndev, bytes, dev, &g))) return e;
    CUmulticastObjectProp mp{};
    mp.numDevices = unsigned(ndev);
    mp.size = size_t(round_up(bytes, g));
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    CUmemGenericAllocationHandle mc = 0;
    CUresult r = d.mc_create(&mc, &mp);
    if (r != CUDA_SUCCESS) return rc(r);
    int out = -1;
    r = d.export_handle(&out, mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    if (r != CUDA_SUCCESS) {
        d.mem_release(mc);
        return rc(r);
    }
    h->mc_handle = uint64_t(mc);
    h->bytes = uint64_t(mp.size);
    h->device = int(dev);
    *fd = out;
    return 0;
}

int ugdr_x_nvls_import(int fd, int ndev, uint64_t bytes, ugdr_x_nvls *h) {
    if (h == nullptr || fd < 0 || ndev < 1 || bytes == 0) return int(cudaErrorInvalidValue);
    const Driver &d = drv();
    if (!d.ok) return int(cudaErrorNotSupported);
    *h = ugdr_x_nvls{};
    CUdevice dev;
    int e = current_device(&dev);
    if (e) return e;
    size_t g = 0;
    if ((e = granularity(ndev, bytes, dev, &g))) return e;
    CUmemGenericAllocationHandle mc = 0;
    const CUresult r =
        d.import_handle(&mc, reinterpret_cast<void *>(uintptr_t(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    if (r != CUDA_SUCCESS) return rc(r);
    h->mc_handle = uint64_t(mc);
    h->bytes = round_up(bytes, g);
    h->device = int(dev);
    return 0;
}

int ugdr_x_nvls_add_device(ugdr_x_nvls *h) {
    if (h == nullptr || h->mc_handle == 0) return int(cudaErrorInvalidValue);
    return rc(drv().mc_add_device(CUmemGenericAllocationHandle(h->mc_handle), CUdevice(h->device)));
}

int ugdr_x_nvls_bind(ugdr_x_nvls *h) {
    if (h == nullptr || h->mc_handle == 0 || h->mem_handle != 0) return int(cudaErrorInvalidValue);
    const Driver &d = drv();
    const CUdevice dev = CUdevice(h->device);
    const CUmemGenericAllocationHandle mc = CUmemGenericAllocationHandle(h->mc_handle);
    const size_t n = size_t(h->bytes);
    const CUmemAllocationProp pp = phys_prop(dev);
    CUmemGenericAllocationHandle mem = 0;
    CUresult r = d.mem_create(&mem, n, &pp, 0);
    if (r != CUDA_SUCCESS) return rc(r);
    CUdeviceptr uc = 0, mv = 0;
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = int(dev);
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    bool bound = false, uc_mapped = false;
    auto fail = [&](CUresult why) {
        if (uc_mapped) d.unmap(uc, n);
        if (uc) d.address_free(uc, n);
        if (bound) d.mc_unbind(mc, dev, 0, n);
        if (mv) d.address_free(mv, n);
        d.mem_release(mem);
        return rc(why);
    };
    if ((r = d.mc_bind_mem(mc, 0, mem, 0, n, 0)) != CUDA_SUCCESS) return fail(r);
    bound = true;
    if ((r = d.reserve(&uc, n, 0, 0, 0)) != CUDA_SUCCESS) return fail(r);
    if ((r = d.map(uc, n, 0, mem, 0)) != CUDA_SUCCESS) return fail(r);
    uc_mapped = true;
    if ((r = d.set_access(uc, n, &acc, 1)) != CUDA_SUCCESS) return fail(r);
    if ((r = d.reserve(&mv, n, 0, 0, 0)) != CUDA_SUCCESS) return fail(r);
    if ((r = d.map(mv, n, 0, mc, 0)) != CUDA_SUCCESS) {
        d.address_free(mv, n);
        mv = 0;
        return fail(r);
    }
    if ((r = d.set_access(mv, n, &acc, 1)) != CUDA_SUCCESS) {
        d.unmap(mv, n);
        return fail(r);
    }
    h->mem_handle = uint64_t(mem);
    h->uc = reinterpret_cast<void *>(uc);
    h->mc = reinterpret_cast<void *>(mv);
    return 0;
}

int ugdr_x_nvls_release(ugdr_x_nvls *h) {
    if (h == nullptr) return int(cudaErrorInvalidValue);
    const Driver &d = drv();
    if (!d.ok) return int(cudaErrorNotSupported);
    const size_t n = size_t(h->bytes);
    const CUmemGenericAllocationHandle mc = CUmemGenericAllocationHandle(h->mc_handle);
    if (h->mc != nullptr) {
        d.unmap(CUdeviceptr(reinterpret_cast<uintptr_t>(h->mc)), n);
        d.address_free(CUdeviceptr(reinterpret_cast<uintptr_t>(h->mc)), n);
    }
    if (h->mem_handle != 0) d.mc_unbind(mc, CUdevice(h->device), 0, n);
    if (h->uc != nullptr) {
        d.unmap(CUdeviceptr(reinterpret_cast<uintptr_t>(h->uc)), n);
        d.address_free(CUdeviceptr(reinterpret_cast<uintptr_t>(h->uc)), n);
    }
    if (h->mem_handle != 0) d.mem_release(CUmemGenericAllocationHandle(h->mem_handle));
    if (mc != 0) d.mem_release(mc);
    *h = ugdr_x_nvls{};
    return 0;
}

}  // extern "C"
