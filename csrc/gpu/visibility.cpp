#include "gpu/visibility.hpp"

#include <cuda_runtime_api.h>

#include <cerrno>

namespace ugdr::gpu {

int CudaVisibilitySource::query(int device, VisibilityAttrs *out) {
    int sup = 0, opts = 0, ord = 0;
    if (cudaDeviceGetAttribute(&sup, cudaDevAttrGPUDirectRDMASupported, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&opts, cudaDevAttrGPUDirectRDMAFlushWritesOptions, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&ord, cudaDevAttrGPUDirectRDMAWritesOrdering, device) != cudaSuccess) {
        cudaGetLastError();
        return ENODEV;
    }
    out->rdma_supported = sup != 0;
    out->flush_options = opts;
    out->writes_ordering = ord;
    return 0;
}

int CudaVisibilitySource::flush(int device) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return ENODEV;
    if (cur != device && cudaSetDevice(device) != cudaSuccess) return ENODEV;
    const cudaError_t e =
        cudaDeviceFlushGPUDirectRDMAWrites(cudaFlushGPUDirectRDMAWritesTargetCurrentDevice,
                                           cudaFlushGPUDirectRDMAWritesToOwner);
    if (cur != device) cudaSetDevice(cur);
    return e == cudaSuccess ? 0 : EIO;
}

int VisibilityGate::init(int device) {
    device_ = device;
    const int rc = src_.query(device_, &attrs_);
    if (rc != 0) {
        mode_ = Mode::kUnavailable;
        return rc;
    }
    if (attrs_.rdma_supported && attrs_.writes_ordering >= kOrderingOwner)
        mode_ = Mode::kOrdered;
    else if (attrs_.rdma_supported && (attrs_.flush_options & kFlushHost) != 0)
        mode_ = Mode::kFlush;
    else
        mode_ = Mode::kUnavailable;
    return 0;
}

int VisibilityGate::before_publish() {
    switch (mode_) {
    case Mode::kOrdered:
        return 0;
    case Mode::kFlush: {
        const int rc = src_.flush(device_);
        if (rc == 0) ++flushes_;
        return rc;
    }
    case Mode::kUnavailable:
        break;
    }
    return EOPNOTSUPP;
}

}  // namespace ugdr::gpu
