// GPUDirect write-visibility gate (parity: the reference's src/gpu/gpudirect_visibility.cu:37-126).
//
// When a third party (a NIC, or any GPUDirect RDMA writer) writes GPU memory, CUDA only
// guarantees that a kernel sees those writes in order if the device reports
// GPU_DIRECT_RDMA_WRITES_ORDERING >= OWNER; below that, the host must flush
// (cudaDeviceFlushGPUDirectRDMAWrites) before it tells a kernel the data is there.  The executor
// is told about new work by the host (relaunch) and by ring cursors in host memory; the gate is
// consulted on that path.  Payload moved by the executor itself over NVLink never needs a flush
// (the GPU is the writer), so on B200 the gate normally reports "ordered" and costs a branch.
//
// Attribute queries and the flush go through small interfaces so the decision logic is tested
// on the host with fakes.
#pragma once

#include <cstdint>

namespace ugdr::gpu {

struct VisibilityAttrs {
    bool rdma_supported = false;
    int flush_options = 0;    // bitmask: 1 = host flush call available, 2 = stream memops
    int writes_ordering = 0;  // 0 none, 100 owner, 200 all devices
};

class VisibilitySource {
  public:
    virtual ~VisibilitySource() = default;
    virtual int query(int device, VisibilityAttrs *out) = 0;  // 0 or a positive errno
    virtual int flush(int device) = 0;                          // 0 or a positive errno
};

// The CUDA runtime's attributes and flush.
class CudaVisibilitySource final : public VisibilitySource {
  public:
    int query(int device, VisibilityAttrs *out) override;
    int flush(int device) override;
};

class VisibilityGate {
  public:
    enum class Mode { kOrdered, kFlush, kUnavailable };
    static constexpr int kOrderingOwner = 100;
    static constexpr int kFlushHost = 1;

    explicit VisibilityGate(VisibilitySource &src) : src_(src) {}
    // Query `device` once.  Returns 0, or the query's error (the gate then stays unavailable).
    int init(int device);
    Mode mode() const { return mode_; }
    const VisibilityAttrs &attrs() const { return attrs_; }
    // Call before telling a kernel that externally written data is ready.  Ordered: nothing to
    // do.  Flush: one host flush; a failure is returned and the caller must not publish.
    // Unavailable (no GPUDirect RDMA, or ordering below owner with no host flush): returns
    // EOPNOTSUPP so that a caller relying on third-party writes cannot silently proceed.
    int before_publish();
    uint64_t flushes() const { return flushes_; }

  private:
    VisibilitySource &src_;
    int device_ = 0;
    VisibilityAttrs attrs_{};
    Mode mode_ = Mode::kUnavailable;
    uint64_t flushes_ = 0;
};

}  // namespace ugdr::gpu
