// One GPU's engine: device-memory mirrors of the MR / QP / CQ tables, ring registration with
// CUDA, and the launch / monitor / quiesce life cycle of the persistent executor kernel.
//
// Parity: reference PersistentCudaCopyBackend / PersistentCudaCopyHost
// (src/gpu/persistent_copy_backend.cu:59-692) and the queue owners of
// src/gpu/persistent_copy.cu:2098-3049.  The reference keeps a host thread on the data path
// (batching 8 KiB tasks into a mapped ring); this engine's host thread only (re)launches the
// kernel when rings hold work and the kernel is not running, and stops it for control
// operations that retire device-visible objects.
#pragma once

#include "control/objects.hpp"

#include <memory>
#include <mutex>

namespace ugdr::gpu {

struct GpuEngineConfig {
    int ordinal = 0;
    int ctas = 148;
    uint32_t idle_exit_us = 200000;
    uint32_t max_wait_ms = 2000;  // bound on every device-side spin
    uint32_t bulk_min_bytes = 8192;  // TMA bulk-copy path for aligned chunk pieces this long (0: off)
};

// Build the engine for one GPU.  Returns 0 or a positive errno (ENODEV without CUDA).
int make_gpu_engine(const GpuEngineConfig &cfg, std::mutex &objects_mu,
                    std::unique_ptr<control::Engine> *out);

}  // namespace ugdr::gpu
