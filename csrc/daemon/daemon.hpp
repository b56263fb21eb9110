// The daemon composition root: control plane + IPC server + one engine per device.
//
// Parity: reference apps/daemon/main.cpp:22-63, which serves the control plane only (no data
// path); here the daemon also owns the executors, so a client's posted WRs are executed
// without any test harness in between.
#pragma once

#include "control/objects.hpp"

#include <atomic>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace ugdr::control {
class ControlPlane;
}
namespace ugdr::ipc {
class Server;
}

namespace ugdr::daemon {

struct Options {
    std::string socket_path;
    int gpus = -1;          // GPUs to own (-1: all visible)
    bool cpu_device = true; // expose the host-memory engine as a device
    int executor_ctas = 0;  // CTAs per GPU executor (0: one per SM)
    int bulk_min_bytes = -1;  // TMA bulk-copy threshold of the executors (-1: engine default, 0: off)
    uint32_t idle_exit_us = 200000;  // executor exits after this long without work
};

class Daemon {
  public:
    explicit Daemon(Options opt);
    ~Daemon();
    // Bind the socket and build the engines.  Returns 0 or a positive errno.
    int start();
    // Serve until `stop` becomes true.
    int run(const std::atomic<bool> &stop);
    // Serve one poll round (tests).
    int poll_once(int timeout_ms);
    size_t device_count() const;

  private:
    class LockedHandler;
    Options opt_;
    std::mutex objects_mu_;
    std::vector<std::unique_ptr<control::Engine>> engines_;
    std::unique_ptr<control::MemoryBackend> memory_;
    std::unique_ptr<control::ControlPlane> plane_;
    std::unique_ptr<LockedHandler> handler_;
    std::unique_ptr<ipc::Server> server_;
};

}  // namespace ugdr::daemon
