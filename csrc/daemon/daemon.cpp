#include "daemon/daemon.hpp"

#include "control/service.hpp"
#include "engine/cpu_engine.hpp"
#include "gpu/cuda_memory.hpp"
#include "gpu/gpu_engine.hpp"
#include "ipc/ipc.hpp"

#include <chrono>
#include <cerrno>
#include <cstdio>

namespace ugdr::daemon {

// Serialises control requests against the engines' host threads.
class Daemon::LockedHandler : public ipc::Handler {
  public:
    LockedHandler(std::mutex &mu, control::ControlPlane &plane) : mu_(mu), plane_(plane) {}
    ipc::Message handle(ipc::SessionId s, ipc::Message &&m) override {
        std::lock_guard<std::mutex> lk(mu_);
        return plane_.handle(s, std::move(m));
    }
    void on_disconnect(ipc::SessionId s) noexcept override {
        std::lock_guard<std::mutex> lk(mu_);
        plane_.on_disconnect(s);
    }

  private:
    std::mutex &mu_;
    control::ControlPlane &plane_;
};

Daemon::Daemon(Options opt) : opt_(std::move(opt)) {}

Daemon::~Daemon() {
    if (server_) server_->close();
    {
        std::lock_guard<std::mutex> lk(objects_mu_);
        plane_.reset();
    }
    engines_.clear();
}

int Daemon::start() {
    gpu::GpuInventory inv = gpu::probe_gpus(opt_.gpus);
    if (inv.count > 1) gpu::enable_all_peer_access(inv.count);
    for (int g = 0; g < inv.count; ++g) {
        gpu::GpuEngineConfig cfg;
        cfg.ordinal = g;
        cfg.ctas = opt_.executor_ctas > 0 ? opt_.executor_ctas : inv.sm_count[g];
        cfg.idle_exit_us = opt_.idle_exit_us;
        if (opt_.bulk_min_bytes >= 0) cfg.bulk_min_bytes = uint32_t(opt_.bulk_min_bytes);
        std::unique_ptr<control::Engine> e;
        if (int rc = gpu::make_gpu_engine(cfg, objects_mu_, &e); rc != 0) {
            std::fprintf(stderr, "ugdr_daemon: GPU %d engine unavailable (%d)\n", g, rc);
            continue;
        }
        engines_.push_back(std::move(e));
    }
    if (opt_.cpu_device) engines_.push_back(std::make_unique<engine::CpuEngine>(objects_mu_));
    if (engines_.empty()) return ENODEV;
    std::vector<control::Engine *> raw;
    for (auto &e : engines_) raw.push_back(e.get());
    memory_ = std::make_unique<gpu::DaemonMemoryBackend>(inv);
    plane_ = std::make_unique<control::ControlPlane>(raw, *memory_);
    handler_ = std::make_unique<LockedHandler>(objects_mu_, *plane_);
    server_ = std::make_unique<ipc::Server>(*handler_);
    return server_->start(opt_.socket_path);
}

int Daemon::poll_once(int timeout_ms) { return server_ ? server_->poll_once(timeout_ms) : EBADF; }

// Clients send control requests in bursts (create, modify, connect, ...): for 200 us after a
// request the loop polls without sleeping, so the next request is not delayed by a wake-up.
int Daemon::run(const std::atomic<bool> &stop) {
    while (!stop.load()) {
        const uint64_t now = uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                          std::chrono::steady_clock::now().time_since_epoch())
                                          .count());
        const uint64_t last = server_->last_served_ns();
        const int timeout_ms = last != 0 && now - last < 200000 ? 0 : 50;
        if (int rc = server_->poll_once(timeout_ms); rc != 0) return rc;
    }
    return 0;
}

size_t Daemon::device_count() const { return engines_.size(); }

}  // namespace ugdr::daemon
