// Client-side control channel: one daemon connection per process, typed request helpers, and a
// connection epoch that advances on every (re)connect so proxies from a lost connection are
// recognisably stale (reference: src/control/device_context.cpp:240-370).
#pragma once

#include "control/rpc.hpp"
#include "ipc/ipc.hpp"

#include <cstdint>
#include <mutex>
#include <string>

namespace ugdr::control {

class ControlClient {
  public:
    int connect(const std::string &path);
    void close();
    bool connected() const { return ipc_.connected(); }
    uint64_t epoch() const { return epoch_; }
    // Transport failures close the channel (the epoch then changes on reconnect) and come back
    // as a positive errno; service failures come back in resp->status.
    int call(Request &&req, Response *resp, uint64_t min_wait_ms = 0);

  private:
    ipc::Client ipc_;
    uint64_t epoch_ = 0;
};

}  // namespace ugdr::control
