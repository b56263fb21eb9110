// Control RPC payloads carried inside the IPC envelope.
//
// Request prefix (32 B, big-endian): version u16 = 1, reserved u16 = 0, identity u64,
// length u64, access u32, opaque length u32, fd-index count u32; then the opaque bytes, then one
// u32 per fd index.  Response prefix (20 B): version, reserved, identity u64, opaque length u32,
// index count u32; the status travels in the envelope.  Same framing as the reference
// (src/control/ipc_adapter.cpp:87-258); methods 1-15 keep its numbering
// (src/control/device_context.hpp:16-32), methods from 32 up are this build's extensions.
#pragma once

#include "common/fd.hpp"
#include "ipc/ipc.hpp"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace ugdr::control {

constexpr uint16_t kPayloadVersion = 1;
constexpr size_t kRequestPrefix = 32;
constexpr size_t kResponsePrefix = 20;

enum Method : uint32_t {
    kListDevices = 1,
    kCreateContext = 2,
    kDestroyContext = 3,
    kCreatePd = 4,
    kDestroyPd = 5,
    kRegisterMr = 6,
    kDeregisterMr = 7,
    kCreateCq = 8,
    kDestroyCq = 9,
    kCreateQp = 10,
    kDestroyQp = 11,
    kQueryQp = 12,
    kModifyQp = 13,
    kQueryQpConnInfo = 14,
    kConnectQp = 15,
    // extensions
    kEngineStats = 32,
    kEngineHold = 33,
    kTimedDrain = 34,
    kQpStats = 35,
    kEngineTrace = 36,
    kDaemonStats = 37,
};

struct Request {
    uint32_t method = 0;
    uint64_t identity = 0;
    uint64_t length = 0;
    uint32_t access = 0;
    std::vector<std::byte> opaque;
    std::vector<Fd> fds;  // attached descriptors, in index order
};

struct Response {
    int32_t status = 0;  // 0 or a positive errno
    uint64_t identity = 0;
    std::vector<std::byte> opaque;
    std::vector<Fd> fds;
};

int encode_request(Request &&req, ipc::Message *out);
int decode_request(ipc::Message &&msg, Request *out);
int encode_response(uint32_t method, Response &&resp, ipc::Message *out);
int decode_response(ipc::Message &&msg, Response *out);

}  // namespace ugdr::control
