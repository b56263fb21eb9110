// Client <-> daemon control transport: Unix SOCK_SEQPACKET, one datagram per message, file
// descriptors carried with SCM_RIGHTS.
//
// Wire envelope (36 bytes, big-endian), kept identical to the reference so either side can talk
// to the other (src/ipc/protocol.cpp:42-70): magic u32 0x49504331, version u16.u16 = 1.0,
// method u32, flags u32 (bit 0 = response), request id u64, status i32, payload length u32,
// fd count u32.  Payload <= 1 MiB, <= 16 fds.
#pragma once

#include "common/fd.hpp"

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <unordered_map>
#include <vector>

namespace ugdr::ipc {

constexpr uint32_t kMagic = 0x49504331u;
constexpr uint16_t kVersionMajor = 1;
constexpr uint16_t kVersionMinor = 0;
constexpr uint32_t kFlagResponse = 1u;
constexpr size_t kEnvelopeBytes = 36;
constexpr size_t kMaxPayload = 1u << 20;
constexpr size_t kMaxFds = 16;

struct Envelope {
    uint32_t magic = kMagic;
    uint16_t major = kVersionMajor;
    uint16_t minor = kVersionMinor;
    uint32_t method = 0;
    uint32_t flags = 0;
    uint64_t request_id = 0;
    int32_t status = 0;
    uint32_t payload_length = 0;
    uint32_t fd_count = 0;
};

struct Message {
    Envelope env;
    std::vector<std::byte> payload;
    std::vector<Fd> fds;
    // The payload arrived whole but the kernel could not install every attached descriptor
    // (the receiver is at its descriptor limit).  `fds` holds the ones that did arrive.
    bool fds_truncated = false;
};

void encode_envelope(const Envelope &e, uint8_t out[kEnvelopeBytes]);
Envelope decode_envelope(const uint8_t in[kEnvelopeBytes]);

// Send one message.  Returns 0 or a positive errno.
int send_message(int sock, const Message &m);
// Receive one message.  Returns 0, ECONNRESET on orderly EOF, or a positive errno (EPROTO for a
// malformed envelope, EMSGSIZE for truncation).
// `nonblocking`: return EAGAIN at once when no message is waiting.
int recv_message(int sock, Message *m, bool nonblocking = false);

class Client {
  public:
    int connect(const std::string &path);
    // Synchronous request / response; `resp` keeps the reply.  Returns 0 or a positive errno
    // for transport failures; the reply's env.status carries the service result.
    // `min_wait_ms` raises the reply deadline for this call (requests that wait on purpose, such
    // as a timed drain).
    int call(uint32_t method, std::vector<std::byte> payload, std::vector<Fd> fds, Message *resp,
             uint64_t min_wait_ms = 0);
    void close() { sock_.reset(); }
    bool connected() const { return sock_.valid(); }

  private:
    Fd sock_;
    uint64_t next_id_ = 1;
    uint64_t timeout_ms_ = 0;  // reply deadline set at connect (0: none)
};

using SessionId = uint64_t;

class Handler {
  public:
    virtual ~Handler() = default;
    // Build the response for `req` (the server fills id / flags / method).
    virtual Message handle(SessionId session, Message &&req) = 0;
    virtual void on_disconnect(SessionId) noexcept {}
};

class Server {
  public:
    explicit Server(Handler &h) : handler_(h) {}
    ~Server() { close(); }
    Server(const Server &) = delete;
    Server &operator=(const Server &) = delete;

    // Bind and listen on `path`.  An existing socket file is replaced only when nothing is
    // accepting on it (a stale socket from a dead daemon).
    int start(const std::string &path);
    // Wait up to `timeout_ms` for activity and serve it.  Returns 0 or a positive errno.
    int poll_once(int timeout_ms);
    void close() noexcept;
    size_t session_count() const { return sessions_.size(); }
    // Steady-clock nanoseconds of the last request served (0 before the first).
    uint64_t last_served_ns() const { return last_served_ns_; }
    bool running() const { return listener_.valid(); }
    const std::string &path() const { return path_; }

  private:
    void drop(int fd) noexcept;

    Handler &handler_;
    Fd listener_;
    // A descriptor held back so that, at the descriptor limit, a pending connection can still be
    // accepted and closed (the client sees the refusal) instead of keeping the listener readable.
    Fd reserve_;
    std::string path_;
    uint64_t sock_dev_ = 0, sock_ino_ = 0;
    struct Session {
        Fd sock;
        SessionId id = 0;
    };
    std::unordered_map<int, Session> sessions_;
    SessionId next_session_ = 1;
    uint64_t last_served_ns_ = 0;
};

}  // namespace ugdr::ipc
