// IPC envelope and transport tests (reference: tests/unit/ipc_protocol_test.cpp, ipc_adapter_test.cpp,
// tests/integration/ipc_client_server_test.cpp).
#include "harness.hpp"

#include "control/rpc.hpp"
#include "control/handles.hpp"
#include "ipc/ipc.hpp"

#include <fcntl.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <cstring>
#include <string>
#include <thread>

using namespace ugdr;

TEST(ipc_envelope_is_big_endian_36_bytes) {
    ipc::Envelope e;
    e.method = 0x01020304;
    e.flags = 1;
    e.request_id = 0x1122334455667788ull;
    e.status = -5;
    e.payload_length = 9;
    e.fd_count = 2;
    uint8_t b[ipc::kEnvelopeBytes];
    ipc::encode_envelope(e, b);
    const uint8_t magic[4] = {0x49, 0x50, 0x43, 0x31};
    CHECK(std::memcmp(b, magic, 4) == 0);
    CHECK_EQ(b[4], 0);
    CHECK_EQ(b[5], 1);  // major 1
    CHECK_EQ(b[8], 0x01);
    CHECK_EQ(b[11], 0x04);
    CHECK_EQ(b[16], 0x11);
    CHECK_EQ(b[23], 0x88);
    const ipc::Envelope d = ipc::decode_envelope(b);
    CHECK_EQ(d.method, e.method);
    CHECK_EQ(d.request_id, e.request_id);
    CHECK_EQ(d.status, -5);
    CHECK_EQ(d.payload_length, 9u);
    CHECK_EQ(d.fd_count, 2u);
}

TEST(ipc_socketpair_roundtrip_with_fds) {
    int sv[2];
    CHECK_EQ(::socketpair(AF_UNIX, SOCK_SEQPACKET, 0, sv), 0);
    ipc::Message m;
    m.env.method = 7;
    m.env.request_id = 42;
    m.payload.resize(1000);
    for (size_t i = 0; i < m.payload.size(); ++i) m.payload[i] = std::byte(i * 7);
    int p[2];
    CHECK_EQ(::pipe(p), 0);
    m.fds.emplace_back(p[0]);
    CHECK_EQ(ipc::send_message(sv[0], m), 0);
    ipc::Message r;
    CHECK_EQ(ipc::recv_message(sv[1], &r), 0);
    CHECK_EQ(r.env.method, 7u);
    CHECK_EQ(r.env.request_id, 42u);
    CHECK(r.payload == m.payload);
    CHECK_EQ(r.fds.size(), 1u);
    // The received descriptor is the pipe's read end: data written to p[1] comes out of it.
    CHECK_EQ(::write(p[1], "x", 1), 1);
    char c = 0;
    CHECK_EQ(::read(r.fds[0].get(), &c, 1), 1);
    CHECK_EQ(c, 'x');
    ::close(p[1]);
    ::close(sv[0]);
    ipc::Message eof;
    CHECK_EQ(ipc::recv_message(sv[1], &eof), ECONNRESET);
    ::close(sv[1]);
}

TEST(ipc_rejects_bad_magic_and_length) {
    int sv[2];
    CHECK_EQ(::socketpair(AF_UNIX, SOCK_SEQPACKET, 0, sv), 0);
    uint8_t b[ipc::kEnvelopeBytes + 4] = {};
    ipc::Envelope e;
    e.payload_length = 4;
    ipc::encode_envelope(e, b);
    b[0] = 0;  // bad magic
    CHECK_EQ(::send(sv[0], b, sizeof(b), 0), ssize_t(sizeof(b)));
    ipc::Message r;
    CHECK_EQ(ipc::recv_message(sv[1], &r), EPROTO);
    ipc::encode_envelope(e, b);
    CHECK_EQ(::send(sv[0], b, ipc::kEnvelopeBytes + 2, 0), ssize_t(ipc::kEnvelopeBytes + 2));  // short
    CHECK_EQ(ipc::recv_message(sv[1], &r), EPROTO);
    CHECK_EQ(::send(sv[0], b, 10, 0), 10);  // truncated header
    CHECK_EQ(ipc::recv_message(sv[1], &r), EPROTO);
    ::close(sv[0]);
    ::close(sv[1]);
}

TEST(ipc_send_validates) {
    ipc::Message m;
    m.payload.resize(ipc::kMaxPayload + 1);
    CHECK_EQ(ipc::send_message(3, m), EINVAL);
    ipc::Message f;
    for (int i = 0; i < 17; ++i) f.fds.emplace_back(::dup(0));
    CHECK_EQ(ipc::send_message(3, f), EINVAL);
}

namespace {
class Echo : public ipc::Handler {
  public:
    ipc::Message handle(ipc::SessionId s, ipc::Message &&req) override {
        ipc::Message r;
        r.env.status = int32_t(s);
        r.payload = req.payload;
        return r;
    }
    void on_disconnect(ipc::SessionId s) noexcept override {
        last_gone.store(int64_t(s));
        if (watch.load() == int64_t(s)) watched_gone.store(true);
        disconnects++;
    }
    std::atomic<int> disconnects{0};
    std::atomic<int64_t> last_gone{-1}, watch{-1};
    std::atomic<bool> watched_gone{false};
};
}  // namespace

TEST(ipc_client_server_sessions) {
    const std::string path = "/tmp/ugdr-test-" + std::to_string(::getpid()) + ".sock";
    Echo h;
    ipc::Server srv(h);
    CHECK_EQ(srv.start(path), 0);
    ipc::Server second(h);
    CHECK_EQ(second.start(path), EADDRINUSE);  // a live server keeps its socket
    std::atomic<bool> stop{false};
    std::thread loop([&] {
        while (!stop.load()) srv.poll_once(10);
    });
    ipc::Client a, b;
    CHECK_EQ(a.connect(path), 0);
    CHECK_EQ(b.connect(path), 0);
    ipc::Message ra, rb;
    std::vector<std::byte> pa(3, std::byte(1)), pb(5, std::byte(2));
    CHECK_EQ(a.call(9, pa, {}, &ra), 0);
    CHECK_EQ(b.call(9, pb, {}, &rb), 0);
    CHECK(ra.payload == pa && rb.payload == pb);
    CHECK(ra.env.status != rb.env.status);  // distinct session ids
    CHECK_EQ(ra.env.flags, ipc::kFlagResponse);
    // The second server's liveness probe is also a session (it connects and leaves), so watch
    // for client a's session id specifically.
    h.watch.store(int64_t(ra.env.status));
    a.close();
    for (int i = 0; i < 5000 && !h.watched_gone.load(); ++i) usleep(1000);  // bounded: 5 s
    CHECK(h.watched_gone.load());
    CHECK(h.disconnects.load() <= 2);  // a, and possibly the probe; b is still connected
    stop.store(true);
    loop.join();
    srv.close();
    CHECK(::access(path.c_str(), F_OK) != 0);  // socket file removed
}

TEST(rpc_request_response_roundtrip) {
    control::Request q;
    q.method = control::kRegisterMr;
    q.identity = 0x0203000000000001ull;
    q.length = 4096;
    q.access = 3;
    q.opaque = {std::byte(1), std::byte(2)};
    int p[2];
    CHECK_EQ(::pipe(p), 0);
    q.fds.emplace_back(p[0]);
    q.fds.emplace_back(p[1]);
    ipc::Message m;
    CHECK_EQ(control::encode_request(std::move(q), &m), 0);
    CHECK_EQ(m.payload.size(), control::kRequestPrefix + 2 + 8);
    control::Request d;
    CHECK_EQ(control::decode_request(std::move(m), &d), 0);
    CHECK_EQ(d.method, uint32_t(control::kRegisterMr));
    CHECK_EQ(d.identity, 0x0203000000000001ull);
    CHECK_EQ(d.length, 4096u);
    CHECK_EQ(d.access, 3u);
    CHECK_EQ(d.opaque.size(), 2u);
    CHECK_EQ(d.fds.size(), 2u);

    control::Response s;
    s.status = EBUSY;
    s.identity = 77;
    s.opaque.resize(5);
    ipc::Message rm;
    CHECK_EQ(control::encode_response(6, std::move(s), &rm), 0);
    CHECK_EQ(rm.payload.size(), control::kResponsePrefix + 5);
    control::Response sd;
    CHECK_EQ(control::decode_response(std::move(rm), &sd), 0);
    CHECK_EQ(sd.status, EBUSY);
    CHECK_EQ(sd.identity, 77u);
    CHECK_EQ(sd.opaque.size(), 5u);
}

TEST(rpc_rejects_malformed) {
    ipc::Message m;
    m.env.method = 1;
    m.payload.resize(10);
    control::Request d;
    CHECK_EQ(control::decode_request(std::move(m), &d), EPROTO);
    control::Request q;
    q.method = 1;
    ipc::Message ok;
    CHECK_EQ(control::encode_request(std::move(q), &ok), 0);
    ok.payload[0] = std::byte(9);  // version
    CHECK_EQ(control::decode_request(std::move(ok), &d), EPROTONOSUPPORT);
}

TEST(registry_generations_and_sessions) {
    control::Registry<int> reg(control::ObjectType::pd, 4);
    const uint64_t a = reg.insert(1, std::make_unique<int>(10));
    CHECK(a != 0);
    CHECK_EQ(uint32_t(control::identity_type(a)), uint32_t(control::ObjectType::pd));
    CHECK(reg.find(1, a) != nullptr);
    CHECK(reg.find(2, a) == nullptr);       // foreign session
    CHECK(reg.find_any(a) != nullptr);
    CHECK(reg.erase(a) != nullptr);
    CHECK(reg.find(1, a) == nullptr);       // stale
    const uint64_t b = reg.insert(1, std::make_unique<int>(11));
    CHECK_EQ(control::identity_slot(b), control::identity_slot(a));  // slot reused ...
    CHECK(b != a);                                                     // ... with a new generation
    CHECK(reg.find(1, a) == nullptr);
    for (int i = 0; i < 3; ++i) CHECK(reg.insert(1, std::make_unique<int>(i)) != 0);
    CHECK(reg.full());
    CHECK_EQ(reg.insert(1, std::make_unique<int>(99)), 0u);
    CHECK_EQ(reg.owned_by(1).size(), 4u);
    CHECK(reg.find_any(control::make_identity(control::ObjectType::qp, control::identity_gen(b),
                                              control::identity_slot(b))) == nullptr);  // wrong type
}
