#include "ipc/ipc.hpp"

#include "common/bytes.hpp"

#include <poll.h>
#include <fcntl.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/time.h>
#include <sys/un.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

namespace ugdr::ipc {

void encode_envelope(const Envelope &e, uint8_t out[kEnvelopeBytes]) {
    std::vector<std::byte> v;
    v.reserve(kEnvelopeBytes);
    ByteWriter w(&v);
    w.be(e.magic).be(e.major).be(e.minor).be(e.method).be(e.flags).be(e.request_id);
    w.be(uint32_t(e.status)).be(e.payload_length).be(e.fd_count);
    std::memcpy(out, v.data(), kEnvelopeBytes);
}

Envelope decode_envelope(const uint8_t in[kEnvelopeBytes]) {
    Envelope e;
    ByteReader r(reinterpret_cast<const std::byte *>(in), kEnvelopeBytes);
    uint32_t status = 0;
    r.be(&e.magic);
    r.be(&e.major);
    r.be(&e.minor);
    r.be(&e.method);
    r.be(&e.flags);
    r.be(&e.request_id);
    r.be(&status);
    r.be(&e.payload_length);
    r.be(&e.fd_count);
    e.status = int32_t(status);
    return e;
}

int send_message(int sock, const Message &m) {
    if (sock < 0 || m.payload.size() > kMaxPayload || m.fds.size() > kMaxFds) return EINVAL;
    for (const Fd &f : m.fds)
        if (!f.valid()) return EBADF;
    Envelope e = m.env;
    e.payload_length = uint32_t(m.payload.size());
    e.fd_count = uint32_t(m.fds.size());
    uint8_t head[kEnvelopeBytes];
    encode_envelope(e, head);

    iovec iov[2];
    iov[0] = {head, kEnvelopeBytes};
    iov[1] = {const_cast<std::byte *>(m.payload.data()), m.payload.size()};
    msghdr mh{};
    mh.msg_iov = iov;
    mh.msg_iovlen = m.payload.empty() ? 1 : 2;
    alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int) * kMaxFds)];
    if (!m.fds.empty()) {
        const size_t len = sizeof(int) * m.fds.size();
        std::memset(control, 0, sizeof(control));
        mh.msg_control = control;
        mh.msg_controllen = CMSG_SPACE(len);
        cmsghdr *c = CMSG_FIRSTHDR(&mh);
        c->cmsg_level = SOL_SOCKET;
        c->cmsg_type = SCM_RIGHTS;
        c->cmsg_len = CMSG_LEN(len);
        int *dst = reinterpret_cast<int *>(CMSG_DATA(c));
        for (size_t i = 0; i < m.fds.size(); ++i) dst[i] = m.fds[i].get();
    }
    for (;;) {
        const ssize_t n = ::sendmsg(sock, &mh, MSG_NOSIGNAL);
        if (n >= 0) return size_t(n) == kEnvelopeBytes + m.payload.size() ? 0 : EMSGSIZE;
        if (errno != EINTR) return errno;
    }
}

int recv_message(int sock, Message *m, bool nonblocking) {
    if (sock < 0 || m == nullptr) return EINVAL;
    // One receive buffer per thread, large enough for any datagram plus one byte (to detect an
    // oversized one), reused and never cleared: a fresh zero-filled MiB per message cost more
    // than the round trip itself.
    constexpr size_t kBufBytes = kEnvelopeBytes + kMaxPayload + 1;
    struct FreeBuf {
        void operator()(uint8_t *p) const noexcept { std::free(p); }
    };
    thread_local std::unique_ptr<uint8_t, FreeBuf> tls_buf;
    if (!tls_buf) tls_buf.reset(static_cast<uint8_t *>(std::malloc(kBufBytes)));
    if (!tls_buf) return ENOMEM;
    uint8_t *const buf = tls_buf.get();
    iovec iov{buf, kBufBytes};
    msghdr mh{};
    mh.msg_iov = &iov;
    mh.msg_iovlen = 1;
    alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int) * kMaxFds)];
    mh.msg_control = control;
    mh.msg_controllen = sizeof(control);
    ssize_t n;
    for (;;) {
        n = ::recvmsg(sock, &mh, MSG_CMSG_CLOEXEC | (nonblocking ? MSG_DONTWAIT : 0));
        if (n >= 0) break;
        if (errno != EINTR) return errno;
    }
    // Adopt any descriptors first so an error path never leaks them.
    std::vector<Fd> fds;
    for (cmsghdr *c = CMSG_FIRSTHDR(&mh); c != nullptr; c = CMSG_NXTHDR(&mh, c)) {
        if (c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) {
            const size_t count = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
            const int *src = reinterpret_cast<const int *>(CMSG_DATA(c));
            for (size_t i = 0; i < count; ++i) fds.emplace_back(src[i]);
        }
    }
    if (n == 0) return ECONNRESET;
    if ((mh.msg_flags & MSG_TRUNC) != 0) return EMSGSIZE;
    // A lost descriptor leaves the byte stream in step (one datagram per message), so the
    // message is still delivered, marked, for the receiver to refuse with EMFILE.
    const bool fds_truncated = (mh.msg_flags & MSG_CTRUNC) != 0;
    if (size_t(n) < kEnvelopeBytes) return EPROTO;
    const Envelope e = decode_envelope(buf);
    if (e.magic != kMagic || e.major != kVersionMajor || (e.flags & ~kFlagResponse) != 0 ||
        e.payload_length != size_t(n) - kEnvelopeBytes || e.payload_length > kMaxPayload ||
        (fds_truncated ? e.fd_count <= fds.size() || e.fd_count > kMaxFds : e.fd_count != fds.size())) {
        return EPROTO;
    }
    m->fds_truncated = fds_truncated;
    m->env = e;
    m->payload.assign(reinterpret_cast<std::byte *>(buf + kEnvelopeBytes), reinterpret_cast<std::byte *>(buf + n));
    m->fds = std::move(fds);
    return 0;
}

namespace {

int make_address(const std::string &path, sockaddr_un *addr) {
    if (path.empty() || path.size() >= sizeof(addr->sun_path)) return ENAMETOOLONG;
    std::memset(addr, 0, sizeof(*addr));
    addr->sun_family = AF_UNIX;
    std::memcpy(addr->sun_path, path.c_str(), path.size() + 1);
    return 0;
}

}  // namespace

namespace {

void set_recv_timeout(int sock, uint64_t ms) {
    timeval tv{};  // zero: no deadline
    tv.tv_sec = time_t(ms / 1000);
    tv.tv_usec = suseconds_t((ms % 1000) * 1000);
    ::setsockopt(sock, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
}

}  // namespace

int Client::connect(const std::string &path) {
    sockaddr_un addr;
    if (int rc = make_address(path, &addr); rc != 0) return rc;
    Fd s(::socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC, 0));
    if (!s.valid()) return errno;
    for (;;) {
        if (::connect(s.get(), reinterpret_cast<sockaddr *>(&addr), sizeof(addr)) == 0) break;
        if (errno != EINTR) return errno;
    }
    // A daemon that stops answering must not hang its clients: every reply has a deadline
    // (UGDR_RPC_TIMEOUT_MS, default 120 s, 0 = wait forever), after which the call fails with
    // ETIMEDOUT and the connection is closed.  The longest legitimate request (quiescing a GPU's
    // executor around a destroy) is bounded well below the default.
    uint64_t ms = 120000;
    if (const char *e = std::getenv("UGDR_RPC_TIMEOUT_MS"); e != nullptr && e[0] != '\0')
        ms = std::strtoull(e, nullptr, 10);
    set_recv_timeout(s.get(), ms);
    timeout_ms_ = ms;
    sock_ = std::move(s);
    return 0;
}

int Client::call(uint32_t method, std::vector<std::byte> payload, std::vector<Fd> fds, Message *resp,
                 uint64_t min_wait_ms) {
    if (!sock_.valid()) return ENOTCONN;
    if (resp == nullptr) return EINVAL;
    Message req;
    req.env.method = method;
    req.env.request_id = next_id_++;
    req.payload = std::move(payload);
    req.fds = std::move(fds);
    if (int rc = send_message(sock_.get(), req); rc != 0) {
        close();
        return rc;
    }
    // The daemon answers most requests within tens of microseconds: poll for the reply briefly
    // before sleeping in recvmsg, which saves the wake-up on the common path.
    Message r;
    int rc = EAGAIN;
    const auto spin_until = std::chrono::steady_clock::now() + std::chrono::microseconds(50);
    do {
        rc = recv_message(sock_.get(), &r, true);
    } while (rc == EAGAIN && std::chrono::steady_clock::now() < spin_until);
    const bool longer = timeout_ms_ != 0 && min_wait_ms > timeout_ms_;
    if (longer) set_recv_timeout(sock_.get(), min_wait_ms);
    if (rc == EAGAIN || rc == EWOULDBLOCK) rc = recv_message(sock_.get(), &r);
    if (longer) set_recv_timeout(sock_.get(), timeout_ms_);
    if (rc == EAGAIN || rc == EWOULDBLOCK) rc = ETIMEDOUT;  // SO_RCVTIMEO ran out
    if (rc != 0) {
        close();
        return rc;
    }
    if ((r.env.flags & kFlagResponse) == 0 || r.env.request_id != req.env.request_id ||
        r.env.method != method) {
        close();
        return EPROTO;
    }
    *resp = std::move(r);
    return 0;
}

int Server::start(const std::string &path) {
    if (listener_.valid()) return EALREADY;
    sockaddr_un addr;
    if (int rc = make_address(path, &addr); rc != 0) return rc;
    Fd s(::socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC | SOCK_NONBLOCK, 0));
    if (!s.valid()) return errno;
    if (::bind(s.get(), reinterpret_cast<sockaddr *>(&addr), sizeof(addr)) != 0) {
        if (errno != EADDRINUSE) return errno;
        // Replace only a stale socket: something that is a socket but refuses connections.
        struct stat st {};
        if (::lstat(path.c_str(), &st) != 0 || !S_ISSOCK(st.st_mode)) return EADDRINUSE;
        Fd probe(::socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC, 0));
        if (probe.valid() &&
            ::connect(probe.get(), reinterpret_cast<sockaddr *>(&addr), sizeof(addr)) == 0)
            return EADDRINUSE;
        ::unlink(path.c_str());
        if (::bind(s.get(), reinterpret_cast<sockaddr *>(&addr), sizeof(addr)) != 0) return errno;
    }
    if (::listen(s.get(), 64) != 0) {
        const int err = errno;
        ::unlink(path.c_str());
        return err;
    }
    struct stat st {};
    if (::stat(path.c_str(), &st) == 0) {
        sock_dev_ = st.st_dev;
        sock_ino_ = st.st_ino;
    }
    listener_ = std::move(s);
    reserve_ = Fd(::open("/dev/null", O_RDONLY | O_CLOEXEC));
    path_ = path;
    return 0;
}

void Server::drop(int fd) noexcept {
    auto it = sessions_.find(fd);
    if (it == sessions_.end()) return;
    const SessionId id = it->second.id;
    sessions_.erase(it);
    handler_.on_disconnect(id);
}

int Server::poll_once(int timeout_ms) {
    if (!listener_.valid()) return EBADF;
    std::vector<pollfd> pfds;
    pfds.reserve(sessions_.size() + 1);
    pfds.push_back({listener_.get(), POLLIN, 0});
    for (const auto &kv : sessions_) pfds.push_back({kv.first, POLLIN, 0});
    int n = ::poll(pfds.data(), pfds.size(), timeout_ms);
    if (n < 0) return errno == EINTR ? 0 : errno;
    if (n == 0) return 0;
    for (size_t i = 1; i < pfds.size(); ++i) {
        const int fd = pfds[i].fd;
        if (pfds[i].revents == 0) continue;
        if ((pfds[i].revents & POLLIN) != 0) {
            Message req;
            const int rc = recv_message(fd, &req);
            if (rc == EAGAIN || rc == EWOULDBLOCK) continue;  // nothing after all (sockets are non-blocking)
            if (rc != 0 || (req.env.flags & kFlagResponse) != 0) {
                drop(fd);
                continue;
            }
            auto it = sessions_.find(fd);
            if (it == sessions_.end()) continue;
            const uint32_t method = req.env.method;
            const uint64_t request_id = req.env.request_id;
            Message resp = handler_.handle(it->second.id, std::move(req));
            resp.env.method = method;
            resp.env.request_id = request_id;
            resp.env.flags = kFlagResponse;
            // Session sockets are non-blocking: a client whose unread replies fill its socket
            // buffer (EAGAIN) is dropped rather than allowed to stall every other client.
            if (send_message(fd, resp) != 0) drop(fd);
            last_served_ns_ = uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                           std::chrono::steady_clock::now().time_since_epoch())
                                           .count());
        } else {
            drop(fd);  // HUP / ERR without data
        }
    }
    if ((pfds[0].revents & POLLIN) != 0) {
        for (;;) {
            int c = ::accept4(listener_.get(), nullptr, nullptr, SOCK_CLOEXEC | SOCK_NONBLOCK);
            if (c < 0 && (errno == EMFILE || errno == ENFILE) && reserve_.valid()) {
                reserve_ = Fd();  // frees one descriptor
                const int refused = ::accept4(listener_.get(), nullptr, nullptr, SOCK_CLOEXEC);
                if (refused >= 0) ::close(refused);
                reserve_ = Fd(::open("/dev/null", O_RDONLY | O_CLOEXEC));
                if (refused >= 0) continue;
            }
            if (c < 0) break;
            sessions_.emplace(c, Session{Fd(c), next_session_++});
        }
    }
    return 0;
}

void Server::close() noexcept {
    std::vector<int> fds;
    for (const auto &kv : sessions_) fds.push_back(kv.first);
    for (int fd : fds) drop(fd);
    if (listener_.valid()) {
        listener_.reset();
        struct stat st {};
        if (!path_.empty() && ::stat(path_.c_str(), &st) == 0 && st.st_dev == sock_dev_ &&
            st.st_ino == sock_ino_)
            ::unlink(path_.c_str());
    }
}

}  // namespace ugdr::ipc
