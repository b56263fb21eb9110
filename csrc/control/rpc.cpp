#include "control/rpc.hpp"

#include "common/bytes.hpp"

#include <cerrno>

namespace ugdr::control {
namespace {

void put_indices(ByteWriter &w, size_t n) {
    for (size_t i = 0; i < n; ++i) w.be(uint32_t(i));
}

// Reorder descriptors according to the wire's index list.
bool take_indices(ByteReader &r, uint32_t count, std::vector<Fd> *fds) {
    if (count != fds->size()) return false;
    std::vector<Fd> ordered(count);
    std::vector<bool> used(count, false);
    for (uint32_t i = 0; i < count; ++i) {
        uint32_t idx = 0;
        if (!r.be(&idx) || idx >= count || used[idx]) return false;
        used[idx] = true;
        ordered[i] = std::move((*fds)[idx]);
    }
    *fds = std::move(ordered);
    return true;
}

}  // namespace

int encode_request(Request &&req, ipc::Message *out) {
    if (out == nullptr || req.method == 0 || req.fds.size() > ipc::kMaxFds) return EINVAL;
    if (req.opaque.size() + kRequestPrefix + 4 * req.fds.size() > ipc::kMaxPayload) return EMSGSIZE;
    ipc::Message m;
    m.env.method = req.method;
    ByteWriter w(&m.payload);
    w.be(kPayloadVersion).be(uint16_t(0)).be(req.identity).be(req.length).be(req.access);
    w.be(uint32_t(req.opaque.size())).be(uint32_t(req.fds.size()));
    w.raw(req.opaque.data(), req.opaque.size());
    put_indices(w, req.fds.size());
    m.fds = std::move(req.fds);
    *out = std::move(m);
    return 0;
}

int decode_request(ipc::Message &&msg, Request *out) {
    if (out == nullptr || msg.env.method == 0) return EINVAL;
    ByteReader r(msg.payload);
    uint16_t version = 0, reserved = 0;
    uint32_t opaque_len = 0, count = 0;
    Request req;
    req.method = msg.env.method;
    if (!r.be(&version) || !r.be(&reserved) || !r.be(&req.identity) || !r.be(&req.length) ||
        !r.be(&req.access) || !r.be(&opaque_len) || !r.be(&count))
        return EPROTO;
    if (version != kPayloadVersion || reserved != 0) return EPROTONOSUPPORT;
    if (opaque_len > r.remaining() || r.remaining() - opaque_len != size_t(count) * 4) return EPROTO;
    req.opaque.resize(opaque_len);
    r.raw(req.opaque.data(), opaque_len);
    req.fds = std::move(msg.fds);
    if (!take_indices(r, count, &req.fds)) return EPROTO;
    *out = std::move(req);
    return 0;
}

int encode_response(uint32_t method, Response &&resp, ipc::Message *out) {
    if (out == nullptr || method == 0 || resp.fds.size() > ipc::kMaxFds) return EINVAL;
    if (resp.opaque.size() + kResponsePrefix + 4 * resp.fds.size() > ipc::kMaxPayload)
        return EMSGSIZE;
    ipc::Message m;
    m.env.method = method;
    m.env.flags = ipc::kFlagResponse;
    m.env.status = resp.status;
    ByteWriter w(&m.payload);
    w.be(kPayloadVersion).be(uint16_t(0)).be(resp.identity);
    w.be(uint32_t(resp.opaque.size())).be(uint32_t(resp.fds.size()));
    w.raw(resp.opaque.data(), resp.opaque.size());
    put_indices(w, resp.fds.size());
    m.fds = std::move(resp.fds);
    *out = std::move(m);
    return 0;
}

int decode_response(ipc::Message &&msg, Response *out) {
    if (out == nullptr || (msg.env.flags & ipc::kFlagResponse) == 0) return EINVAL;
    ByteReader r(msg.payload);
    uint16_t version = 0, reserved = 0;
    uint32_t opaque_len = 0, count = 0;
    Response resp;
    resp.status = msg.env.status;
    if (!r.be(&version) || !r.be(&reserved) || !r.be(&resp.identity) || !r.be(&opaque_len) ||
        !r.be(&count))
        return EPROTO;
    if (version != kPayloadVersion || reserved != 0) return EPROTONOSUPPORT;
    if (opaque_len > r.remaining() || r.remaining() - opaque_len != size_t(count) * 4) return EPROTO;
    resp.opaque.resize(opaque_len);
    r.raw(resp.opaque.data(), opaque_len);
    resp.fds = std::move(msg.fds);
    if (!take_indices(r, count, &resp.fds)) return EPROTO;
    *out = std::move(resp);
    return 0;
}

}  // namespace ugdr::control
