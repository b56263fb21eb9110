#include "control/client.hpp"

#include "common/bytes.hpp"

#include <cerrno>

namespace ugdr::control {

int ControlClient::connect(const std::string &path) {
    ipc_.close();
    const int rc = ipc_.connect(path);
    if (rc == 0) epoch_ += 1;
    return rc;
}

void ControlClient::close() { ipc_.close(); }

int ControlClient::call(Request &&req, Response *resp, uint64_t min_wait_ms) {
    if (!ipc_.connected()) return ENOTCONN;
    ipc::Message msg;
    const uint32_t method = req.method;
    if (int rc = encode_request(std::move(req), &msg); rc != 0) return rc;
    ipc::Message reply;
    if (int rc = ipc_.call(method, std::move(msg.payload), std::move(msg.fds), &reply, min_wait_ms); rc != 0)
        return rc;
    // This process is at its descriptor limit: the reply's rings were lost.  The connection is
    // still in step; the call fails with EMFILE, and an object the daemon created for it (a CQ
    // or QP whose rings never arrived) is destroyed again rather than left to the session's end.
    if (reply.fds_truncated) {
        const uint32_t destroy = method == kCreateCq   ? uint32_t(kDestroyCq)
                                 : method == kCreateQp ? uint32_t(kDestroyQp)
                                                       : 0u;
        ByteReader rd(reply.payload);
        uint16_t version = 0, reserved = 0;
        uint64_t identity = 0;
        if (destroy != 0 && reply.env.status == 0 && rd.be(&version) && rd.be(&reserved) && rd.be(&identity) &&
            identity != 0) {
            Request undo;
            undo.method = destroy;
            undo.identity = identity;
            Response ignored;
            (void)call(std::move(undo), &ignored);
        }
        return EMFILE;
    }
    if (int rc = decode_response(std::move(reply), resp); rc != 0) {
        ipc_.close();
        return rc;
    }
    return 0;
}

}  // namespace ugdr::control
