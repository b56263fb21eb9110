#include "control/client.hpp"

#include <cerrno>

namespace ugdr::control {

int ControlClient::connect(const std::string &path) {
    ipc_.close();
    const int rc = ipc_.connect(path);
    if (rc == 0) epoch_ += 1;
    return rc;
}

void ControlClient::close() { ipc_.close(); }

int ControlClient::call(Request &&req, Response *resp) {
    if (!ipc_.connected()) return ENOTCONN;
    ipc::Message msg;
    const uint32_t method = req.method;
    if (int rc = encode_request(std::move(req), &msg); rc != 0) return rc;
    ipc::Message reply;
    if (int rc = ipc_.call(method, std::move(msg.payload), std::move(msg.fds), &reply); rc != 0)
        return rc;
    // This process is at its descriptor limit: the reply's rings or regions were lost.  The
    // connection is still in step; the call fails with EMFILE.
    if (reply.fds_truncated) return EMFILE;
    if (int rc = decode_response(std::move(reply), resp); rc != 0) {
        ipc_.close();
        return rc;
    }
    return 0;
}

}  // namespace ugdr::control
