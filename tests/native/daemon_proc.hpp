// Starts the real ugdr_daemon (next to the test binary, or $UGDR_DAEMON_BIN) on a private
// socket with the host-memory device only, for native tests of the public API.
#pragma once

#include <signal.h>
#include <sys/prctl.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>

namespace th {

inline std::string daemon_binary() {
    if (const char *e = std::getenv("UGDR_DAEMON_BIN"); e != nullptr && e[0] != '\0') return e;
    char self[4096];
    const ssize_t n = readlink("/proc/self/exe", self, sizeof(self) - 1);
    if (n <= 0) return {};
    self[n] = '\0';
    std::string dir(self);
    dir.resize(dir.rfind('/'));
    return dir + "/ugdr_daemon";
}

inline bool socket_ready(const std::string &path) {
    const int fd = ::socket(AF_UNIX, SOCK_SEQPACKET | SOCK_CLOEXEC, 0);
    if (fd < 0) return false;
    sockaddr_un a{};
    a.sun_family = AF_UNIX;
    std::strncpy(a.sun_path, path.c_str(), sizeof(a.sun_path) - 1);
    const bool ok = ::connect(fd, reinterpret_cast<sockaddr *>(&a), sizeof(a)) == 0;
    ::close(fd);
    return ok;
}

struct DaemonProc {
    pid_t pid = -1;
    std::string dir, sock;
    bool start() {
        const std::string bin = daemon_binary();
        struct stat st{};
        if (bin.empty() || ::stat(bin.c_str(), &st) != 0) return false;
        char tmpl[] = "/tmp/ugdr-alloc-XXXXXX";
        if (::mkdtemp(tmpl) == nullptr) return false;
        dir = tmpl;
        sock = dir + "/ugdr.sock";
        pid = ::fork();
        if (pid == 0) {
            ::prctl(PR_SET_PDEATHSIG, SIGTERM);  // never outlive a test binary that aborted
            ::execl(bin.c_str(), bin.c_str(), "--socket", sock.c_str(), "--gpus", "0", static_cast<char *>(nullptr));
            ::_exit(127);
        }
        for (int i = 0; i < 500 && pid > 0; ++i) {
            if (socket_ready(sock)) return true;
            std::this_thread::sleep_for(std::chrono::milliseconds(10));
        }
        return false;
    }
    ~DaemonProc() {
        if (pid > 0) {
            ::kill(pid, SIGTERM);
            int status = 0;
            for (int i = 0; i < 300 && ::waitpid(pid, &status, WNOHANG) == 0; ++i)
                std::this_thread::sleep_for(std::chrono::milliseconds(10));
            if (::waitpid(pid, &status, WNOHANG) == 0) {
                ::kill(pid, SIGKILL);
                ::waitpid(pid, &status, 0);
            }
        }
        if (!sock.empty()) ::unlink(sock.c_str());
        if (!dir.empty()) ::rmdir(dir.c_str());
    }
};

}  // namespace th
