// ugdr_daemon: serve the ugdr control plane and execute posted work on the host and the GPUs.
#include "daemon/daemon.hpp"

#include <sys/resource.h>

#include <atomic>
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace {
std::atomic<bool> g_stop{false};
extern "C" void on_signal(int) { g_stop.store(true); }

void usage(FILE *f) {
    std::fprintf(f,
                 "usage: ugdr_daemon [--socket PATH] [--gpus N] [--no-cpu-device] [--ctas N]\n"
                 "                   [--idle-exit-us N] [--bulk-min BYTES]\n"
                 "  --bulk-min: chunk pieces of at least BYTES (16-byte aligned) are copied by the\n"
                 "    TMA bulk-copy engine (default 8192, 0 = never; also $UGDR_EXECUTOR_BULK_MIN)\n"
                 "  PATH defaults to $UGDR_DAEMON_SOCKET, then /run/ugdr/ugdr.sock\n");
}
}  // namespace

int main(int argc, char **argv) {
    // Every CQ holds one ring descriptor, every QP two, every host MR one: lift the soft
    // descriptor limit to the hard one so thousands of QPs fit.
    if (rlimit rl{}; ::getrlimit(RLIMIT_NOFILE, &rl) == 0 && rl.rlim_cur < rl.rlim_max) {
        rl.rlim_cur = rl.rlim_max;
        ::setrlimit(RLIMIT_NOFILE, &rl);
    }
    ugdr::daemon::Options opt;
    const char *env = std::getenv("UGDR_DAEMON_SOCKET");
    opt.socket_path = (env != nullptr && env[0] != '\0') ? env : "/run/ugdr/ugdr.sock";
    if (const char *b = std::getenv("UGDR_EXECUTOR_BULK_MIN"); b != nullptr && b[0] != '\0')
        opt.bulk_min_bytes = std::atoi(b);
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&]() -> const char * {
            if (i + 1 >= argc) {
                usage(stderr);
                std::exit(2);
            }
            return argv[++i];
        };
        if (a == "--help") {
            usage(stdout);
            return 0;
        } else if (a == "--socket") {
            opt.socket_path = next();
        } else if (a == "--gpus") {
            opt.gpus = std::atoi(next());
        } else if (a == "--no-cpu-device") {
            opt.cpu_device = false;
        } else if (a == "--ctas") {
            opt.executor_ctas = std::atoi(next());
        } else if (a == "--bulk-min") {
            opt.bulk_min_bytes = std::atoi(next());
        } else if (a == "--idle-exit-us") {
            opt.idle_exit_us = uint32_t(std::strtoul(next(), nullptr, 10));
        } else {
            usage(stderr);
            return 2;
        }
    }
    std::signal(SIGINT, on_signal);
    std::signal(SIGTERM, on_signal);
    std::signal(SIGPIPE, SIG_IGN);
    ugdr::daemon::Daemon d(opt);
    if (int rc = d.start(); rc != 0) {
        std::fprintf(stderr, "ugdr_daemon: start failed: %s\n", std::strerror(rc));
        return 1;
    }
    std::fprintf(stderr, "ugdr_daemon: serving %zu device(s) on %s\n", d.device_count(),
                 opt.socket_path.c_str());
    const int rc = d.run(g_stop);
    return rc == 0 ? 0 : 1;
}
