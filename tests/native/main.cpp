#include "harness.hpp"

#include <cstring>

namespace th {
std::vector<Case> &registry() {
    static std::vector<Case> r;
    return r;
}
int g_failures = 0;
}  // namespace th

int main(int argc, char **argv) {
    if (argc == 2 && std::strcmp(argv[1], "--list") == 0) {
        for (const auto &c : th::registry()) std::printf("%s\n", c.name);
        return 0;
    }
    int failed_cases = 0, ran = 0;
    for (const auto &c : th::registry()) {
        bool selected = argc == 1;
        for (int i = 1; i < argc && !selected; ++i) selected = std::strcmp(argv[i], c.name) == 0;
        if (!selected) continue;
        const int before = th::g_failures;
        c.fn();
        ++ran;
        const bool ok = th::g_failures == before;
        std::printf("[%s] %s\n", ok ? " ok " : "FAIL", c.name);
        if (!ok) ++failed_cases;
    }
    if (ran == 0) {
        std::fprintf(stderr, "no test matched\n");
        return 2;
    }
    return failed_cases;
}
