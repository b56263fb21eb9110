// ugdr_client: list the daemon's devices (smoke check of the public API).
#include "ugdr/api.hpp"

#include <cerrno>
#include <cstdio>
#include <cstring>

int main() {
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (list == nullptr) {
        std::fprintf(stderr, "ugdr_client: no daemon: %s\n", std::strerror(errno));
        return 1;
    }
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0)
            std::printf("%s kind=%s gpu=%d\n", info.name, info.kind == 1 ? "gpu" : "cpu",
                        info.gpu_ordinal);
    }
    ugdr_free_device_list(list);
    return 0;
}
