// Minimal native test harness: TEST(name) registers a case; CHECK / CHECK_EQ record failures.
// `ugdr_native_tests --list` prints case names; `ugdr_native_tests NAME...` runs them
// (all when none given).  Exit status is the number of failed cases.
#pragma once

#include <cstdio>
#include <functional>
#include <string>
#include <vector>

namespace th {

struct Case {
    const char *name;
    std::function<void()> fn;
};
std::vector<Case> &registry();
extern int g_failures;

struct Registrar {
    Registrar(const char *name, std::function<void()> fn) { registry().push_back({name, std::move(fn)}); }
};

}  // namespace th

#define TH_CAT2(a, b) a##b
#define TH_CAT(a, b) TH_CAT2(a, b)
#define TEST(name)                                                                  \
    static void name();                                                             \
    static th::Registrar TH_CAT(reg_, name)(#name, name);                           \
    static void name()

#define CHECK(cond)                                                                 \
    do {                                                                            \
        if (!(cond)) {                                                              \
            std::fprintf(stderr, "  %s:%d: CHECK(%s) failed\n", __FILE__, __LINE__, #cond); \
            ++th::g_failures;                                                       \
        }                                                                           \
    } while (0)

#define CHECK_EQ(a, b)                                                              \
    do {                                                                            \
        const auto _va = (a);                                                       \
        const auto _vb = (b);                                                       \
        if (!(_va == _vb)) {                                                        \
            std::fprintf(stderr, "  %s:%d: CHECK_EQ(%s, %s) failed: %lld vs %lld\n", __FILE__, \
                         __LINE__, #a, #b, (long long)_va, (long long)_vb);        \
            ++th::g_failures;                                                       \
        }                                                                           \
    } while (0)
