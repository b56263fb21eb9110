// GPUDirect visibility gate decisions against a fake attribute / flush source (reference suite
// semantics: tests/unit/persistent_copy_backend_test.cpp FakeVisibilityGate - flush before
// publish, flush failure blocks the publish).
#include "harness.hpp"

#include "gpu/visibility.hpp"

#include <cerrno>

using ugdr::gpu::VisibilityAttrs;
using ugdr::gpu::VisibilityGate;

namespace {

struct FakeSource : ugdr::gpu::VisibilitySource {
    VisibilityAttrs attrs;
    int query_rc = 0, flush_rc = 0, flush_calls = 0, last_device = -1;
    int query(int device, VisibilityAttrs *out) override {
        last_device = device;
        if (query_rc) return query_rc;
        *out = attrs;
        return 0;
    }
    int flush(int device) override {
        last_device = device;
        ++flush_calls;
        return flush_rc;
    }
};

}  // namespace

TEST(visibility_owner_ordering_needs_no_flush) {
    FakeSource f;
    f.attrs = {true, 1, 100};
    VisibilityGate g(f);
    CHECK_EQ(g.init(3), 0);
    CHECK(g.mode() == VisibilityGate::Mode::kOrdered);
    for (int i = 0; i < 5; ++i) CHECK_EQ(g.before_publish(), 0);
    CHECK_EQ(f.flush_calls, 0);
    CHECK_EQ(f.last_device, 3);
}

TEST(visibility_unordered_flushes_before_every_publish) {
    FakeSource f;
    f.attrs = {true, 1, 0};
    VisibilityGate g(f);
    CHECK_EQ(g.init(1), 0);
    CHECK(g.mode() == VisibilityGate::Mode::kFlush);
    CHECK_EQ(g.before_publish(), 0);
    CHECK_EQ(g.before_publish(), 0);
    CHECK_EQ(f.flush_calls, 2);
    CHECK_EQ(int(g.flushes()), 2);
}

TEST(visibility_flush_failure_blocks_publish) {
    FakeSource f;
    f.attrs = {true, 1, 0};
    f.flush_rc = EIO;
    VisibilityGate g(f);
    CHECK_EQ(g.init(0), 0);
    CHECK_EQ(g.before_publish(), EIO);
    CHECK_EQ(int(g.flushes()), 0);
}

TEST(visibility_unavailable_without_rdma_or_flush) {
    FakeSource a;
    a.attrs = {false, 1, 200};
    VisibilityGate ga(a);
    CHECK_EQ(ga.init(0), 0);
    CHECK(ga.mode() == VisibilityGate::Mode::kUnavailable);
    CHECK_EQ(ga.before_publish(), EOPNOTSUPP);
    FakeSource b;
    b.attrs = {true, 0, 0};  // unordered and no host flush
    VisibilityGate gb(b);
    CHECK_EQ(gb.init(0), 0);
    CHECK_EQ(gb.before_publish(), EOPNOTSUPP);
    FakeSource c;
    c.query_rc = ENODEV;
    VisibilityGate gc(c);
    CHECK_EQ(gc.init(0), ENODEV);
    CHECK(gc.mode() == VisibilityGate::Mode::kUnavailable);
    CHECK_EQ(b.flush_calls + c.flush_calls, 0);
}
