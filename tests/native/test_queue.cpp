// Shared ring tests (reference suite semantics: tests/unit/shared_ring_test.cpp — capacity 1,
// non-power-of-two capacities, wrap, two-span batches, threaded producer/consumer, two
// mappings, malformed header rejection).
#include "harness.hpp"

#include "queue/ring.hpp"

#include <unistd.h>

#include <atomic>
#include <cstring>
#include <thread>

using namespace ugdr::queue;

namespace {

Ring make(uint32_t cap, uint32_t stride = 64, RingKind kind = kSendRing) {
    Ring r;
    CHECK_EQ(Ring::create({kind, cap, stride}, &r), 0);
    return r;
}

Ring attach_dup(const Ring &r) {
    Ring other;
    CHECK_EQ(Ring::attach(::dup(r.fd()), r.geometry(), &other), 0);
    return other;
}

}  // namespace

TEST(ring_header_layout) {
    Ring r = make(5, 128);
    const RingHeader *h = r.header();
    CHECK_EQ(h->meta.magic, kRingMagic);
    CHECK_EQ(h->meta.version, kRingVersion);
    CHECK_EQ(h->meta.kind, uint16_t(kSendRing));
    CHECK_EQ(h->meta.header_bytes, 192u);
    CHECK_EQ(h->meta.capacity, 5u);
    CHECK_EQ(h->meta.slot_stride, 128u);
    CHECK_EQ(h->meta.mapping_bytes, uint64_t(r.bytes()));
    CHECK_EQ(r.bytes() % 4096, 0u);
    CHECK_EQ(r.slot(0) - reinterpret_cast<uint8_t *>(r.mapping()), 192);
}

TEST(ring_capacity_one) {
    Ring p = make(1);
    Ring c = attach_dup(p);
    for (int i = 0; i < 10; ++i) {
        SlotRun run = p.reserve(3);
        CHECK_EQ(run.count(), 1u);
        std::memcpy(run.first, &i, sizeof(i));
        p.publish(1);
        CHECK_EQ(p.reserve(1).count(), 0u);  // full
        SlotRun got = c.peek(4);
        CHECK_EQ(got.count(), 1u);
        int v = -1;
        std::memcpy(&v, got.first, sizeof(v));
        CHECK_EQ(v, i);
        c.release(1);
    }
}

TEST(ring_non_power_of_two_wrap_two_spans) {
    Ring p = make(7);
    Ring c = attach_dup(p);
    uint64_t produced = 0, consumed = 0;
    for (int round = 0; round < 50; ++round) {
        const uint32_t want = 1 + (round * 3) % 7;
        SlotRun run = p.reserve(want);
        for (uint32_t i = 0; i < run.count(); ++i) {
            uint8_t *s = i < run.first_count ? run.first + i * 64 : run.second + (i - run.first_count) * 64;
            const uint64_t v = produced + i;
            std::memcpy(s, &v, 8);
        }
        if (run.second_count > 0) CHECK(run.second == p.slot(0));
        p.publish(run.count());
        produced += run.count();
        SlotRun got = c.peek(5);
        for (uint32_t i = 0; i < got.count(); ++i) {
            const uint8_t *s = i < got.first_count ? got.first + i * 64 : got.second + (i - got.first_count) * 64;
            uint64_t v = 0;
            std::memcpy(&v, s, 8);
            CHECK_EQ(v, consumed + i);
        }
        c.release(got.count());
        consumed += got.count();
    }
    CHECK(produced > 100);
    CHECK_EQ(p.tail(), produced);
    CHECK_EQ(c.head(), consumed);
}

TEST(ring_threaded_producer_consumer) {
    Ring p = make(13);
    Ring c = attach_dup(p);
    constexpr uint64_t kN = 200000;
    std::thread prod([&] {
        uint64_t next = 0;
        while (next < kN) {
            SlotRun run = p.reserve(8);
            const uint32_t n = uint32_t(std::min<uint64_t>(run.count(), kN - next));
            for (uint32_t i = 0; i < n; ++i) {
                uint8_t *s = i < run.first_count ? run.first + i * 64 : run.second + (i - run.first_count) * 64;
                const uint64_t v = next + i;
                std::memcpy(s, &v, 8);
            }
            p.publish(n);
            next += n;
        }
    });
    uint64_t seen = 0;
    bool in_order = true;
    while (seen < kN) {
        SlotRun got = c.peek(16);
        for (uint32_t i = 0; i < got.count(); ++i) {
            const uint8_t *s = i < got.first_count ? got.first + i * 64 : got.second + (i - got.first_count) * 64;
            uint64_t v = 0;
            std::memcpy(&v, s, 8);
            in_order &= v == seen + i;
        }
        c.release(got.count());
        seen += got.count();
    }
    prod.join();
    CHECK(in_order);
    CHECK_EQ(seen, kN);
}

TEST(ring_attach_rejects_mismatch) {
    Ring r = make(8, 128, kRecvRing);
    Ring x;
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kSendRing, 8, 128}, &x), EPROTO);     // kind
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kRecvRing, 16, 128}, &x), EPROTO);    // size differs
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kRecvRing, 8, 96}, &x), EINVAL);      // stride % 64
    r.header()->meta.magic = 0x12345678;
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kRecvRing, 8, 128}, &x), EPROTO);     // magic
    r.header()->meta.magic = kRingMagic;
    r.header()->tail.value = 100;  // tail - head > capacity
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kRecvRing, 8, 128}, &x), EPROTO);
    r.header()->tail.value = 0;
    CHECK_EQ(Ring::attach(::dup(r.fd()), {kRecvRing, 8, 128}, &x), 0);
}

TEST(ring_geometry_validation) {
    Ring r;
    CHECK_EQ(Ring::create({kSendRing, 0, 64}, &r), EINVAL);
    CHECK_EQ(Ring::create({kSendRing, 4, 0}, &r), EINVAL);
    CHECK_EQ(Ring::create({RingKind(9), 4, 64}, &r), EINVAL);
    CHECK_EQ(send_stride(1), 64u);   // 40 + 16 = 56 -> 64
    CHECK_EQ(send_stride(2), 128u);  // 72 -> 128
    CHECK_EQ(send_stride(16), 320u); // 296 -> 320
    CHECK_EQ(recv_stride(1), 64u);
    CHECK_EQ(recv_stride(4), 128u);  // 80 -> 128
    CHECK_EQ(completion_stride(), 64u);
}

TEST(ring_memfd_is_sealed) {
    Ring r = make(4);
    CHECK(::ftruncate(r.fd(), 1 << 20) != 0);  // grow sealed
    CHECK(::ftruncate(r.fd(), 0) != 0);        // shrink sealed
}

TEST(ring_error_word_roundtrip) {
    Ring r = make(4);
    Ring c = attach_dup(r);
    CHECK_EQ(c.error_word(), 0u);
    r.set_error_word(6);
    CHECK_EQ(c.error_word(), 6u);
}
