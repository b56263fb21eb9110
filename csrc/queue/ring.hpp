// Shared single-producer / single-consumer descriptor ring over a sealed memfd.
//
// Same header and slot layout as the reference ring (src/queue/shared_ring.cpp:158-270,
// :323-423); the implementation here is independent.  The producer and the consumer each keep
// a private cursor plus a cached copy of the other side's cursor, so the common case of a
// reserve or a peek touches no shared cache line; the shared cursor is re-read only when the
// cached view says "full" or "empty".  Publication is a release store, observation an acquire
// load, so a slot's bytes are visible before the cursor that covers them.
#pragma once

#include "common/shm.hpp"
#include "queue/layout.hpp"

#include <atomic>
#include <cstdint>

namespace ugdr::queue {

struct RingGeometry {
    RingKind kind = kSendRing;
    uint32_t capacity = 0;
    uint32_t stride = 0;
    bool operator==(const RingGeometry &o) const {
        return kind == o.kind && capacity == o.capacity && stride == o.stride;
    }
};

// Up to two contiguous slot runs (the second one after wrap-around).
struct SlotRun {
    uint8_t *first = nullptr;
    uint32_t first_count = 0;
    uint8_t *second = nullptr;
    uint32_t second_count = 0;
    uint32_t count() const { return first_count + second_count; }
};

class Ring {
  public:
    Ring() = default;
    Ring(Ring &&) noexcept = default;
    Ring &operator=(Ring &&) noexcept = default;
    Ring(const Ring &) = delete;
    Ring &operator=(const Ring &) = delete;

    // Bytes of a mapping for `g` (header + slots, page-rounded); 0 if invalid / overflow.
    static size_t mapping_bytes(const RingGeometry &g);
    static int create(const RingGeometry &g, Ring *out);
    // Map `fd` (ownership taken) and validate its header against `expected`.
    static int attach(int fd, const RingGeometry &expected, Ring *out);

    bool valid() const { return map_.address != nullptr; }
    const RingGeometry &geometry() const { return geom_; }
    RingHeader *header() const { return static_cast<RingHeader *>(map_.address); }
    uint8_t *slots() const { return static_cast<uint8_t *>(map_.address) + kRingHeaderBytes; }
    uint8_t *slot(uint64_t cursor) const {
        return slots() + uint64_t(cursor % geom_.capacity) * geom_.stride;
    }
    int fd() const { return map_.fd.get(); }
    void *mapping() const { return map_.address; }
    size_t bytes() const { return map_.bytes; }

    // Producer: claim up to `want` free slots (never more than are free).  Returns the run.
    SlotRun reserve(uint32_t want);
    // Producer: claim every slot that is free according to the consumer cursor seen last; the
    // shared cursor is re-read only when that shows none free, or when `refresh` is set.
    SlotRun reserve_free(bool refresh);
    // Producer: make `n` previously reserved slots visible to the consumer.
    void publish(uint32_t n);
    // Consumer: look at up to `want` published slots without consuming them.
    SlotRun peek(uint32_t want);
    // Consumer: hand `n` peeked slots back to the producer.
    void release(uint32_t n);

    // Shared cursors (acquire loads).
    uint64_t tail() const;
    uint64_t head() const;
    // Reload the private cursors from the shared ones (after another party moved them).
    void resync();

    // QP error word in the send-ring metadata (see layout.hpp).
    uint64_t error_word() const;
    void set_error_word(uint64_t v);

  private:
    SlotRun run_at(uint32_t index, uint32_t count) const;

    SharedMapping map_;
    RingGeometry geom_;
    uint64_t prod_tail_ = 0, prod_head_seen_ = 0;
    uint64_t cons_head_ = 0, cons_tail_seen_ = 0;
    // prod_tail_ % capacity and cons_head_ % capacity, kept up to date by publish / release so
    // the fast paths never divide (capacity need not be a power of two).
    uint32_t prod_index_ = 0, cons_index_ = 0;
    uint32_t reserved_ = 0, peeked_ = 0;
};

}  // namespace ugdr::queue
