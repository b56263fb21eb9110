#include "queue/ring.hpp"

#include <algorithm>
#include <cerrno>
#include <cstring>

namespace ugdr::queue {
namespace {

std::atomic_ref<uint64_t> cursor_ref(uint64_t &v) { return std::atomic_ref<uint64_t>(v); }

bool geometry_ok(const RingGeometry &g) {
    if (g.kind < kSendRing || g.kind > kCompletionRing) return false;
    if (g.capacity == 0 || g.stride == 0 || g.stride % kSlotAlign != 0) return false;
    if (g.kind == kCompletionRing && g.stride < sizeof(Cqe)) return false;
    return true;
}

}  // namespace

size_t Ring::mapping_bytes(const RingGeometry &g) {
    if (!geometry_ok(g)) return 0;
    const uint64_t slots = uint64_t(g.capacity) * g.stride;
    if (slots > (uint64_t(1) << 40)) return 0;
    return round_up_pages(size_t(kRingHeaderBytes + slots));
}

int Ring::create(const RingGeometry &g, Ring *out) {
    if (out == nullptr) return EINVAL;
    const size_t bytes = mapping_bytes(g);
    if (bytes == 0) return geometry_ok(g) ? EOVERFLOW : EINVAL;
    Ring r;
    if (int rc = create_shared_mapping("ugdr-ring", bytes, &r.map_); rc != 0) return rc;
    RingHeader *h = r.header();
    std::memset(h, 0, sizeof(RingHeader));
    h->meta.magic = kRingMagic;
    h->meta.version = kRingVersion;
    h->meta.kind = g.kind;
    h->meta.header_bytes = kRingHeaderBytes;
    h->meta.mapping_bytes = r.map_.bytes;
    h->meta.capacity = g.capacity;
    h->meta.slot_stride = g.stride;
    std::atomic_thread_fence(std::memory_order_release);
    r.geom_ = g;
    *out = std::move(r);
    return 0;
}

int Ring::attach(int fd, const RingGeometry &expected, Ring *out) {
    if (out == nullptr || fd < 0) {
        Fd close_it(fd);
        return EINVAL;
    }
    const size_t bytes = mapping_bytes(expected);
    if (bytes == 0) {
        Fd close_it(fd);
        return EINVAL;
    }
    Ring r;
    if (int rc = map_shared_fd(fd, bytes, &r.map_); rc != 0) return rc;
    const RingHeader *h = r.header();
    if (h->meta.magic != kRingMagic || h->meta.version != kRingVersion ||
        h->meta.kind != expected.kind || h->meta.header_bytes != kRingHeaderBytes ||
        h->meta.mapping_bytes != bytes || h->meta.capacity != expected.capacity ||
        h->meta.slot_stride != expected.stride) {
        return EPROTO;
    }
    r.geom_ = expected;
    r.resync();
    if (r.prod_tail_ - r.cons_head_ > expected.capacity) return EPROTO;
    *out = std::move(r);
    return 0;
}

uint64_t Ring::tail() const { return cursor_ref(header()->tail.value).load(std::memory_order_acquire); }
uint64_t Ring::head() const { return cursor_ref(header()->head.value).load(std::memory_order_acquire); }

void Ring::resync() {
    prod_tail_ = cons_tail_seen_ = tail();
    cons_head_ = prod_head_seen_ = head();
    prod_index_ = uint32_t(prod_tail_ % geom_.capacity);
    cons_index_ = uint32_t(cons_head_ % geom_.capacity);
    reserved_ = peeked_ = 0;
}

SlotRun Ring::run_at(uint32_t index, uint32_t count) const {
    SlotRun run;
    if (count == 0) return run;
    const uint32_t first = std::min(count, geom_.capacity - index);
    run.first = slots() + uint64_t(index) * geom_.stride;
    run.first_count = first;
    if (first < count) {
        run.second = slots();
        run.second_count = count - first;
    }
    return run;
}

SlotRun Ring::reserve(uint32_t want) {
    uint64_t used = prod_tail_ - prod_head_seen_;
    if (geom_.capacity - used < want) {
        prod_head_seen_ = head();
        used = prod_tail_ - prod_head_seen_;
    }
    const uint32_t n = uint32_t(std::min<uint64_t>(want, geom_.capacity - used));
    reserved_ = n;
    return run_at(prod_index_, n);
}

SlotRun Ring::reserve_free(bool refresh) {
    uint64_t used = prod_tail_ - prod_head_seen_;
    if (refresh || used >= geom_.capacity) {
        prod_head_seen_ = head();
        used = prod_tail_ - prod_head_seen_;
    }
    const uint32_t n = used >= geom_.capacity ? 0u : uint32_t(geom_.capacity - used);
    reserved_ = n;
    return run_at(prod_index_, n);
}

void Ring::publish(uint32_t n) {
    n = std::min(n, reserved_);
    reserved_ = 0;
    if (n == 0) return;
    prod_tail_ += n;
    prod_index_ += n;
    if (prod_index_ >= geom_.capacity) prod_index_ -= geom_.capacity;
    cursor_ref(header()->tail.value).store(prod_tail_, std::memory_order_release);
}

SlotRun Ring::peek(uint32_t want) {
    uint64_t avail = cons_tail_seen_ - cons_head_;
    if (avail < want) {
        cons_tail_seen_ = tail();
        avail = cons_tail_seen_ - cons_head_;
        if (avail > geom_.capacity) avail = 0;  // corrupt producer cursor: see nothing
    }
    const uint32_t n = uint32_t(std::min<uint64_t>(want, avail));
    peeked_ = n;
    return run_at(cons_index_, n);
}

void Ring::release(uint32_t n) {
    n = std::min(n, peeked_);
    peeked_ = 0;
    if (n == 0) return;
    cons_head_ += n;
    cons_index_ += n;
    if (cons_index_ >= geom_.capacity) cons_index_ -= geom_.capacity;
    cursor_ref(header()->head.value).store(cons_head_, std::memory_order_release);
}

uint64_t Ring::error_word() const {
    return cursor_ref(header()->meta.reserved[kQpErrorWordIndex]).load(std::memory_order_acquire);
}

void Ring::set_error_word(uint64_t v) {
    cursor_ref(header()->meta.reserved[kQpErrorWordIndex]).store(v, std::memory_order_release);
}

}  // namespace ugdr::queue
