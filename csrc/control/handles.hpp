// Typed generation handles for daemon objects.
//
// identity = type << 56 | generation << 24 | slot (the reference's encoding,
// src/control/object_identity.cpp:6-32, kept so identities read the same in traces).  A slot's
// generation advances on every reuse, so a stale identity never resolves to a newer object;
// a slot whose generation would wrap is retired for good.  Every object records the session that
// created it and only that session can name it.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <vector>

namespace ugdr::control {

enum class ObjectType : uint8_t { invalid = 0, context = 1, pd = 2, mr = 3, cq = 4, qp = 5 };

constexpr uint32_t kMaxSlot = 0x00ffffffu;

inline uint64_t make_identity(ObjectType t, uint32_t gen, uint32_t slot) {
    return (uint64_t(t) << 56) | (uint64_t(gen) << 24) | uint64_t(slot & kMaxSlot);
}
inline ObjectType identity_type(uint64_t id) { return ObjectType(id >> 56); }
inline uint32_t identity_gen(uint64_t id) { return uint32_t(id >> 24); }
inline uint32_t identity_slot(uint64_t id) { return uint32_t(id & kMaxSlot); }

template <typename T> class Registry {
  public:
    explicit Registry(ObjectType type, uint32_t max_slots = kMaxSlot + 1)
        : type_(type), max_slots_(max_slots) {}

    // Returns the new identity, or 0 when no slot is left.
    uint64_t insert(uint64_t owner, std::unique_ptr<T> obj) {
        uint32_t slot;
        if (!free_.empty()) {
            slot = free_.back();
            free_.pop_back();
        } else {
            if (slots_.size() >= max_slots_) return 0;
            slot = uint32_t(slots_.size());
            slots_.emplace_back();
        }
        Slot &s = slots_[slot];
        s.gen += 1;
        s.owner = owner;
        s.obj = std::move(obj);
        ++live_;
        return make_identity(type_, s.gen, slot);
    }

    // Resolve an identity owned by `owner`; nullptr for wrong type / stale / foreign.
    T *find(uint64_t owner, uint64_t id) const {
        Slot *s = lookup(id);
        return (s != nullptr && s->owner == owner) ? s->obj.get() : nullptr;
    }
    // Resolve without the ownership check (cross-session peers).
    T *find_any(uint64_t id) const {
        Slot *s = lookup(id);
        return s != nullptr ? s->obj.get() : nullptr;
    }
    uint64_t owner_of(uint64_t id) const {
        Slot *s = lookup(id);
        return s != nullptr ? s->owner : 0;
    }

    std::unique_ptr<T> erase(uint64_t id) {
        Slot *s = lookup(id);
        if (s == nullptr) return nullptr;
        std::unique_ptr<T> out = std::move(s->obj);
        const uint32_t slot = identity_slot(id);
        if (s->gen != 0xffffffffu) free_.push_back(slot);  // else retired forever
        --live_;
        return out;
    }

    // Visit every live object: fn(identity, owner, T&).
    void for_each(const std::function<void(uint64_t, uint64_t, T &)> &fn) const {
        for (uint32_t i = 0; i < slots_.size(); ++i) {
            const Slot &s = slots_[i];
            if (s.obj) fn(make_identity(type_, s.gen, i), s.owner, *s.obj);
        }
    }
    std::vector<uint64_t> owned_by(uint64_t owner) const {
        std::vector<uint64_t> ids;
        for (uint32_t i = 0; i < slots_.size(); ++i)
            if (slots_[i].obj && slots_[i].owner == owner)
                ids.push_back(make_identity(type_, slots_[i].gen, i));
        return ids;
    }
    size_t size() const { return live_; }
    bool full() const { return free_.empty() && slots_.size() >= max_slots_; }

  private:
    struct Slot {
        uint32_t gen = 0;
        uint64_t owner = 0;
        std::unique_ptr<T> obj;
    };
    Slot *lookup(uint64_t id) const {
        if (identity_type(id) != type_) return nullptr;
        const uint32_t slot = identity_slot(id);
        if (slot >= slots_.size()) return nullptr;
        Slot &s = const_cast<Slot &>(slots_[slot]);
        if (!s.obj || s.gen != identity_gen(id)) return nullptr;
        return &s;
    }

    ObjectType type_;
    uint32_t max_slots_;
    std::vector<Slot> slots_;
    std::vector<uint32_t> free_;
    size_t live_ = 0;
};

}  // namespace ugdr::control
