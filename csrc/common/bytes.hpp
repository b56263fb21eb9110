// Big-endian byte writer / reader used by every control-plane codec.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

namespace ugdr {

class ByteWriter {
  public:
    explicit ByteWriter(std::vector<std::byte> *out) : out_(out) {}
    template <typename T> ByteWriter &be(T v) {
        uint8_t tmp[sizeof(T)];
        for (size_t i = 0; i < sizeof(T); ++i) tmp[i] = uint8_t(uint64_t(v) >> (8 * (sizeof(T) - 1 - i)));
        raw(tmp, sizeof(T));
        return *this;
    }
    ByteWriter &raw(const void *p, size_t n) {
        const auto *b = static_cast<const std::byte *>(p);
        out_->insert(out_->end(), b, b + n);
        return *this;
    }

  private:
    std::vector<std::byte> *out_;
};

class ByteReader {
  public:
    ByteReader(const std::byte *p, size_t n) : p_(p), n_(n) {}
    explicit ByteReader(const std::vector<std::byte> &v) : p_(v.data()), n_(v.size()) {}
    template <typename T> bool be(T *v) {
        if (n_ - off_ < sizeof(T)) return false;
        uint64_t acc = 0;
        for (size_t i = 0; i < sizeof(T); ++i) acc = (acc << 8) | uint8_t(p_[off_ + i]);
        *v = T(acc);
        off_ += sizeof(T);
        return true;
    }
    bool raw(void *dst, size_t n) {
        if (n_ - off_ < n) return false;
        if (n == 0) return true;  // an empty read: dst and p_ may be null
        std::memcpy(dst, p_ + off_, n);
        off_ += n;
        return true;
    }
    size_t remaining() const { return n_ - off_; }
    bool done() const { return off_ == n_; }

  private:
    const std::byte *p_;
    size_t n_;
    size_t off_ = 0;
};

}  // namespace ugdr
