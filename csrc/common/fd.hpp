// Owning file-descriptor handle and small POSIX helpers shared by every layer.
#pragma once

#include <cerrno>
#include <unistd.h>

namespace ugdr {

class Fd {
  public:
    Fd() noexcept = default;
    explicit Fd(int fd) noexcept : fd_(fd) {}
    ~Fd() { reset(); }
    Fd(const Fd &) = delete;
    Fd &operator=(const Fd &) = delete;
    Fd(Fd &&o) noexcept : fd_(o.release()) {}
    Fd &operator=(Fd &&o) noexcept {
        if (this != &o) reset(o.release());
        return *this;
    }
    int get() const noexcept { return fd_; }
    bool valid() const noexcept { return fd_ >= 0; }
    int release() noexcept {
        int f = fd_;
        fd_ = -1;
        return f;
    }
    void reset(int fd = -1) noexcept {
        if (fd_ >= 0) {
            while (::close(fd_) < 0 && errno == EINTR) {
            }
        }
        fd_ = fd;
    }

  private:
    int fd_ = -1;
};

}  // namespace ugdr
