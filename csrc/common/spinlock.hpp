// Test-and-test-and-set spin lock for the short critical sections of the posting and polling
// paths (a few slot copies and one cursor store): uncontended it costs one atomic exchange and
// one store, about a third of a pthread mutex.  Under contention it pauses, then yields.
// Satisfies Lockable, so std::lock_guard works with it.
#pragma once

#include <atomic>
#include <thread>

#if defined(__x86_64__) || defined(__i386__)
#include <immintrin.h>
#endif

namespace ugdr {

class SpinLock {
  public:
    void lock() noexcept {
        for (uint32_t spins = 0;; ++spins) {
            if (!locked_.exchange(true, std::memory_order_acquire)) return;
            while (locked_.load(std::memory_order_relaxed)) {
                if (++spins < 64) {
                    relax();
                } else {
                    std::this_thread::yield();
                }
            }
        }
    }
    bool try_lock() noexcept {
        return !locked_.load(std::memory_order_relaxed) && !locked_.exchange(true, std::memory_order_acquire);
    }
    void unlock() noexcept { locked_.store(false, std::memory_order_release); }

  private:
    static void relax() noexcept {
#if defined(__x86_64__) || defined(__i386__)
        _mm_pause();
#endif
    }
    std::atomic<bool> locked_{false};
};

}  // namespace ugdr
