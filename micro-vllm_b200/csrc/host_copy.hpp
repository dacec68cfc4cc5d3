// host_copy.hpp -- large host copies split over a few persistent threads.
//
// The host-pointer entries stage the caller's activation rows into pinned
// memory and the results back out (about a megabyte each way at config[1]'s
// batch 32; 8 MB for moe_block's f32 rows).  A single thread copies at about
// 10 GB/s, which puts tens to hundreds of microseconds on every call; three
// helper threads plus the caller cut that by about four.
//
// The helpers are created on first use and never destroyed (they wait on a
// condition variable until the process exits).  A process forked after they
// exist has none, so it copies on its own thread.
#pragma once

#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace mvb {

class HostCopier {
  public:
    static HostCopier &get() {
        static HostCopier *h = new HostCopier(); // never destroyed: helpers may be waiting
        return *h;
    }

    // memcpy(dst, src, n), in parallel above kMinBytes.
    void copy(void *dst, const void *src, size_t n) {
        if (n < kMinBytes || helpers_ == 0 || getpid() != pid_) {
            std::memcpy(dst, src, n);
            return;
        }
        std::lock_guard<std::mutex> one(call_mu_); // one parallel copy at a time
        const size_t parts = static_cast<size_t>(helpers_) + 1;
        {
            std::lock_guard<std::mutex> lk(mu_);
            dst_ = static_cast<uint8_t *>(dst);
            src_ = static_cast<const uint8_t *>(src);
            n_ = n;
            chunk_ = ((n + parts - 1) / parts + 63) & ~size_t(63);
            pending_.store(helpers_, std::memory_order_relaxed);
            ++gen_;
        }
        cv_.notify_all();
        part(static_cast<size_t>(helpers_)); // the caller takes the last part
        for (int spin = 0; pending_.load(std::memory_order_acquire) != 0; ++spin)
            if (spin > 64)
                std::this_thread::yield();
    }

  private:
    static constexpr size_t kMinBytes = 256 * 1024;

    HostCopier() : pid_(getpid()) {
        const unsigned hw = std::thread::hardware_concurrency();
        helpers_ = static_cast<int>(std::min<unsigned>(3, hw > 1 ? hw - 1 : 0));
        for (int i = 0; i < helpers_; ++i)
            std::thread([this, i] { run(i); }).detach();
    }

    void part(size_t i) {
        const size_t a = i * chunk_, b = std::min(n_, a + chunk_);
        if (a < b)
            std::memcpy(dst_ + a, src_ + a, b - a);
    }

    void run(int id) {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return gen_ != seen; });
            seen = gen_;
            lk.unlock();
            part(static_cast<size_t>(id));
            pending_.fetch_sub(1, std::memory_order_release);
        }
    }

    const pid_t pid_;
    int helpers_ = 0;
    std::mutex call_mu_, mu_;
    std::condition_variable cv_;
    uint64_t gen_ = 0;
    uint8_t *dst_ = nullptr;
    const uint8_t *src_ = nullptr;
    size_t n_ = 0, chunk_ = 0;
    std::atomic<int> pending_{0};
};

inline void host_copy(void *dst, const void *src, size_t n) { HostCopier::get().copy(dst, src, n); }

} // namespace mvb
