// host_pool.h -- a small persistent host thread pool for the synchronous f32 host path:
// the copies between the caller's pageable buffers and the backend's pinned staging
// buffers are memory-bandwidth bound, and one thread moves only a fraction of what the
// host's memory system and the PCIe link can carry.
#pragma once

#include <algorithm>
#include <condition_variable>
#include <cstddef>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace ql {

class HostPool {
  public:
    explicit HostPool(int threads) {
        for (int i = 0; i < threads; i++) workers_.emplace_back([this] { loop(); });
    }
    ~HostPool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
    }
    HostPool(const HostPool &) = delete;
    HostPool &operator=(const HostPool &) = delete;

    int size() const { return (int)workers_.size() + 1; }

    // Runs fn(0) .. fn(n - 1) on the workers and the calling thread; returns when all ran.
    void parallel_for(int n, const std::function<void(int)> &fn) {
        if (n <= 0) return;
        if (n == 1 || workers_.empty()) {
            for (int i = 0; i < n; i++) fn(i);
            return;
        }
        {
            std::lock_guard<std::mutex> g(mu_);
            fn_ = &fn;
            n_ = n;
            next_ = 0;
            pending_ = n;
            gen_++;
        }
        cv_.notify_all();
        run_tasks();
        std::unique_lock<std::mutex> l(mu_);
        done_.wait(l, [this] { return pending_ == 0; });
        fn_ = nullptr;
    }

    // memcpy of rows (bytes per row, source / destination row strides in bytes) split over
    // the pool in pieces of at least min_piece bytes.
    void copy_rows(void *dst, size_t dst_stride, const void *src, size_t src_stride, size_t rows,
                   size_t row_bytes, size_t min_piece = 256 << 10) {
        const size_t total = rows * row_bytes;
        if (total == 0) return;
        const bool dense = dst_stride == row_bytes && src_stride == row_bytes;
        const int pieces = (int)std::max<size_t>(
            1, std::min<size_t>((size_t)size() * 2, total / std::max<size_t>(min_piece, 1)));
        char *d = static_cast<char *>(dst);
        const char *s = static_cast<const char *>(src);
        if (dense) {
            parallel_for(pieces, [&](int i) {
                const size_t a = total * i / pieces, b = total * (i + 1) / pieces;
                std::memcpy(d + a, s + a, b - a);
            });
            return;
        }
        const int prow = (int)std::min<size_t>(pieces, rows);
        parallel_for(prow, [&](int i) {
            const size_t a = rows * i / prow, b = rows * (i + 1) / prow;
            for (size_t r = a; r < b; r++)
                std::memcpy(d + r * dst_stride, s + r * src_stride, row_bytes);
        });
    }

  private:
    void run_tasks() {
        while (true) {
            int i;
            {
                std::lock_guard<std::mutex> g(mu_);
                if (!fn_ || next_ >= n_) return;
                i = next_++;
            }
            (*fn_)(i);
            std::lock_guard<std::mutex> g(mu_);
            if (--pending_ == 0) done_.notify_all();
        }
    }
    void loop() {
        unsigned long long seen = 0;
        while (true) {
            {
                std::unique_lock<std::mutex> l(mu_);
                cv_.wait(l, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
            }
            run_tasks();
        }
    }

    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::function<void(int)> *fn_ = nullptr;
    int n_ = 0, next_ = 0, pending_ = 0;
    unsigned long long gen_ = 0;
    bool stop_ = false;
};

}  // namespace ql
