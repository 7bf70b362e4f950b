// staging.h — how an upload of many host byte ranges is cut into pinned chunks.
//
// The bytes of every segment, taken in order, form one stream; chunk i of a
// `cap`-byte staging buffer holds stream bytes [i*cap, (i+1)*cap). A chunk is
// described by its pieces: which segment, where in it, where in the chunk,
// how many bytes. Host threads fill a chunk by stage ranges (stage_fill), and
// each piece then goes to its own device destination in one copy. Plain host
// code with no CUDA types, so the arithmetic is checked on the CPU as well.
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace strata {

struct StageSeg {
    uint8_t* dst;        // device destination (opaque here)
    const uint8_t* src;  // host source
    size_t n;            // bytes
};

struct StagePiece {
    int64_t seg;     // index into the segment list
    size_t seg_off;  // first byte within the segment
    size_t off;      // first byte within the chunk
    size_t n;        // bytes
};

struct StageCursor {
    int64_t seg = 0;  // next segment to read
    size_t off = 0;   // bytes of it already planned
};

// Plans the next chunk of at most `cap` bytes starting at `cur`, which it
// advances; returns the bytes planned (0 once every segment is done).
// Empty segments are passed over.
inline size_t stage_plan(const StageSeg* segs, int64_t nseg, StageCursor& cur, size_t cap,
                         std::vector<StagePiece>& out) {
    out.clear();
    size_t fill = 0;
    while (fill < cap && cur.seg < nseg) {
        const size_t left = segs[cur.seg].n - cur.off;
        const size_t take = left < cap - fill ? left : cap - fill;
        if (take) out.push_back({cur.seg, cur.off, fill, take});
        fill += take;
        cur.off += take;
        if (cur.off == segs[cur.seg].n) {
            ++cur.seg;
            cur.off = 0;
        }
    }
    return fill;
}

// Copies chunk bytes [a, b) from their sources into `stage` (one host
// thread's share of a chunk).
inline void stage_fill(const std::vector<StagePiece>& pieces, const StageSeg* segs, uint8_t* stage, size_t a,
                       size_t b) {
    for (const StagePiece& p : pieces) {
        const size_t lo = p.off > a ? p.off : a;
        const size_t hi = p.off + p.n < b ? p.off + p.n : b;
        if (lo < hi) memcpy(stage + lo, segs[p.seg].src + p.seg_off + (lo - p.off), hi - lo);
    }
}

// Copies n bytes between host buffers (the pinned staging and a caller's
// slice). One host thread copies at roughly 10 GB/s, so a synchronous call
// returning a few MB would spend most of its time here: copies of 2 MiB and
// more are split over up to 8 threads, at least 1 MiB each, in 64-byte-aligned
// parts; the calling thread copies the first part. If a thread cannot be
// started, its part is copied here instead.
inline void copy_host(void* dst, const void* src, size_t n) {
    constexpr size_t kMin = size_t(2) << 20, kPerThread = size_t(1) << 20;
    constexpr int kMaxThreads = 8;
    if (n < kMin) {
        if (n) memcpy(dst, src, n);
        return;
    }
    const size_t T = n / kPerThread < (size_t)kMaxThreads ? n / kPerThread : (size_t)kMaxThreads;  // >= 2
    const size_t part = ((n + T - 1) / T + 63) & ~size_t(63);  // T parts cover n
    char* d = static_cast<char*>(dst);
    const char* s = static_cast<const char*>(src);
    std::thread th[kMaxThreads];
    for (size_t t = 1; t < T; ++t) {
        const size_t a = t * part;
        if (a >= n) break;
        const size_t len = a + part < n ? part : n - a;
        try {
            th[t] = std::thread([d, s, a, len] { memcpy(d + a, s + a, len); });
        } catch (...) {
            memcpy(d + a, s + a, len);
        }
    }
    memcpy(d, s, part);
    for (auto& x : th)
        if (x.joinable()) x.join();
}

// A host copy split over persistent worker threads: started on first use
// and kept until the pool is destroyed, so a synchronous call that returns a
// few MB pays no thread start-up. Between copies a worker spins on the job
// counter for a while (about 100 us) and then sleeps on a condition variable;
// prime() wakes sleeping workers into that spin ahead of a copy whose data is
// still in flight, so the copy does not wait for threads to wake. copy() blocks until
// every part is written; one copy at a time (the owner serialises its calls).
// Copies under `kMin` bytes, or when no worker can be started, are one memcpy
// on the caller. copy2d() copies `height` rows of `width` bytes between
// pitched buffers, the rows' bytes split evenly over the threads.
class CopyPool {
  public:
    static constexpr size_t kMin = size_t(256) << 10;
    static constexpr int kWorkers = 7;
    static constexpr int kSpin = 1 << 17;  // polls before a worker sleeps

    CopyPool() = default;
    CopyPool(const CopyPool&) = delete;
    CopyPool& operator=(const CopyPool&) = delete;
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_.store(true);
        }
        go_.notify_all();
        for (auto& t : th_) t.join();
    }

    // Wakes the workers (starting them on first use) so they spin, ready for
    // a copy of at least kMin bytes that is about to come.
    void prime() {
        if (!start()) return;
        {
            std::lock_guard<std::mutex> g(m_);
            wake_.fetch_add(1);
        }
        go_.notify_all();
    }

    void copy(void* dst, const void* src, size_t n) { copy2d(dst, n, src, n, n, 1); }

    void copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height) {
        const size_t n = width * height;
        if (n < kMin || !start()) {
            for (size_t r = 0; r < height && width; ++r)
                memcpy(static_cast<char*>(dst) + r * dpitch, static_cast<const char*>(src) + r * spitch, width);
            return;
        }
        const size_t parts = (size_t)th_.size() + 1;
        const size_t part = ((n + parts - 1) / parts + 63) & ~size_t(63);
        {
            std::lock_guard<std::mutex> g(m_);
            d_ = static_cast<char*>(dst);
            s_ = static_cast<const char*>(src);
            dp_ = dpitch;
            sp_ = spitch;
            w_ = width;
            n_ = n;
            part_ = part;
            pending_.store((int)th_.size());
            gen_.fetch_add(1);
        }
        go_.notify_all();
        span(d_, dp_, s_, sp_, w_, 0, part < n ? part : n);  // the caller's part: the first
        while (pending_.load() != 0) std::this_thread::yield();
    }

  private:
    // bytes [a, b) of the rows laid end to end
    static void span(char* d, size_t dp, const char* s, size_t sp, size_t w, size_t a, size_t b) {
        while (a < b) {
            const size_t r = a / w, c = a % w, len = b - a < w - c ? b - a : w - c;
            memcpy(d + r * dp + c, s + r * sp + c, len);
            a += len;
        }
    }
    bool start() {
        if (started_) return !th_.empty();
        started_ = true;
        for (int w = 0; w < kWorkers; ++w) {
            try {
                th_.emplace_back([this, w] { run(w + 1); });
            } catch (...) {
                break;
            }
        }
        return !th_.empty();
    }
    void run(size_t idx) {
        uint64_t seen = 0, woken = 0;
        for (;;) {
            int spin = 0;
            while (gen_.load() == seen && !stop_.load() && spin < kSpin) ++spin;
            char* d;
            const char* s;
            size_t n, part, dp, sp, w;
            {
                std::unique_lock<std::mutex> g(m_);
                go_.wait(g, [&] { return stop_.load() || gen_.load() != seen || wake_.load() != woken; });
                if (stop_.load()) return;
                woken = wake_.load();
                if (gen_.load() == seen) continue;  // primed: spin for the coming copy
                seen = gen_.load();
                d = d_;
                s = s_;
                dp = dp_;
                sp = sp_;
                w = w_;
                n = n_;
                part = part_;
            }
            const size_t a = idx * part;
            if (a < n) span(d, dp, s, sp, w, a, a + part < n ? a + part : n);
            pending_.fetch_sub(1);
        }
    }

    std::mutex m_;
    std::condition_variable go_;
    std::vector<std::thread> th_;
    bool started_ = false;
    std::atomic<bool> stop_{false};
    std::atomic<uint64_t> gen_{0}, wake_{0};
    std::atomic<int> pending_{0};
    char* d_ = nullptr;
    const char* s_ = nullptr;
    size_t n_ = 0, part_ = 0, dp_ = 0, sp_ = 0, w_ = 0;
};

}  // namespace strata
