// Parallel host memcpy for the host-buffer entry points: a caller's pageable
// array is copied into (or out of) pinned staging by the calling thread plus
// a few persistent worker threads, in 128 KiB pieces.
//
// Each copy is one Job object shared with the workers by shared_ptr.  Pieces
// are claimed from the job's own counter, so a worker that wakes late (after
// the caller has finished the job and returned) finds no piece left and
// touches no memory; the caller returns once every claimed piece is done.
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "launch.h"

namespace moeb200 {

namespace {

constexpr size_t kPiece = 128 << 10;
constexpr size_t kParallelMin = 512 << 10;   // below this one memcpy is faster

struct Job {
    char* dst;
    const char* src;
    size_t bytes;
    size_t pieces;
    uint64_t gen;
    std::atomic<size_t> next{0};
    std::atomic<size_t> done{0};

    void run() {
        for (;;) {
            const size_t i = next.fetch_add(1, std::memory_order_relaxed);
            if (i >= pieces) return;
            const size_t at = i * kPiece;
            const size_t n = bytes - at < kPiece ? bytes - at : kPiece;
            std::memcpy(dst + at, src + at, n);
            done.fetch_add(1, std::memory_order_release);
        }
    }
};

class CopyPool {
public:
    CopyPool() {
        const unsigned hw = std::thread::hardware_concurrency();
        const unsigned n = hw > 2 ? (hw - 1 < 7 ? hw - 1 : 7) : 0;
        for (unsigned i = 0; i < n; ++i) workers_.emplace_back([this] { loop(); });
        for (auto& t : workers_) t.detach();   // the pool lives until the process ends
    }

    void copy(void* dst, const void* src, size_t bytes) {
        if (bytes < kParallelMin || workers_.empty()) {
            std::memcpy(dst, src, bytes);
            return;
        }
        std::lock_guard<std::mutex> one(call_);   // one job at a time
        auto job = std::make_shared<Job>();
        job->dst = static_cast<char*>(dst);
        job->src = static_cast<const char*>(src);
        job->bytes = bytes;
        job->pieces = (bytes + kPiece - 1) / kPiece;
        {
            std::lock_guard<std::mutex> lk(m_);
            job->gen = ++gen_;
            cur_ = job;
        }
        cv_.notify_all();
        job->run();
        while (job->done.load(std::memory_order_acquire) < job->pieces) std::this_thread::yield();
    }

private:
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            std::shared_ptr<Job> job;
            {
                std::unique_lock<std::mutex> lk(m_);
                cv_.wait(lk, [&] { return cur_ && cur_->gen != seen; });
                job = cur_;
                seen = job->gen;
            }
            job->run();
        }
    }

    std::vector<std::thread> workers_;
    std::mutex m_, call_;
    std::condition_variable cv_;
    std::shared_ptr<Job> cur_;
    uint64_t gen_ = 0;
};

}  // namespace

void host_parallel_copy(void* dst, const void* src, size_t bytes) {
    static CopyPool* pool = new CopyPool();   // never destroyed: detached workers
    pool->copy(dst, src, bytes);
}

}  // namespace moeb200
