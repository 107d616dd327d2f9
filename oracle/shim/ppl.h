/* Stand-in for MSVC's <ppl.h> so the reference sources compile with g++ on
 * Linux.  Only Concurrency::parallel_for(first, last, body) is used by the
 * reference (cpp/dequant_k.cpp:387); this one splits [first, last) over the
 * host's hardware threads with std::thread.  Test infrastructure only. */
#pragma once
#include <algorithm>
#include <thread>
#include <vector>

namespace Concurrency {
template <class T, class F>
void parallel_for(T first, T last, F body) {
    const T count = last - first;
    if (count <= 0) return;
    unsigned hw = std::thread::hardware_concurrency();
    const T workers = std::max<T>(1, std::min<T>(count, (T)(hw ? hw : 1)));
    std::vector<std::thread> pool;
    for (T w = 0; w < workers; ++w) {
        pool.emplace_back([=, &body]() {
            for (T i = first + w; i < last; i += workers) body(i);
        });
    }
    for (auto& t : pool) t.join();
}
}  // namespace Concurrency
