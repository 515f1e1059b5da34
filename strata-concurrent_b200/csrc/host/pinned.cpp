// pinned.cpp - the page-locked host block pool behind parked conversations (include/strata_kv/pinned.hpp).
#include "strata_kv/pinned.hpp"

#include <cuda_runtime.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace strata::kv {
namespace {

struct Block {
    size_t cls = 0;       // the size actually allocated
    bool locked = false;  // page-locked (cudaHostAlloc) vs heap
};

struct Pool {
    std::mutex mu;
    std::unordered_map<void*, Block> live;
    std::map<size_t, std::vector<void*>> free_by_class;   // page-locked blocks waiting for reuse
    size_t live_bytes = 0, cached_bytes = 0, lock_calls = 0, heap_blocks = 0;
    size_t cache_limit = size_t(8) << 30;
    int cuda = -1;   // -1 unknown, 0 unusable, 1 usable
};

Pool& pool() {
    static Pool* p = new Pool();   // never destroyed: blocks may be freed during static destruction
    return *p;
}

/// Power-of-two classes from 64 KiB to 16 MiB; above that, whole 2 MiB multiples.
size_t size_class(size_t bytes) {
    if (bytes > (size_t(16) << 20)) return (bytes + (size_t(2) << 20) - 1) & ~((size_t(2) << 20) - 1);
    size_t c = kPinnedMinBytes;
    while (c < bytes) c <<= 1;
    return c;
}

bool cuda_usable(Pool& P) {
    if (P.cuda < 0) {
        int n = 0;
        P.cuda = cudaGetDeviceCount(&n) == cudaSuccess && n > 0 ? 1 : 0;
        if (!P.cuda) (void) cudaGetLastError();
    }
    return P.cuda == 1;
}

void release_locked(void* p) { (void) cudaFreeHost(p); }

}  // namespace

void* pinned_alloc(size_t bytes) {
    if (bytes == 0) bytes = 1;
    Pool& P = pool();
    if (bytes < kPinnedMinBytes) {
        void* p = std::aligned_alloc(256, (bytes + 255) & ~size_t(255));
        if (!p) throw std::bad_alloc();
        std::lock_guard<std::mutex> lock(P.mu);
        P.live[p] = Block{bytes, false};
        ++P.heap_blocks;
        return p;
    }
    const size_t cls = size_class(bytes);
    {
        std::lock_guard<std::mutex> lock(P.mu);
        auto it = P.free_by_class.find(cls);
        if (it != P.free_by_class.end() && !it->second.empty()) {
            void* p = it->second.back();
            it->second.pop_back();
            P.cached_bytes -= cls;
            P.live[p] = Block{cls, true};
            P.live_bytes += cls;
            return p;
        }
    }
    void* p = nullptr;
    bool locked = false;
    if (cuda_usable(P) && cudaHostAlloc(&p, cls, cudaHostAllocPortable | cudaHostAllocMapped) == cudaSuccess) {
        locked = true;
    } else {
        (void) cudaGetLastError();
        p = std::aligned_alloc(256, cls);
        if (!p) throw std::bad_alloc();
    }
    std::lock_guard<std::mutex> lock(P.mu);
    P.live[p] = Block{cls, locked};
    P.live_bytes += cls;
    if (locked) ++P.lock_calls;
    else ++P.heap_blocks;
    return p;
}

void pinned_free(void* p, size_t) noexcept {
    if (!p) return;
    Pool& P = pool();
    std::unique_lock<std::mutex> lock(P.mu);
    auto it = P.live.find(p);
    if (it == P.live.end()) return;
    const Block b = it->second;
    P.live.erase(it);
    if (!b.locked) {
        if (b.cls >= kPinnedMinBytes) P.live_bytes -= b.cls;
        --P.heap_blocks;
        lock.unlock();
        std::free(p);
        return;
    }
    P.live_bytes -= b.cls;
    if (P.cached_bytes + b.cls <= P.cache_limit) {
        P.free_by_class[b.cls].push_back(p);
        P.cached_bytes += b.cls;
        return;
    }
    lock.unlock();
    release_locked(p);
}

bool pinned_is_locked(const void* p) {
    Pool& P = pool();
    std::lock_guard<std::mutex> lock(P.mu);
    auto it = P.live.find(const_cast<void*>(p));
    if (it != P.live.end()) return it->second.locked;
    for (const auto& [base, b] : P.live)
        if (b.locked && p >= base && static_cast<const uint8_t*>(p) < static_cast<const uint8_t*>(base) + b.cls)
            return true;
    return false;
}

PinnedStats pinned_stats() {
    Pool& P = pool();
    std::lock_guard<std::mutex> lock(P.mu);
    return PinnedStats{P.live_bytes, P.cached_bytes, P.lock_calls, P.heap_blocks};
}

void pinned_trim() {
    Pool& P = pool();
    std::vector<void*> out;
    {
        std::lock_guard<std::mutex> lock(P.mu);
        for (auto& [cls, v] : P.free_by_class) out.insert(out.end(), v.begin(), v.end());
        P.free_by_class.clear();
        P.cached_bytes = 0;
    }
    for (void* p : out) release_locked(p);
}

void pinned_set_cache_limit(size_t bytes) {
    Pool& P = pool();
    std::lock_guard<std::mutex> lock(P.mu);
    P.cache_limit = bytes;
}

}  // namespace strata::kv
