// include/strata_kv/pinned.hpp - page-locked host memory for parked conversations.
//
// The reference parks into pageable std::vector segments (include/strata/core/conversation_buffer.hpp:16-152),
// so every park/mount copy is a staged, synchronous cudaMemcpy.  Here the large host buffers of a parked
// conversation come from a process-wide pool of page-locked, device-mapped blocks, so the copy engine moves
// them at PCIe speed asynchronously.  Page-locking is expensive (it is a kernel call per block), so freed blocks
// are kept by size class and handed out again.
//
// Without a usable CUDA device (host-only tools and tests) the same calls hand out ordinary heap memory; the
// copies then take the staged path, they do not change.
#pragma once

#include <cstddef>
#include <cstdint>
#include <limits>
#include <new>

namespace strata::kv {

/// Requests below this many bytes come from the heap (small buffers gain nothing from page-locking).
inline constexpr size_t kPinnedMinBytes = 64 * 1024;

/// `bytes` of host memory, 256-byte aligned; page-locked and device-mapped when CUDA is usable.  Never null:
/// throws std::bad_alloc, which is what the reference's park path already handles (`park_current`).
void* pinned_alloc(size_t bytes);
/// Return a block from pinned_alloc (the same `bytes`).  Page-locked blocks go back to the cache.
void pinned_free(void* p, size_t bytes) noexcept;
/// Whether `p` (anywhere inside a live block) is page-locked memory.
bool pinned_is_locked(const void* p);

struct PinnedStats {
    size_t live_bytes = 0;       ///< handed out and not yet freed (class-rounded)
    size_t cached_bytes = 0;     ///< page-locked and waiting for reuse
    size_t lock_calls = 0;       ///< page-locking allocations made so far
    size_t heap_blocks = 0;      ///< live blocks that are ordinary heap memory
};
PinnedStats pinned_stats();
/// Release every cached page-locked block back to the system.
void pinned_trim();
/// Upper bound on cached (free) page-locked bytes; freeing beyond it releases blocks.  Default 8 GiB.
void pinned_set_cache_limit(size_t bytes);

/// A std::allocator over pinned_alloc, for contiguous running-state vectors.
template <class T>
struct PinnedAllocator {
    using value_type = T;
    PinnedAllocator() noexcept = default;
    template <class U>
    PinnedAllocator(const PinnedAllocator<U>&) noexcept {}
    T* allocate(size_t n) {
        if (n > std::numeric_limits<size_t>::max() / sizeof(T)) throw std::bad_alloc();
        return static_cast<T*>(pinned_alloc(n * sizeof(T)));
    }
    void deallocate(T* p, size_t n) noexcept { pinned_free(p, n * sizeof(T)); }
    template <class U>
    bool operator==(const PinnedAllocator<U>&) const noexcept { return true; }
    template <class U>
    bool operator!=(const PinnedAllocator<U>&) const noexcept { return false; }
};

}  // namespace strata::kv
