// include/strata_kv/conversation_buffer.hpp - host storage of one parked K/V stream.
//
// Same interface and byte accounting as the reference's ConversationBuffer
// (include/strata/core/conversation_buffer.hpp:16-152): a directory of segments of at most 16 MiB, no data()
// (payloads are reached with visit()/read()), appends never move existing bytes, and bytes() counts what the
// directory and the segments hold.  What differs is where the segments live: page-locked, device-mapped host
// blocks from strata::kv::pinned_alloc, so the park and mount copies run asynchronously at PCIe speed.
//
// Growth policy (kept identical because the conversation cache's RAM budget is computed from it): a buffer
// filled from empty allocates exactly its payload; later growth first fills the last segment's spare capacity,
// then adds segments whose capacity grows geometrically (at least 64 KiB, at most 16 MiB).
#pragma once

#include "strata_kv/pinned.hpp"

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <initializer_list>
#include <utility>
#include <vector>

namespace strata::core {

class ConversationBuffer {
public:
    static constexpr size_t segment_bytes = size_t(16) << 20;

    /// One directory entry: a pinned block holding `size` payload bytes out of `capacity`.
    struct Segment {
        uint8_t* data = nullptr;
        size_t size = 0;
        size_t capacity = 0;
    };

    ConversationBuffer() = default;
    ConversationBuffer(std::initializer_list<uint8_t> values) {
        resize(values.size());
        size_t at = 0;
        for (auto& s : dir_) {
            std::memcpy(s.data, values.begin() + at, s.size);
            at += s.size;
        }
    }
    ConversationBuffer(const ConversationBuffer& other) { copy_from(other); }
    ConversationBuffer& operator=(const ConversationBuffer& other) {
        if (this != &other) {
            ConversationBuffer tmp(other);
            swap(tmp);
        }
        return *this;
    }
    ConversationBuffer(ConversationBuffer&& other) noexcept
        : dir_(std::move(other.dir_)), size_(std::exchange(other.size_, 0)) {
        other.dir_.clear();
    }
    ConversationBuffer& operator=(ConversationBuffer&& other) noexcept {
        if (this != &other) {
            release();
            dir_ = std::move(other.dir_);
            other.dir_.clear();
            size_ = std::exchange(other.size_, 0);
        }
        return *this;
    }
    ~ConversationBuffer() { release(); }

    void swap(ConversationBuffer& other) noexcept {
        dir_.swap(other.dir_);
        std::swap(size_, other.size_);
    }

    size_t size() const { return size_; }
    bool empty() const { return size_ == 0; }

    /// The host bytes this buffer holds: the directory plus every segment's capacity.
    size_t bytes() const {
        size_t n = dir_.capacity() * sizeof(Segment);
        for (const auto& s : dir_) n += s.capacity;
        return n;
    }

    /// bytes() while a resize to `n` is in flight (the old directory counted until its replacement exists);
    /// SIZE_MAX when the arithmetic would overflow, so an impossible request fails the budget check.
    size_t allocation_peak(size_t n) const {
        size_t total = bytes();
        if (n <= size_) return total;
        size_t need = n - size_;
        const size_t spare = dir_.empty() ? 0 : dir_.back().capacity - dir_.back().size;
        need -= std::min(need, spare);
        const size_t whole = need / segment_bytes, rest = need % segment_bytes;
        if (!grow(total, whole * segment_bytes)) return SIZE_MAX;
        if (rest) {
            const size_t prev = whole ? segment_bytes : (dir_.empty() ? 0 : dir_.back().capacity);
            if (!grow(total, capacity_for(rest, prev, size_ != 0))) return SIZE_MAX;
        }
        size_t entries = dir_.size();
        if (!grow(entries, whole + (rest ? 1 : 0))) return SIZE_MAX;
        if (entries > dir_.capacity()) {
            if (entries > SIZE_MAX / sizeof(Segment) || !grow(total, entries * sizeof(Segment))) return SIZE_MAX;
        }
        return total;
    }

    void resize(size_t n, uint8_t value = 0) {
        if (n <= size_) {
            shrink(n);
            return;
        }
        const bool appending = size_ != 0;
        size_t need = n - size_;
        const size_t spare = dir_.empty() ? 0 : dir_.back().capacity - dir_.back().size;
        const size_t fill = std::min(need, spare);
        const size_t rest = need - fill;
        dir_.reserve(dir_.size() + rest / segment_bytes + (rest % segment_bytes ? 1 : 0));
        if (fill) {
            Segment& last = dir_.back();
            std::memset(last.data + last.size, value, fill);
            last.size += fill;
            size_ += fill;
        }
        while (size_ < n) {
            const size_t count = std::min(segment_bytes, n - size_);
            const size_t prev = dir_.empty() ? 0 : dir_.back().capacity;
            Segment s;
            s.capacity = capacity_for(count, prev, appending);
            s.data = static_cast<uint8_t*>(strata::kv::pinned_alloc(s.capacity));
            s.size = count;
            std::memset(s.data, value, count);
            dir_.push_back(s);
            size_ += count;
        }
    }
    void pop_back() { resize(size_ - 1); }

    /// fn(pointer, count, absolute_offset) over [offset, offset + count) in segment order; false from fn
    /// aborts.  False when the range is outside the buffer.
    template <class Fn>
    bool visit(size_t offset, size_t count, Fn fn) {
        return walk(dir_, size_, offset, count, fn);
    }
    template <class Fn>
    bool visit(size_t offset, size_t count, Fn fn) const {
        return walk(dir_, size_, offset, count, fn);
    }
    bool read(void* target, size_t offset, size_t count) const {
        return visit(offset, count, [&](const uint8_t* p, size_t n, size_t at) {
            std::memcpy(static_cast<uint8_t*>(target) + (at - offset), p, n);
            return true;
        });
    }
    bool operator==(const ConversationBuffer& other) const {
        if (size_ != other.size_) return false;
        size_t i = 0, j = 0, a = 0, b = 0;
        while (i < dir_.size() && j < other.dir_.size()) {
            const Segment& x = dir_[i];
            const Segment& y = other.dir_[j];
            const size_t n = std::min(x.size - a, y.size - b);
            if (n && std::memcmp(x.data + a, y.data + b, n) != 0) return false;
            a += n;
            b += n;
            if (a == x.size) ++i, a = 0;
            if (b == y.size) ++j, b = 0;
        }
        return true;
    }
    bool operator!=(const ConversationBuffer& other) const { return !(*this == other); }

    /// The segment directory, for the copy planner (device <-> host transfers of the payload).
    const std::vector<Segment>& segments() const { return dir_; }

private:
    static bool grow(size_t& n, size_t extra) {
        if (extra > SIZE_MAX - n) return false;
        n += extra;
        return true;
    }
    /// A fresh buffer allocates exactly; an appending one reserves geometrically (64 KiB .. 16 MiB).
    static size_t capacity_for(size_t count, size_t previous, bool appending) {
        if (!appending) return count;
        const size_t doubled = std::min(previous, segment_bytes / 2) * 2;
        return std::max(count, std::min(segment_bytes, std::max<size_t>(65536, doubled)));
    }
    template <class Dir, class Fn>
    static bool walk(Dir& dir, size_t total, size_t offset, size_t count, Fn& fn) {
        if (offset > total || count > total - offset) return false;
        size_t start = 0;
        for (auto& s : dir) {
            if (!count) break;
            const size_t end = start + s.size;
            if (offset < end) {
                const size_t n = std::min(count, end - offset);
                if (!fn(s.data + (offset - start), n, offset)) return false;
                offset += n;
                count -= n;
            }
            start = end;
        }
        return count == 0;
    }
    void shrink(size_t n) {
        while (!dir_.empty() && size_ - dir_.back().size >= n) {
            size_ -= dir_.back().size;
            strata::kv::pinned_free(dir_.back().data, dir_.back().capacity);
            dir_.pop_back();
        }
        if (size_ > n) {
            dir_.back().size -= size_ - n;
            size_ = n;
        }
        size_ = n;
    }
    /// A copy holds exactly the payload (like copying a std::vector): directory and segments sized to fit.
    void copy_from(const ConversationBuffer& other) {
        dir_.reserve(other.dir_.size());
        for (const auto& s : other.dir_) {
            Segment c;
            c.capacity = s.size;
            c.size = s.size;
            c.data = static_cast<uint8_t*>(strata::kv::pinned_alloc(s.capacity));
            std::memcpy(c.data, s.data, s.size);
            dir_.push_back(c);
        }
        size_ = other.size_;
    }
    void release() noexcept {
        for (auto& s : dir_) strata::kv::pinned_free(s.data, s.capacity);
        dir_.clear();
        size_ = 0;
    }

    std::vector<Segment> dir_;
    size_t size_ = 0;
};

}  // namespace strata::core
