// include/strata_kv/conversation_cache.hpp - parked conversations: the image types and the park store.
//
// Interface and policy of the reference's include/strata/core/conversation_cache.hpp:47-456, implemented here:
//   * the image types (ConversationCheckpoint, ConversationKv, ConversationKvReuse, ConversationStageSnapshot,
//     SavedConversation) with their byte accounting.  The K/V streams (over 90 % of a park's bytes) are pinned
//     ConversationBuffers; the running-state vectors keep the reference's plain std::vector<uint8_t> type so
//     code that takes them as such keeps compiling;
//   * the prefix rules (conversation_prefix: a strict prefix of the prompt; conversation_same_branch: exactly
//     the branch), with image identity compared in order;
//   * ConversationCache: a fixed number of slots and a byte budget, least-recently-used eviction that prefers
//     entries no running request has claimed, claims (an entry claimed by one request is never offered to
//     another), and the retained K/V of the last mount for an incremental re-park.
#pragma once

#include "strata_kv/conversation_buffer.hpp"
#include "strata_kv/pinned.hpp"

#include <algorithm>
#include <array>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <utility>
#include <vector>

namespace strata::core {

/// `SavedConversation::owner` of an entry no running request owns.
constexpr int64_t kNoOwner = -1;

struct ConversationImageKey {
    int64_t start = 0;
    uint64_t hash = 0;
    bool operator==(const ConversationImageKey&) const = default;
};

struct ConversationCheckpoint {
    std::vector<int32_t> ids;
    std::vector<ConversationImageKey> imgs;
    std::vector<uint8_t> gdn, ple, tails, dead, block_pos;
    uint64_t used = 0;
    /// A layer-split checkpoint: one part per LATER stage, in stage order (this one is the first stage's).
    std::vector<ConversationCheckpoint> stage_parts;

    size_t bytes() const {
        size_t n = ids.capacity() * sizeof(int32_t) + imgs.capacity() * sizeof(ConversationImageKey);
        for (const auto* b : {&gdn, &ple, &tails, &dead, &block_pos}) n += b->capacity();
        n += stage_parts.capacity() * sizeof(ConversationCheckpoint);
        for (const auto& part : stage_parts) n += part.bytes();
        return n;
    }
};

/// One QSA layer's parked K/V in logical (identity) page order, whatever table the pool used.
struct ConversationKv {
    int format = 0;
    int64_t cells = 0, heads = 0, head_dim = 0, page_size = 0, pooled_rows = 0, idx_dim = 0;
    ConversationBuffer k, v, k_scale, v_scale, pooled;
    size_t bytes() const { return k.bytes() + v.bytes() + k_scale.bytes() + v_scale.bytes() + pooled.bytes(); }
};

struct ConversationKvReuse {
    std::vector<ConversationKv> kv;
    int64_t captured_tokens = 0, unchanged_tokens = 0;
    size_t bytes() const {
        size_t n = kv.capacity() * sizeof(ConversationKv);
        for (const auto& layer : kv) n += layer.bytes();
        return n;
    }
};

/// One LATER stage of a layer split inside a parked conversation.
struct ConversationStageSnapshot {
    int64_t layer_lo = 0, layer_hi = 0;
    ConversationCheckpoint state;
    std::vector<ConversationKv> kv;
    size_t bytes() const {
        size_t n = state.bytes() + kv.capacity() * sizeof(ConversationKv);
        for (const auto& k : kv) n += k.bytes();
        return n;
    }
};

struct SavedConversation {
    std::array<int64_t, 18> geometry{};
    int64_t layer_lo = 0, layer_hi = 0;
    ConversationCheckpoint live;
    std::vector<ConversationCheckpoint> checkpoints;
    std::vector<ConversationKv> kv;   ///< main layers, then the draft layer
    std::vector<ConversationStageSnapshot> stage_parts;
    bool cvec = true;
    int64_t owner = kNoOwner;          ///< the running request whose branch this is, or kNoOwner

    size_t bytes() const {
        size_t n = live.bytes() + checkpoints.capacity() * sizeof(ConversationCheckpoint) +
                   kv.capacity() * sizeof(ConversationKv) + stage_parts.capacity() * sizeof(ConversationStageSnapshot);
        for (const auto& c : checkpoints) n += c.bytes();
        for (const auto& k : kv) n += k.bytes();
        for (const auto& p : stage_parts) n += p.bytes();
        return n;
    }
};

namespace conversation_match_detail {
/// The images of `c` are exactly the images of the query that start inside its `n` tokens, in order.
inline bool images_agree(const ConversationCheckpoint& c, const std::vector<ConversationImageKey>& images, size_t n) {
    size_t j = 0;
    for (const auto& image : images) {
        if (image.start >= (int64_t) n) continue;
        if (j == c.imgs.size() || !(c.imgs[j] == image)) return false;
        ++j;
    }
    return j == c.imgs.size();
}
}  // namespace conversation_match_detail

/// Tokens reusable from `c` for `prompt`: its whole length when it is a STRICT prefix of the prompt (the last
/// prompt token must still be read) with the same images; otherwise 0.
template <class Token>
int64_t conversation_prefix(const ConversationCheckpoint& c, const std::vector<Token>& prompt,
                            const std::vector<ConversationImageKey>& images) {
    const size_t n = c.ids.size();
    if (n == 0 || n >= prompt.size()) return 0;
    if (!std::equal(c.ids.begin(), c.ids.end(), prompt.begin())) return 0;
    return conversation_match_detail::images_agree(c, images, n) ? (int64_t) n : 0;
}

/// Tokens of `c` when it IS `branch` (same length, same tokens, same images); otherwise 0.
template <class Token>
int64_t conversation_same_branch(const ConversationCheckpoint& c, const std::vector<Token>& branch,
                                 const std::vector<ConversationImageKey>& images) {
    const size_t n = c.ids.size();
    if (n == 0 || n != branch.size()) return 0;
    if (!std::equal(c.ids.begin(), c.ids.end(), branch.begin())) return 0;
    return conversation_match_detail::images_agree(c, images, n) ? (int64_t) n : 0;
}

class ConversationCache {
public:
    struct Match {
        size_t index = 0;
        int64_t tokens = 0;
        bool live = false;
    };
    static constexpr size_t default_slots = 8;

    ConversationCache(size_t budget, size_t slots) : budget_(budget), slots_(slots) {}

    bool enabled() const { return budget_ != 0 && slots_ != 0; }
    size_t bytes() const { return parked_bytes_ + retained_.bytes(); }
    size_t size() const { return entries_.size(); }
    size_t slots() const { return slots_; }
    size_t budget() const { return budget_; }
    size_t evictions() const { return evictions_; }
    uint64_t clock() const { return clock_; }
    uint64_t use(size_t index) const { return stamps_.at(index); }

    /// Keep the K/V a mount just restored, for an incremental re-park; never evicts anything to fit.
    void retain(std::vector<ConversationKv>&& kv, int64_t tokens) {
        retained_ = {};
        ConversationKvReuse candidate{std::move(kv), tokens, tokens};
        if (enabled() && candidate.bytes() <= budget_ - parked_bytes_) retained_ = std::move(candidate);
    }
    /// A rewrite at `first_dirty` bounds how much of the retained K/V is still valid.
    void limit_reuse(int64_t first_dirty) {
        retained_.unchanged_tokens = std::min(retained_.unchanged_tokens, first_dirty);
        if (retained_.unchanged_tokens <= 0) retained_ = {};
    }
    ConversationKvReuse take_reuse() { return std::exchange(retained_, {}); }
    size_t retained_bytes() const { return retained_.bytes(); }

    bool can_fit(size_t incoming, size_t held = 0) const {
        if (!enabled() || held > budget_ || incoming > budget_ - held) return false;
        return entries_.size() < slots_ && bytes() <= budget_ - held - incoming;
    }

    /// Index of the smallest stamp; equal stamps resolve to the earlier index.  0 for n == 0.
    static size_t lru_victim(const uint64_t* stamps, size_t n) {
        size_t best = 0;
        for (size_t i = 1; i < n; ++i)
            if (stamps[i] < stamps[best]) best = i;
        return best;
    }

    /// The longest reusable prefix for `prompt`, among entries not claimed by another request (a hit is a use).
    template <class Token>
    Match best(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
               int64_t requester = kNoOwner) {
        const Match m = search(prompt, images, cvec, requester);
        if (m.tokens > 0) touch(m.index);
        return m;
    }

    /// The same search without counting it as a use.
    template <class Token>
    Match probe(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
                int64_t requester = kNoOwner) const {
        return search(prompt, images, cvec, requester);
    }

    /// The parked LIVE branch that is exactly `branch` (a hand-over back to the slot that parked it).
    template <class Token>
    Match best_exact(const std::vector<Token>& branch, const std::vector<ConversationImageKey>& images, bool cvec,
                     int64_t requester = kNoOwner) {
        Match found;
        for (size_t i = entries_.size(); i-- > 0;) {
            const SavedConversation& e = entries_[i];
            if (e.cvec != cvec || claimed_by_other(i, requester)) continue;
            const int64_t n = conversation_same_branch(e.live, branch, images);
            if (n > found.tokens) found = Match{i, n, true};
        }
        if (found.tokens > 0) touch(found.index);
        return found;
    }

    void touch(size_t index) { stamps_.at(index) = ++clock_; }

    bool claimed_by_other(size_t index, int64_t requester) const {
        const int64_t o = entries_.at(index).owner;
        return o != kNoOwner && requester != kNoOwner && o != requester;
    }
    void release_owner(int64_t id) {
        for (auto& e : entries_)
            if (e.owner == id) e.owner = kNoOwner;
    }
    int64_t owner(size_t index) const { return entries_.at(index).owner; }

    /// Remove and return the entry (a mount).  The clock advances so the next park is newer than all entries.
    SavedConversation take(size_t index) {
        SavedConversation out = std::move(entries_.at(index));
        parked_bytes_ -= out.bytes();
        drop(index);
        ++clock_;
        return out;
    }

    /// Evict until `incoming` bytes fit beside `held` (an image taken out but still alive) and a slot is free.
    bool make_room(size_t incoming, size_t held = 0) {
        if (!enabled() || held > budget_ || incoming > budget_ - held) return false;
        const size_t room = budget_ - held - incoming;
        if (bytes() > room) retained_ = {};
        while (!entries_.empty() && (entries_.size() >= slots_ || parked_bytes_ > room)) {
            const size_t v = victim_to_prune();
            parked_bytes_ -= entries_[v].bytes();
            drop(v);
            ++evictions_;
        }
        return true;
    }

    /// Least recently used among unclaimed entries; least recently used overall when all are claimed.
    size_t victim_to_prune() const {
        if (entries_.empty()) return 0;
        bool have_free = false;
        size_t best = 0;
        for (size_t i = 0; i < entries_.size(); ++i) {
            if (entries_[i].owner != kNoOwner) continue;
            if (!have_free || stamps_[i] < stamps_[best]) best = i;
            have_free = true;
        }
        return have_free ? best : lru_victim(stamps_.data(), stamps_.size());
    }

    /// Park `image`, claimed by `owner` (kNoOwner: the cache's).  False when it cannot fit at all.
    bool put(SavedConversation&& image, int64_t owner = kNoOwner, size_t held = 0) {
        const size_t n = image.bytes();
        if (!make_room(n, held)) return false;
        image.owner = owner;
        entries_.push_back(std::move(image));
        stamps_.push_back(++clock_);
        parked_bytes_ += n;
        return true;
    }

private:
    void drop(size_t index) {
        entries_.erase(entries_.begin() + (std::ptrdiff_t) index);
        stamps_.erase(stamps_.begin() + (std::ptrdiff_t) index);
    }

    /// Longest exact prefix over every entry's live branch and checkpoints, newest entry first; equal lengths
    /// keep the first found (the newest entry, its live branch before its checkpoints).
    template <class Token>
    Match search(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
                 int64_t requester) const {
        Match found;
        for (size_t i = entries_.size(); i-- > 0;) {
            const SavedConversation& e = entries_[i];
            if (e.cvec != cvec || claimed_by_other(i, requester)) continue;
            const int64_t live = conversation_prefix(e.live, prompt, images);
            if (live > found.tokens) found = Match{i, live, true};
            for (const auto& c : e.checkpoints) {
                const int64_t n = conversation_prefix(c, prompt, images);
                if (n > found.tokens) found = Match{i, n, false};
            }
        }
        return found;
    }

    size_t budget_ = 0, slots_ = 0, parked_bytes_ = 0, evictions_ = 0;
    uint64_t clock_ = 0;
    std::deque<SavedConversation> entries_;   // park order, oldest first
    std::vector<uint64_t> stamps_;            // entries_[i]'s last use
    ConversationKvReuse retained_;
};

}  // namespace strata::core
