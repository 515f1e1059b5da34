// include/strata_kv/conversation_cache.hpp - parked conversations: the image types and the park store.
//
// Interface and policy of the reference's include/strata/core/conversation_cache.hpp:47-456, written here from the
// policy (the class comment below states it):
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
#include <optional>
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

/// The park store.  Its policy, as the engine relies on it:
///   * capacity: at most `slots` entries, and the entries plus the retained K/V within `budget` bytes (an image's
///     bytes() at the time it was parked);
///   * use clock: every park, every match handed out (best, best_exact) and every touch() stamps the entry with the
///     next tick; a take() advances the clock too, so a later park is newer than everything before it;
///   * eviction: entries no request has claimed go first, least recently used first; only when every entry is
///     claimed does the least recently used claimed one go.  The retained K/V is dropped before any entry;
///   * claims: an entry parked with an owner is offered to that request (and to callers that name no request),
///     never to another request, until release_owner();
///   * matching: the longest strict prefix of a prompt over every entry's live branch and retained checkpoints
///     (best / probe), or the live branch that IS a given branch (best_exact); among equal lengths the newest
///     entry wins, and within an entry its live branch before its checkpoints.
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
    size_t bytes() const { return parked_ + kept_.bytes(); }
    size_t size() const { return shelf_.size(); }
    size_t slots() const { return slots_; }
    size_t budget() const { return budget_; }
    size_t evictions() const { return evictions_; }
    uint64_t clock() const { return clock_; }
    uint64_t use(size_t index) const { return shelf_.at(index).last_use; }

    /// Keep the K/V a mount just restored (all of it valid for `tokens` tokens) for an incremental re-park, if it
    /// fits beside the parked entries; nothing is evicted for it.
    void retain(std::vector<ConversationKv>&& kv, int64_t tokens) {
        kept_ = {};
        ConversationKvReuse offer{std::move(kv), tokens, tokens};
        if (enabled() && offer.bytes() <= budget_ - parked_) kept_ = std::move(offer);
    }
    /// The session was rewritten from token `first_dirty` on: the retained K/V is valid only before it.
    void limit_reuse(int64_t first_dirty) {
        kept_.unchanged_tokens = std::min(kept_.unchanged_tokens, first_dirty);
        if (kept_.unchanged_tokens <= 0) kept_ = {};
    }
    ConversationKvReuse take_reuse() { return std::exchange(kept_, {}); }
    size_t retained_bytes() const { return kept_.bytes(); }

    /// `incoming` bytes could be parked beside `held` bytes (an image taken out and still alive) without evicting.
    bool can_fit(size_t incoming, size_t held = 0) const {
        const std::optional<size_t> room = headroom(incoming, held);
        return room && shelf_.size() < slots_ && bytes() <= *room;
    }

    /// The position of the smallest stamp among `n`, the earlier position on a tie; 0 when n is 0.
    static size_t lru_victim(const uint64_t* stamps, size_t n) {
        return (size_t) (std::min_element(stamps, stamps + n) - stamps);
    }

    /// The longest reusable prefix of `prompt` among the entries offered to `requester`; a hit counts as a use.
    template <class Token>
    Match best(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
               int64_t requester = kNoOwner) {
        const Match m = longest_prefix(prompt, images, cvec, requester);
        if (m.tokens > 0) touch(m.index);
        return m;
    }

    /// best() without counting the hit as a use.
    template <class Token>
    Match probe(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
                int64_t requester = kNoOwner) const {
        return longest_prefix(prompt, images, cvec, requester);
    }

    /// The parked live branch that is exactly `branch` (a hand-back to the slot that parked it); a hit is a use.
    template <class Token>
    Match best_exact(const std::vector<Token>& branch, const std::vector<ConversationImageKey>& images, bool cvec,
                     int64_t requester = kNoOwner) {
        Match m;
        for_each_offered(cvec, requester, [&](size_t i, const SavedConversation& e) {
            keep_longer(m, i, conversation_same_branch(e.live, branch, images), true);
        });
        if (m.tokens > 0) touch(m.index);
        return m;
    }

    void touch(size_t index) { shelf_.at(index).last_use = ++clock_; }

    /// Entry `index` belongs to a request other than `requester` (requests that name none see every entry).
    bool claimed_by_other(size_t index, int64_t requester) const {
        const int64_t holder = shelf_.at(index).image.owner;
        return holder != kNoOwner && requester != kNoOwner && holder != requester;
    }
    void release_owner(int64_t id) {
        for (Parked& p : shelf_)
            if (p.image.owner == id) p.image.owner = kNoOwner;
    }
    int64_t owner(size_t index) const { return shelf_.at(index).image.owner; }

    /// Hand entry `index` out for a mount; the clock moves on so that the next park is the newest entry.
    SavedConversation take(size_t index) {
        Parked p = std::move(shelf_.at(index));
        shelf_.erase(shelf_.begin() + (std::ptrdiff_t) index);
        parked_ -= p.bytes;
        ++clock_;
        return std::move(p.image);
    }

    /// Evict (the retained K/V first, then entries in eviction order) until `incoming` bytes fit beside `held` and a
    /// slot is free.  False, with nothing evicted, when `incoming` and `held` alone exceed the budget.
    bool make_room(size_t incoming, size_t held = 0) {
        const std::optional<size_t> room = headroom(incoming, held);
        if (!room) return false;
        if (bytes() > *room) kept_ = {};
        while (!shelf_.empty() && (shelf_.size() >= slots_ || parked_ > *room)) {
            const size_t v = victim_to_prune();
            parked_ -= shelf_[v].bytes;
            shelf_.erase(shelf_.begin() + (std::ptrdiff_t) v);
            ++evictions_;
        }
        return true;
    }

    /// The entry eviction takes next: unclaimed before claimed, then the least recently used, then the oldest park.
    size_t victim_to_prune() const {
        const auto order = [](const Parked& p) { return std::make_pair(p.image.owner != kNoOwner, p.last_use); };
        const auto it = std::min_element(shelf_.begin(), shelf_.end(),
                                          [&](const Parked& a, const Parked& b) { return order(a) < order(b); });
        return (size_t) (it - shelf_.begin());
    }

    /// Park `image` for `owner` (kNoOwner: anyone may take it), evicting as needed.  False when it cannot fit.
    bool put(SavedConversation&& image, int64_t owner = kNoOwner, size_t held = 0) {
        const size_t n = image.bytes();
        if (!make_room(n, held)) return false;
        image.owner = owner;
        shelf_.push_back(Parked{std::move(image), n, ++clock_});
        parked_ += n;
        return true;
    }

private:
    struct Parked {
        SavedConversation image;
        size_t bytes = 0;        ///< image.bytes() when it was parked
        uint64_t last_use = 0;   ///< the clock tick of its park or its latest use
    };

    /// Budget left once `held` and `incoming` are set aside, or nothing when the cache is off or they exceed it.
    std::optional<size_t> headroom(size_t incoming, size_t held) const {
        if (!enabled() || held > budget_ || incoming > budget_ - held) return std::nullopt;
        return budget_ - held - incoming;
    }

    /// fn(index, image) for every entry offered to `requester` under conditioning `cvec`, newest park first.
    template <class Fn>
    void for_each_offered(bool cvec, int64_t requester, Fn&& fn) const {
        for (size_t i = shelf_.size(); i-- > 0;)
            if (shelf_[i].image.cvec == cvec && !claimed_by_other(i, requester)) fn(i, shelf_[i].image);
    }
    /// A candidate replaces the match only when it is strictly longer, so the first of equal lengths stays.
    static void keep_longer(Match& m, size_t index, int64_t tokens, bool live) {
        if (tokens > m.tokens) m = Match{index, tokens, live};
    }

    template <class Token>
    Match longest_prefix(const std::vector<Token>& prompt, const std::vector<ConversationImageKey>& images, bool cvec,
                         int64_t requester) const {
        Match m;
        for_each_offered(cvec, requester, [&](size_t i, const SavedConversation& e) {
            keep_longer(m, i, conversation_prefix(e.live, prompt, images), true);
            for (const ConversationCheckpoint& c : e.checkpoints) keep_longer(m, i, conversation_prefix(c, prompt, images), false);
        });
        return m;
    }

    size_t budget_ = 0, slots_ = 0, parked_ = 0, evictions_ = 0;
    uint64_t clock_ = 0;
    std::vector<Parked> shelf_;   // park order, oldest first
    ConversationKvReuse kept_;    // the K/V of the last mount, for an incremental re-park
};

}  // namespace strata::core
