// include/strata_kv/handoff.hpp - the hand-off table: a tmpfs arena of payload slots shared by the split roles.
//
// Interface and on-disk format of the reference's include/strata/core/handoff.hpp (the S4.3.2 arena; its own
// test program runs unchanged against this implementation).  A prefill instance owns one arena file
//
//     <handoff-dir>/<pack16>-<split-spec>/<instance>/arena
//     arena := header(4096) + for each tier i: slot_count[i] x ( slot_header(4096) + slot_bytes[i] )
//
// and a decode instance maps it read-only.  A slot moves FREE -> CLAIMED (claim, under the arena's flock) ->
// READY (payload written with no lock held; then one 48-byte pwrite of the metadata block [96,144), a release
// fence, and one 8-byte pwrite of state+flags at offset 24 - that store is the publish point) -> FREE (the
// reader's ACK).  Dead or recycled owners (pid + /proc start time), expired leases and readers known to be gone
// are reclaimed and flagged abandoned.  A second live writer on one arena is refused; an arena whose creator is
// gone is rebuilt.
//
// On B200 the hand-off itself goes device to device (NVLink pull/push, include/strata_kv.h); this table is the
// control-plane format the split roles agree on, and the path for payloads that leave the node's GPUs.
#pragma once

#include "strata_kv/fnv.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace strata::core {

// ---- constants (an ABI) ----
inline constexpr uint64_t kHandoffHeaderBytes = 4096;
inline constexpr uint32_t kHandoffVersion = 1;
inline constexpr int kHandoffMaxTiers = 8;
inline constexpr uint64_t kHandoffSlackBytes = 64ull << 20;     ///< per-slot room over the priced payload
inline constexpr uint64_t kHandoffDefaultLeaseMs = 300000ull;   ///< STRATA_HANDOFF_LEASE_MS overrides it

enum HandoffSlotState : uint32_t { kHandoffFree = 0, kHandoffClaimed = 1, kHandoffReady = 2 };
enum HandoffSlotFlags : uint32_t { kHandoffFlagCancelled = 1u, kHandoffFlagAbandoned = 2u, kHandoffFlagPartial = 4u };

// arena header offsets
inline constexpr uint64_t kArenaMagicOffset = 0;
inline constexpr uint64_t kArenaVersionOffset = 16;
inline constexpr uint64_t kArenaHeaderBytesOffset = 20;
inline constexpr uint64_t kArenaTierCountOffset = 24;
inline constexpr uint64_t kArenaSlotTotalOffset = 32;
inline constexpr uint64_t kArenaBytesOffset = 40;
inline constexpr uint64_t kArenaPackHashOffset = 48;
inline constexpr uint64_t kArenaGeomHashOffset = 56;
inline constexpr uint64_t kArenaCreatedPidOffset = 64;
inline constexpr uint64_t kArenaCreatedStartOffset = 72;
inline constexpr uint64_t kArenaTierMaxTokensOffset = 80;
inline constexpr uint64_t kArenaTierSlotCountOffset = 144;
inline constexpr uint64_t kArenaTierSlotBytesOffset = 208;
inline constexpr uint64_t kArenaTierSlotOffOffset = 272;
inline constexpr uint64_t kArenaReservedOffset = 336;

// slot header offsets
inline constexpr uint64_t kSlotMagicOffset = 0;
inline constexpr uint64_t kSlotVersionOffset = 16;
inline constexpr uint64_t kSlotHeaderBytesOffset = 20;
inline constexpr uint64_t kSlotStateOffset = 24;
inline constexpr uint64_t kSlotFlagsOffset = 28;
inline constexpr uint64_t kSlotTierOffset = 32;
inline constexpr uint64_t kSlotOwnerOffset = 40;
inline constexpr uint64_t kSlotOwnerStartOffset = 48;
inline constexpr uint64_t kSlotNonceOffset = 56;
inline constexpr uint64_t kSlotClientOffset = 64;
inline constexpr uint64_t kSlotRequestOffset = 72;
inline constexpr uint64_t kSlotPackHashOffset = 80;
inline constexpr uint64_t kSlotGeomHashOffset = 88;
inline constexpr uint64_t kSlotTokensOffset = 96;
inline constexpr uint64_t kSlotPayloadBytesOffset = 104;
inline constexpr uint64_t kSlotPayloadHashOffset = 112;
inline constexpr uint64_t kSlotClaimedMsOffset = 120;
inline constexpr uint64_t kSlotPublishedMsOffset = 128;
inline constexpr uint64_t kSlotSeqOffset = 136;
inline constexpr uint64_t kSlotReservedOffset = 144;
inline constexpr uint64_t kSlotPublishBlockOffset = 96;    ///< tokens .. seq, written before the publish point
inline constexpr uint64_t kSlotPublishBlockBytes = 48;
inline constexpr uint64_t kSlotPublishStateBytes = 8;      ///< state + flags: the publish point

struct HandoffArenaHeader {
    char magic[16];   // "STRATA-HARENA-V1"
    uint32_t version;
    uint32_t header_bytes;
    uint32_t tier_count;
    uint32_t pad;
    uint64_t slot_total;
    uint64_t arena_bytes;
    uint64_t pack_hash;
    uint64_t geom_hash;
    uint64_t created_pid;
    uint64_t created_start;
    uint64_t tier_max_tokens[kHandoffMaxTiers];
    uint64_t tier_slot_count[kHandoffMaxTiers];
    uint64_t tier_slot_bytes[kHandoffMaxTiers];
    uint64_t tier_slot_off[kHandoffMaxTiers];
    uint64_t reserved[kHandoffMaxTiers];
};
static_assert(sizeof(HandoffArenaHeader) <= kHandoffHeaderBytes);
static_assert(offsetof(HandoffArenaHeader, version) == kArenaVersionOffset);
static_assert(offsetof(HandoffArenaHeader, tier_count) == kArenaTierCountOffset);
static_assert(offsetof(HandoffArenaHeader, slot_total) == kArenaSlotTotalOffset);
static_assert(offsetof(HandoffArenaHeader, arena_bytes) == kArenaBytesOffset);
static_assert(offsetof(HandoffArenaHeader, pack_hash) == kArenaPackHashOffset);
static_assert(offsetof(HandoffArenaHeader, created_pid) == kArenaCreatedPidOffset);
static_assert(offsetof(HandoffArenaHeader, tier_max_tokens) == kArenaTierMaxTokensOffset);
static_assert(offsetof(HandoffArenaHeader, tier_slot_count) == kArenaTierSlotCountOffset);
static_assert(offsetof(HandoffArenaHeader, tier_slot_bytes) == kArenaTierSlotBytesOffset);
static_assert(offsetof(HandoffArenaHeader, tier_slot_off) == kArenaTierSlotOffOffset);
static_assert(offsetof(HandoffArenaHeader, reserved) == kArenaReservedOffset);

struct HandoffSlotHeader {
    char magic[16];   // "STRATA-HSLOT-V1"
    uint32_t version;
    uint32_t header_bytes;
    uint32_t state;
    uint32_t flags;
    uint32_t tier;
    uint32_t pad;
    uint64_t owner_pid;
    uint64_t owner_start;
    uint64_t nonce;
    uint64_t client_id;
    uint64_t request_id;
    uint64_t pack_hash;
    uint64_t geom_hash;
    uint64_t tokens;
    uint64_t payload_bytes;
    uint64_t payload_hash;
    uint64_t claimed_ms;
    uint64_t published_ms;
    uint64_t seq;
    uint64_t reserved[7];
};
static_assert(sizeof(HandoffSlotHeader) <= kHandoffHeaderBytes);
static_assert(offsetof(HandoffSlotHeader, state) == kSlotStateOffset);
static_assert(offsetof(HandoffSlotHeader, flags) == kSlotFlagsOffset);
static_assert(offsetof(HandoffSlotHeader, owner_pid) == kSlotOwnerOffset);
static_assert(offsetof(HandoffSlotHeader, nonce) == kSlotNonceOffset);
static_assert(offsetof(HandoffSlotHeader, pack_hash) == kSlotPackHashOffset);
static_assert(offsetof(HandoffSlotHeader, tokens) == kSlotTokensOffset);
static_assert(offsetof(HandoffSlotHeader, payload_hash) == kSlotPayloadHashOffset);
static_assert(offsetof(HandoffSlotHeader, seq) == kSlotSeqOffset);
static_assert(offsetof(HandoffSlotHeader, reserved) == kSlotReservedOffset);
static_assert(kSlotPublishBlockOffset + kSlotPublishBlockBytes == kSlotReservedOffset);

// ---- identity ----
struct HandoffSplitStage {
    int64_t layer_lo = 0;
    int64_t layer_hi = 0;
};
struct HandoffSplit {
    int64_t main_lo = 0;
    int64_t main_hi = 0;
    std::vector<HandoffSplitStage> stages;   ///< later stages only, engine order; empty = no split
    bool draft_on_last = true;               ///< the drafter binds to the last stage
};
/// The canonical, path-safe spelling of a split (carves, stage count, where the draft lives).
std::string handoff_split_spec(const HandoffSplit& split);
/// FNV-1a over the 18-entry geometry key and the split spec: two instances that must not mount each other's
/// payloads differ here.
uint64_t handoff_geom_hash(const std::array<int64_t, 18>& geometry, const std::string& split_spec);
/// <handoff-dir>/<pack16>-<split-spec>/<instance>/arena
std::string handoff_arena_path(const std::string& handoff_dir, uint64_t pack_hash, const std::string& split_spec,
                               const std::string& instance);
inline uint64_t handoff_round_up_64(uint64_t n) { return (n + 63ull) & ~63ull; }

// ---- sizing ----
struct HandoffTierSpec {
    uint64_t max_tokens = 0;
    uint64_t slot_count = 0;
};
struct HandoffSizing {
    std::vector<HandoffTierSpec> tiers;
    std::vector<uint64_t> payload_bytes;   ///< as priced
    std::vector<uint64_t> slot_bytes;      ///< round_up_64(payload) + slack
    std::vector<uint64_t> slot_off;        ///< file offset of tier i's first slot
    uint64_t slot_total = 0;
    uint64_t arena_bytes = 0;
    uint64_t max_tokens = 0;
    std::string describe;
};
/// pricer(tier_tokens, payload_bytes, err): the engine's own byte estimate for a tier (host arithmetic).
using HandoffPricer = std::function<bool(uint64_t tier_tokens, uint64_t& payload_bytes, std::string& err)>;
bool handoff_size_arena(const std::vector<HandoffTierSpec>& tiers, const HandoffPricer& pricer, HandoffSizing& out,
                        std::string& err);
bool handoff_size_arena(const std::vector<HandoffTierSpec>& tiers, const std::vector<uint64_t>& payload_bytes,
                        HandoffSizing& out, std::string& err);

// ---- slots as seen by callers ----
struct HandoffSlotInfo {
    int index = -1;
    uint64_t base = 0, capacity = 0;
    uint32_t state = kHandoffFree, flags = 0, tier = 0;
    uint64_t owner_pid = 0, owner_start = 0, nonce = 0;
    uint64_t client_id = 0, request_id = 0;
    uint64_t pack_hash = 0, geom_hash = 0;
    uint64_t tokens = 0, payload_bytes = 0, payload_hash = 0;
    uint64_t claimed_ms = 0, published_ms = 0, seq = 0;
};
struct HandoffClaim {
    int index = -1;
    uint64_t base = 0, payload_off = 0, capacity = 0;
    uint32_t tier = 0;   ///< the group actually used (a job may land in a larger one)
    uint64_t nonce = 0;
};
struct HandoffReclaim {
    int index = -1;
    uint32_t was_state = 0, flags = 0;
    uint64_t owner_pid = 0, client_id = 0, nonce = 0, payload_bytes = 0;
    uint64_t age_ms = 0;
    std::string why;
};
/// A published payload mapped read-only; unmaps itself.
struct HandoffPayload {
    const uint8_t* data = nullptr;
    uint64_t bytes = 0;
    int index = -1;
    uint32_t tier = 0;
    uint64_t nonce = 0, client_id = 0, request_id = 0;
    uint64_t tokens = 0, payload_bytes = 0, payload_hash = 0, seq = 0;

    HandoffPayload() = default;
    ~HandoffPayload();
    HandoffPayload(const HandoffPayload&) = delete;
    HandoffPayload& operator=(const HandoffPayload&) = delete;
    HandoffPayload(HandoffPayload&& o) noexcept;
    HandoffPayload& operator=(HandoffPayload&& o) noexcept;
    bool valid() const { return data != nullptr; }
    void bind_mapping(void* map, uint64_t map_bytes, const uint8_t* data, uint64_t payload_bytes);
    void unbind();

private:
    void* map_ = nullptr;
    uint64_t map_bytes_ = 0;
};

class HandoffArena {
public:
    HandoffArena();
    ~HandoffArena();
    HandoffArena(const HandoffArena&) = delete;
    HandoffArena& operator=(const HandoffArena&) = delete;
    HandoffArena(HandoffArena&& o) noexcept;
    HandoffArena& operator=(HandoffArena&& o) noexcept;

    // writer (the prefill instance)
    bool open_writer(const std::string& path, const HandoffSizing& sizing, uint64_t pack_hash, uint64_t geom_hash,
                     std::string& err, bool allow_existing_writer = false);
    void set_lease_ms(uint64_t ms) { lease_ms_ = ms; }
    uint64_t lease_ms() const { return lease_ms_; }
    void note_client_pid(uint64_t client_id, uint64_t pid);
    std::vector<HandoffReclaim> reclaim(std::string* err = nullptr);
    bool claim(uint32_t tier, uint64_t client_id, uint64_t request_id, HandoffClaim& out, std::string& err);
    bool write_payload(const HandoffClaim& c, uint64_t offset, const void* data, uint64_t bytes, std::string& err);
    bool publish(const HandoffClaim& c, uint64_t tokens, uint64_t payload_bytes, uint64_t payload_hash,
                 std::string& err);
    bool release(int index, uint64_t nonce, std::string& err);
    bool abort_claim(int index, uint64_t nonce, std::string& err);
    bool cancel(int index, uint64_t nonce, std::string& err);

    // reader (a decode instance)
    bool open_reader(const std::string& path, uint64_t pack_hash, uint64_t geom_hash, std::string& err);
    bool read_slot(int index, uint64_t expect_nonce, uint64_t client_id, HandoffPayload& out, std::string& err);
    static uint64_t payload_hash_of(const HandoffPayload& p);

    // either side
    bool valid() const { return fd_ >= 0; }
    bool is_writer() const { return writer_; }
    const std::string& path() const { return path_; }
    const HandoffArenaHeader& header() const { return hdr_; }
    uint64_t arena_bytes() const { return hdr_.arena_bytes; }
    uint64_t slot_total() const { return hdr_.slot_total; }
    uint32_t tier_count() const { return hdr_.tier_count; }
    uint64_t tier_max_tokens(uint32_t tier) const;
    uint64_t tier_slot_bytes(uint32_t tier) const;
    uint64_t tier_slot_count(uint32_t tier) const;
    uint64_t tier_slot_off(uint32_t tier) const;
    uint64_t max_tokens() const { return hdr_.tier_count == 0 ? 0 : hdr_.tier_max_tokens[hdr_.tier_count - 1]; }
    std::string describe() const;
    bool slot_info(int index, HandoffSlotInfo& out) const;
    std::string free_slots(std::string* err = nullptr) const;

private:
    struct Locked;   // flock + process mutex, released on scope exit
    void close_();
    bool locate_(int index, uint64_t& base, uint32_t& tier, uint64_t& capacity) const;
    bool load_slot_(int index, HandoffSlotHeader& h, uint64_t& base, uint64_t& capacity) const;
    bool store_(uint64_t off, const void* p, uint64_t n) const;
    bool reset_slot_(uint64_t base, uint32_t tier, uint32_t flags) const;
    std::vector<HandoffReclaim> reclaim_locked_(std::string* err);
    std::string free_slots_locked_() const;

    int fd_ = -1;
    bool writer_ = false;
    std::string path_;
    HandoffArenaHeader hdr_{};
    uint64_t lease_ms_ = kHandoffDefaultLeaseMs;
    std::vector<std::pair<uint64_t, uint64_t>> client_pids_;
    mutable std::mutex mu_;
};

bool handoff_pid_alive(uint64_t pid);
/// Field 22 of /proc/<pid>/stat (clock ticks since boot); 0 when unknown.
uint64_t handoff_proc_start_time(uint64_t pid);
/// Alive and (when `start_time` is known) the same process that recorded it; an unknown start counts as alive.
bool handoff_claim_alive(uint64_t pid, uint64_t start_time);
uint64_t handoff_now_ms();

}  // namespace strata::core
