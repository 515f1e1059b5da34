// include/strata_kv/conversation_wire.hpp - the SR4H hand-off payload codec.
//
// Format-identical to the reference's codec (include/strata/core/conversation_wire.hpp:24-81): a payload written
// by either decodes with the other, and encode(decode(x)) == x byte for byte.  The format, in short:
//
//     payload := header_record(256) body_records zero_pad(to 64) blob_pool
//     records := KV[n_kv] CHECKPOINT(live) CHECKPOINT[n_checkpoints] STAGE[n_stage_parts] END!
//     record  := {u32 kind; u32 flags = 0; u64 body_bytes} body          (little-endian throughout)
//     KV body (136 B) := i32 format, i32 0, i64 cells heads head_dim page_size pooled_rows idx_dim, BLOBREF x5
//     CHECKPOINT body := i64 n_ids, i32 ids[], pad to 8, i64 n_imgs, {i64 start, u64 hash}[], BLOBREF x5
//                        (gdn ple tails dead block_pos), u64 used, i64 n_parts, CHECKPOINT[n_parts]
//     STAGE body      := i64 layer_lo, i64 layer_hi, CHECKPOINT, i64 n_kv, KV[n_kv]
//     BLOBREF := {u64 bytes, u64 offset from the payload start}; an empty buffer is {0, 0}; every blob starts
//                on a 64-byte boundary of the pool in emission order, gaps are zero.
//
// The header's payload_hash field is always zero: the FNV-1a of the payload as written travels out of band
// (arena slot header, DONE line) and is returned by the encoder.  `owner` never travels (a received image is
// unclaimed).  A decode builds into a local image and only moves it into the caller's on success.
//
// B200 addition: conversation_wire_pack_device (conversation_wire_device.hpp) emits the same payload straight
// from device K/V pools, the blob pool gathered by one copy kernel.
#pragma once

#include "strata_kv/conversation_cache.hpp"
#include "strata_kv/fnv.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace strata::core {

// ---- the format constants (an ABI: these values are the wire format) ----
inline constexpr uint32_t kWireMagic = 0x48345253u;          // 'S','R','4','H'
inline constexpr uint16_t kWireFormatVersion = 1;
inline constexpr uint64_t kWireHeaderSpecBytes = 232;        // the specified field list
inline constexpr uint64_t kWireHeaderRecordBytes = 256;      // the header record, padded
inline constexpr uint64_t kWireRecordHeaderBytes = 16;
inline constexpr uint64_t kWireBlobAlign = 64;
inline constexpr uint64_t kWireHashSeed = 1469598103934665603ull;   // FNV-1a 64 offset basis
inline constexpr uint64_t kWireChunkBytes = 1ull << 20;      // the largest single read or vector write
inline constexpr int kWireMaxCheckpointDepth = 8;
inline constexpr int64_t kWireMaxKvRecords = 4096;
inline constexpr int64_t kWireMaxCheckpoints = 1 << 20;
inline constexpr int64_t kWireMaxStageParts = 64;
inline constexpr int64_t kWireMaxImages = 1 << 16;

enum WireRecordKind : uint32_t {
    kWireRecordKv = 1,
    kWireRecordCheckpoint = 2,
    kWireRecordStage = 3,
    kWireRecordEnd = 0x21444E45u,   // the bytes 'E','N','D','!'
};

enum WireHeaderFlags : uint16_t {
    kWireFlagCvec = 1u,
    kWireFlagHasStageParts = 2u,
    kWireFlagPartial = 4u,          // never valid in a complete payload
    kWireFlagKnown = kWireFlagCvec | kWireFlagHasStageParts | kWireFlagPartial,
};

/// The 256-byte header record exactly as it lies at payload offset 0.
struct WireHeaderRecord {
    uint32_t magic;
    uint16_t fmt_version;
    uint16_t flags;
    uint64_t geometry[18];
    uint64_t layer_lo;
    uint64_t layer_hi;
    int64_t n_kv;
    int64_t n_checkpoints;
    int64_t n_stage_parts;
    int64_t live_tokens;
    uint64_t blob_pool_off;
    uint64_t blob_pool_bytes;
    uint64_t geom_hash;
    uint64_t pack_hash;
    uint64_t payload_bytes;   // the whole payload, header and pool included
    uint64_t payload_hash;    // always 0 on the wire
    uint64_t reserved;        // 0
};
static_assert(sizeof(WireHeaderRecord) == kWireHeaderRecordBytes);
static_assert(offsetof(WireHeaderRecord, geometry) == 8);
static_assert(offsetof(WireHeaderRecord, layer_lo) == 152);
static_assert(offsetof(WireHeaderRecord, n_kv) == 168);
static_assert(offsetof(WireHeaderRecord, live_tokens) == 192);
static_assert(offsetof(WireHeaderRecord, blob_pool_off) == 200);
static_assert(offsetof(WireHeaderRecord, geom_hash) == 216);
static_assert(offsetof(WireHeaderRecord, payload_bytes) == 232);
static_assert(offsetof(WireHeaderRecord, reserved) == 248);
static_assert(offsetof(WireHeaderRecord, reserved) + 8 - 24 == kWireHeaderSpecBytes);

// ---- sinks ----
/// Receives the payload strictly in order, in arbitrary chunks.
class WireSink {
public:
    virtual ~WireSink() = default;
    virtual bool write(const uint8_t* data, size_t bytes) = 0;
    /// Why it refused (appended to the codec's own message).
    virtual std::string refusal() const { return {}; }
};

class VectorWireSink final : public WireSink {
public:
    explicit VectorWireSink(size_t reserve_bytes = 0) { bytes_.reserve(reserve_bytes); }
    bool write(const uint8_t* data, size_t bytes) override;
    const std::vector<uint8_t>& data() const { return bytes_; }
    std::vector<uint8_t>& data() { return bytes_; }

private:
    std::vector<uint8_t> bytes_;
};

/// Into a hand-off slot: `pwrite` at `offset` of `fd`, or a mapped region when built from a pointer.
class SlotWireSink final : public WireSink {
public:
    SlotWireSink(int fd, uint64_t offset, uint64_t capacity);
    SlotWireSink(uint8_t* mapping, uint64_t capacity);
    bool write(const uint8_t* data, size_t bytes) override;
    std::string refusal() const override { return error_; }
    uint64_t written() const { return pos_; }
    const std::string& error() const { return error_; }

private:
    int fd_ = -1;
    uint64_t at_ = 0;
    uint8_t* map_ = nullptr;
    uint64_t pos_ = 0, capacity_ = 0;
    std::string error_;
};

// ---- sources ----
class WireSource {
public:
    virtual ~WireSource() = default;
    virtual uint64_t size() const = 0;
    /// Fill [offset, offset + bytes); false rather than a short read.
    virtual bool read(uint8_t* dst, uint64_t offset, size_t bytes) const = 0;
    /// A pointer to the run when the source holds it contiguously (no copy), else null.
    virtual const uint8_t* span(uint64_t /*offset*/, size_t /*bytes*/) const { return nullptr; }
};

class SpanWireSource final : public WireSource {
public:
    SpanWireSource(const uint8_t* data, uint64_t bytes) : p_(data), n_(bytes) {}
    uint64_t size() const override { return n_; }
    bool read(uint8_t* dst, uint64_t offset, size_t bytes) const override;
    const uint8_t* span(uint64_t offset, size_t bytes) const override;

private:
    const uint8_t* p_ = nullptr;
    uint64_t n_ = 0;
};

class FileWireSource final : public WireSource {
public:
    FileWireSource(int fd, uint64_t offset, uint64_t bytes) : fd_(fd), at_(offset), n_(bytes) {}
    uint64_t size() const override { return n_; }
    bool read(uint8_t* dst, uint64_t offset, size_t bytes) const override;

private:
    int fd_ = -1;
    uint64_t at_ = 0;
    uint64_t n_ = 0;
};

// ---- encode ----
struct WireIdentity {
    uint64_t geom_hash = 0;
    uint64_t pack_hash = 0;
};

struct WirePlan {
    uint64_t body_bytes = 0;       ///< the record stream, header excluded
    uint64_t blob_pool_off = 0;
    uint64_t blob_pool_bytes = 0;
    uint64_t total_bytes = 0;
    int64_t n_kv = 0, n_checkpoints = 0, n_stage_parts = 0, live_tokens = 0;
    uint16_t flags = 0;
    size_t blobs = 0;
};

struct WireEncoded {
    uint64_t bytes = 0;
    uint64_t payload_hash = 0;     ///< FNV-1a over the payload as written
    uint64_t blob_pool_bytes = 0;
    size_t blobs = 0;
};

bool conversation_wire_plan(const SavedConversation& image, WirePlan& plan, std::string& error);
bool conversation_wire_plan(const SavedConversation& image, int max_checkpoint_depth, WirePlan& plan,
                            std::string& error);
bool conversation_wire_encode(const SavedConversation& image, WireSink& sink, const WireIdentity& identity,
                              WireEncoded& out, std::string& error);
bool conversation_wire_encode(const SavedConversation& image, WireSink& sink, const WireIdentity& identity,
                              int max_checkpoint_depth, WirePlan& plan, WireEncoded& out, std::string& error);

// ---- decode ----
struct WireExpect {
    std::array<int64_t, 18> geometry{};
    bool check_geometry = false;
    uint64_t geom_hash = 0, pack_hash = 0;
    bool check_hashes = false;
    uint64_t payload_hash = 0;
    bool check_payload_hash = false;
    int64_t stage_parts = -1;          ///< -1: no check
    uint64_t max_payload_bytes = 0;    ///< 0: no bound
    int max_checkpoint_depth = kWireMaxCheckpointDepth;
};

struct WireDecoded {
    uint64_t bytes = 0;
    uint64_t payload_hash = 0;
    uint64_t geom_hash = 0, pack_hash = 0;
    std::array<int64_t, 18> geometry{};
    int64_t layer_lo = 0, layer_hi = 0;
    int64_t n_kv = 0, n_checkpoints = 0, n_stage_parts = 0, live_tokens = 0;
    uint16_t flags = 0;
    bool cvec = true;
    uint64_t blob_pool_off = 0, blob_pool_bytes = 0;
    size_t blobs = 0;
};

bool conversation_wire_decode(const WireSource& source, SavedConversation& image, WireDecoded& info,
                              const WireExpect& expect, std::string& error);
bool conversation_wire_decode(const uint8_t* data, uint64_t bytes, SavedConversation& image, WireDecoded& info,
                              const WireExpect& expect, std::string& error);
bool conversation_wire_peek(const uint8_t* data, uint64_t bytes, WireHeaderRecord& header, std::string& error);
uint64_t conversation_wire_payload_hash(const uint8_t* data, uint64_t bytes);
std::string conversation_wire_describe(const WireHeaderRecord& header);

}  // namespace strata::core
