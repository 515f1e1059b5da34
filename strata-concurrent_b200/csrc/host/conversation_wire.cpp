// conversation_wire.cpp - the SR4H payload codec (include/strata_kv/conversation_wire.hpp).
//
// Encode: one traversal of the image in record order drives both passes - the plan pass assigns every
// non-empty buffer its pool offset, the write pass emits the same records with those offsets - so the blob order
// can never differ between the two.  The FNV-1a content hash is folded in as the bytes leave.
// Decode: header checks first (nothing is read past them), then the records with every count bounded by the
// bytes that actually remain, then the blobs are copied into a fresh image that replaces the caller's only on
// success.
#include "strata_kv/conversation_wire.hpp"
#include "wire_detail.hpp"

#include <algorithm>
#include <bit>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>

#include <unistd.h>

namespace strata::core {

uint64_t fnv1a64(const uint8_t* p, uint64_t n, uint64_t seed) {
    uint64_t h = seed;
    for (uint64_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

uint64_t conversation_wire_payload_hash(const uint8_t* data, uint64_t bytes) { return fnv1a64(data, bytes); }

namespace {

constexpr uint64_t kKvBody = 136;

bool refuse(std::string& error, const std::string& why) {
    error = "conversation wire: " + why;
    return false;
}
std::string hex16(uint64_t v) {
    char b[20];
    std::snprintf(b, sizeof b, "%016llx", (unsigned long long) v);
    return b;
}
std::string num(uint64_t v) { return std::to_string(v); }
uint64_t align64(uint64_t n) { return (n + 63) & ~uint64_t(63); }
bool add_to(uint64_t& total, uint64_t n) {
    if (n > std::numeric_limits<uint64_t>::max() - total) return false;
    total += n;
    return true;
}

void le16(uint8_t* p, uint16_t v) { p[0] = (uint8_t) v, p[1] = (uint8_t) (v >> 8); }
void le32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t) (v >> (8 * i));
}
void le64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t) (v >> (8 * i));
}
uint16_t rd16(const uint8_t* p) { return (uint16_t) (p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t) p[i] << (8 * i);
    return v;
}
uint64_t rd64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= (uint64_t) p[i] << (8 * i);
    return v;
}

/// A growable little-endian record buffer.
struct Bytes {
    std::vector<uint8_t> b;
    void u32(uint32_t v) {
        const size_t at = b.size();
        b.resize(at + 4);
        le32(b.data() + at, v);
    }
    void u64(uint64_t v) {
        const size_t at = b.size();
        b.resize(at + 8);
        le64(b.data() + at, v);
    }
};

// ------------------------------------------------------------------------------------------------ encode

/// One pool entry: a ConversationBuffer or a contiguous vector.
struct Blob {
    const ConversationBuffer* buf = nullptr;
    const std::vector<uint8_t>* vec = nullptr;
    uint64_t rel = 0, bytes = 0;
};

uint64_t checkpoint_body_bytes(const ConversationCheckpoint& c) {
    const uint64_t ids = (uint64_t) c.ids.size() * 4;
    uint64_t n = 8 + ids + (ids % 8 ? 4 : 0) + 8 + 16 * (uint64_t) c.imgs.size() + 5 * 16 + 8 + 8;
    for (const auto& p : c.stage_parts) n += kWireRecordHeaderBytes + checkpoint_body_bytes(p);
    return n;
}
uint64_t stage_body_bytes(const ConversationStageSnapshot& s) {
    return 16 + kWireRecordHeaderBytes + checkpoint_body_bytes(s.state) + 8 +
           (uint64_t) s.kv.size() * (kWireRecordHeaderBytes + kKvBody);
}

bool depth_ok(const ConversationCheckpoint& c, int depth, int max_depth) {
    if (depth > max_depth) return false;
    for (const auto& p : c.stage_parts)
        if (!depth_ok(p, depth + 1, max_depth)) return false;
    return true;
}

uint64_t own_size(const void*, uint64_t real) { return real; }

/// Walks the image in record order.  `emit(bytes)` gets each record piece; `blob(buffer)` returns the
/// absolute payload offset of a buffer's pool entry (0 for an empty one); `size_of(buffer, its size())` gives
/// the byte count the records carry for it (its own size, or a side table's for a shape image).
class Traversal {
public:
    using Emit = std::function<bool(const uint8_t*, size_t)>;
    using BlobOf = std::function<uint64_t(const ConversationBuffer*, const std::vector<uint8_t>*)>;
    Traversal(Emit emit, BlobOf blob, const wire_detail::SizeOf& size_of = own_size)
        : emit_(std::move(emit)), blob_(std::move(blob)), size_of_(size_of) {}

    bool body(const SavedConversation& s) {
        for (const auto& k : s.kv)
            if (!kv_record(k)) return false;
        if (!checkpoint_record(s.live)) return false;
        for (const auto& c : s.checkpoints)
            if (!checkpoint_record(c)) return false;
        for (const auto& st : s.stage_parts)
            if (!stage_record(st)) return false;
        return record_header(kWireRecordEnd, 0);
    }

private:
    bool out(const Bytes& b) { return emit_(b.b.data(), b.b.size()); }
    bool record_header(uint32_t kind, uint64_t bytes) {
        Bytes h;
        h.u32(kind);
        h.u32(0);
        h.u64(bytes);
        return out(h);
    }
    void ref(Bytes& b, const ConversationBuffer& buf) {
        b.u64(size_of_(&buf, buf.size()));
        b.u64(blob_(&buf, nullptr));
    }
    void ref(Bytes& b, const std::vector<uint8_t>& vec) {
        b.u64(size_of_(&vec, vec.size()));
        b.u64(blob_(nullptr, &vec));
    }
    bool kv_record(const ConversationKv& k) {
        if (!record_header(kWireRecordKv, kKvBody)) return false;
        Bytes b;
        b.u32((uint32_t) k.format);
        b.u32(0);
        for (int64_t v : {k.cells, k.heads, k.head_dim, k.page_size, k.pooled_rows, k.idx_dim}) b.u64((uint64_t) v);
        for (const ConversationBuffer* buf : {&k.k, &k.v, &k.k_scale, &k.v_scale, &k.pooled}) ref(b, *buf);
        return out(b);
    }
    bool checkpoint_record(const ConversationCheckpoint& c) {
        if (!record_header(kWireRecordCheckpoint, checkpoint_body_bytes(c))) return false;
        Bytes b;
        b.u64(c.ids.size());
        if (!out(b)) return false;
        if constexpr (std::endian::native == std::endian::little) {
            // the wire's little-endian int32 ids are the array's own bytes: emitted in place, no per-id work
            if (!c.ids.empty() && !emit_(reinterpret_cast<const uint8_t*>(c.ids.data()), c.ids.size() * 4))
                return false;
        } else {
            Bytes piece;   // ids go out in bounded pieces, each sized once and filled in one pass
            for (size_t i = 0; i < c.ids.size(); i += 4096) {
                const size_t n = std::min<size_t>(4096, c.ids.size() - i);
                piece.b.resize(4 * n);
                for (size_t j = 0; j < n; ++j) le32(piece.b.data() + 4 * j, (uint32_t) c.ids[i + j]);
                if (!out(piece)) return false;
            }
        }
        Bytes tail;
        if ((c.ids.size() * 4) % 8) tail.u32(0);
        tail.u64(c.imgs.size());
        for (const auto& img : c.imgs) {
            tail.u64((uint64_t) img.start);
            tail.u64(img.hash);
        }
        for (const std::vector<uint8_t>* v : {&c.gdn, &c.ple, &c.tails, &c.dead, &c.block_pos}) ref(tail, *v);
        tail.u64(c.used);
        tail.u64(c.stage_parts.size());
        if (!out(tail)) return false;
        for (const auto& p : c.stage_parts)
            if (!checkpoint_record(p)) return false;
        return true;
    }
    bool stage_record(const ConversationStageSnapshot& s) {
        if (!record_header(kWireRecordStage, stage_body_bytes(s))) return false;
        Bytes b;
        b.u64((uint64_t) s.layer_lo);
        b.u64((uint64_t) s.layer_hi);
        if (!out(b)) return false;
        if (!checkpoint_record(s.state)) return false;
        Bytes n;
        n.u64(s.kv.size());
        if (!out(n)) return false;
        for (const auto& k : s.kv)
            if (!kv_record(k)) return false;
        return true;
    }

    Emit emit_;
    BlobOf blob_;
    wire_detail::SizeOf size_of_;
};

struct Planned {
    WirePlan plan;
    std::vector<Blob> blobs;
};

bool plan_image(const SavedConversation& s, int max_depth, Planned& p, std::string& error,
                const wire_detail::SizeOf& size_of = own_size) {
    if (!s.live.stage_parts.empty())
        return refuse(error, "the live checkpoint carries layer-split stage parts; a parked image keeps them in "
                             "SavedConversation::stage_parts (layer-split parking is not supported that way)");
    if (!depth_ok(s.live, 0, max_depth)) return refuse(error, "checkpoint stage_parts are nested past the bound");
    for (const auto& c : s.checkpoints)
        if (!depth_ok(c, 0, max_depth)) return refuse(error, "checkpoint stage_parts are nested past the bound");
    for (const auto& st : s.stage_parts)
        if (!depth_ok(st.state, 0, max_depth)) return refuse(error, "checkpoint stage_parts are nested past the bound");
    p = Planned{};
    uint64_t body = 0, pool = 0;
    bool overflow = false;
    Traversal walk(
        [&](const uint8_t*, size_t n) {
            overflow |= !add_to(body, n);
            return true;
        },
        [&](const ConversationBuffer* buf, const std::vector<uint8_t>* vec) -> uint64_t {
            const uint64_t n = buf ? size_of(buf, buf->size()) : size_of(vec, vec->size());
            if (!n) return 0;
            const uint64_t rel = align64(pool);
            Blob b{buf, vec, rel, n};
            p.blobs.push_back(b);
            pool = rel;
            overflow |= !add_to(pool, n);
            return 0;
        },
        size_of);
    walk.body(s);
    if (overflow) return refuse(error, "byte count overflow");
    WirePlan& w = p.plan;
    w.body_bytes = body;
    w.blob_pool_off = align64(kWireHeaderRecordBytes + body);
    w.blob_pool_bytes = p.blobs.empty() ? 0 : align64(pool);
    w.total_bytes = w.blob_pool_off + w.blob_pool_bytes;
    w.n_kv = (int64_t) s.kv.size();
    w.n_checkpoints = (int64_t) s.checkpoints.size();
    w.n_stage_parts = (int64_t) s.stage_parts.size();
    w.live_tokens = (int64_t) s.live.ids.size();
    w.flags = (uint16_t) ((s.cvec ? kWireFlagCvec : 0) | (s.stage_parts.empty() ? 0 : kWireFlagHasStageParts));
    w.blobs = p.blobs.size();
    return true;
}

/// Forwards to the sink, hashing and counting; keeps the sink's refusal reason.
class HashedOut {
public:
    HashedOut(WireSink& sink, std::string& error) : sink_(sink), error_(error) {}
    bool operator()(const uint8_t* p, size_t n) {
        if (!n) return true;
        if (!sink_.write(p, n)) {
            std::string why = "the sink refused the payload at byte " + num(pos_);
            const std::string r = sink_.refusal();
            if (!r.empty()) why += ": " + r;
            refuse(error_, why);
            return false;
        }
        hash_ = fnv1a64(p, n, hash_);
        pos_ += n;
        return true;
    }
    uint64_t hash() const { return hash_; }
    uint64_t pos() const { return pos_; }

private:
    WireSink& sink_;
    std::string& error_;
    uint64_t hash_ = kWireHashSeed;
    uint64_t pos_ = 0;
};

void header_bytes(const SavedConversation& s, const WirePlan& w, const WireIdentity& id, uint8_t* h) {
    std::memset(h, 0, kWireHeaderRecordBytes);
    le32(h + 0, kWireMagic);
    le16(h + 4, kWireFormatVersion);
    le16(h + 6, w.flags);
    for (int i = 0; i < 18; ++i) le64(h + 8 + 8 * i, (uint64_t) s.geometry[(size_t) i]);
    le64(h + 152, (uint64_t) s.layer_lo);
    le64(h + 160, (uint64_t) s.layer_hi);
    le64(h + 168, (uint64_t) w.n_kv);
    le64(h + 176, (uint64_t) w.n_checkpoints);
    le64(h + 184, (uint64_t) w.n_stage_parts);
    le64(h + 192, (uint64_t) w.live_tokens);
    le64(h + 200, w.blob_pool_off);
    le64(h + 208, w.blob_pool_bytes);
    le64(h + 216, id.geom_hash);
    le64(h + 224, id.pack_hash);
    le64(h + 232, w.total_bytes);
}

}  // namespace

namespace wire_detail {

bool plan(const SavedConversation& image, int max_depth, const SizeOf& size_of, WirePlan& plan,
          std::vector<PlannedBlob>& blobs, std::string& error) {
    Planned p;
    if (!plan_image(image, max_depth, p, error, size_of)) return false;
    plan = p.plan;
    blobs.clear();
    blobs.reserve(p.blobs.size());
    for (const Blob& b : p.blobs)
        blobs.push_back(PlannedBlob{b.buf ? (const void*) b.buf : (const void*) b.vec, b.rel, b.bytes});
    return true;
}

bool write_records(const SavedConversation& image, const WireIdentity& identity, const WirePlan& plan,
                   const std::vector<PlannedBlob>& blobs, const SizeOf& size_of, uint8_t* out, std::string& error) {
    uint8_t* at = out;
    header_bytes(image, plan, identity, at);
    at += kWireHeaderRecordBytes;
    const uint8_t* end = out + plan.blob_pool_off;
    size_t next = 0;
    bool order_ok = true, room = true;
    Traversal walk(
        [&](const uint8_t* d, size_t n) {
            if ((uint64_t) (end - at) < n) return room = false;
            std::memcpy(at, d, n);
            at += n;
            return true;
        },
        [&](const ConversationBuffer* buf, const std::vector<uint8_t>* vec) -> uint64_t {
            const uint64_t n = buf ? size_of(buf, buf->size()) : size_of(vec, vec->size());
            if (!n) return 0;
            const void* key = buf ? (const void*) buf : (const void*) vec;
            if (next >= blobs.size() || blobs[next].key != key) {
                order_ok = false;
                return 0;
            }
            return plan.blob_pool_off + blobs[next++].rel;
        },
        size_of);
    if (!walk.body(image) || !room) return refuse(error, "internal: the records overran their planned bytes");
    if (!order_ok || next != blobs.size()) return refuse(error, "internal: the blob order changed between passes");
    std::memset(at, 0, (size_t) (end - at));
    return true;
}

}  // namespace wire_detail

bool conversation_wire_plan(const SavedConversation& image, int max_checkpoint_depth, WirePlan& plan,
                            std::string& error) {
    Planned p;
    if (!plan_image(image, max_checkpoint_depth, p, error)) return false;
    plan = p.plan;
    return true;
}

bool conversation_wire_plan(const SavedConversation& image, WirePlan& plan, std::string& error) {
    return conversation_wire_plan(image, kWireMaxCheckpointDepth, plan, error);
}

bool conversation_wire_encode(const SavedConversation& image, WireSink& sink, const WireIdentity& identity,
                              int max_checkpoint_depth, WirePlan& plan, WireEncoded& out, std::string& error) {
    Planned p;
    if (!plan_image(image, max_checkpoint_depth, p, error)) return false;
    plan = p.plan;
    HashedOut w(sink, error);
    uint8_t header[kWireHeaderRecordBytes];
    header_bytes(image, p.plan, identity, header);
    if (!w(header, sizeof header)) return false;
    size_t next = 0;
    bool order_ok = true;
    Traversal walk([&](const uint8_t* d, size_t n) { return w(d, n); },
                   [&](const ConversationBuffer* buf, const std::vector<uint8_t>* vec) -> uint64_t {
                       const uint64_t n = buf ? buf->size() : vec->size();
                       if (!n) return 0;
                       if (next >= p.blobs.size() || p.blobs[next].buf != buf || p.blobs[next].vec != vec) {
                           order_ok = false;
                           return 0;
                       }
                       return p.plan.blob_pool_off + p.blobs[next++].rel;
                   });
    if (!walk.body(image)) return false;
    if (!order_ok || next != p.blobs.size()) return refuse(error, "internal: the blob order changed between passes");
    static const uint8_t zeros[64] = {};
    if (!w(zeros, (size_t) (p.plan.blob_pool_off - w.pos()))) return false;
    uint64_t cursor = 0;
    for (const Blob& b : p.blobs) {
        if (!w(zeros, (size_t) (b.rel - cursor))) return false;
        if (b.vec) {
            for (uint64_t at = 0; at < b.bytes; at += kWireChunkBytes)
                if (!w(b.vec->data() + at, (size_t) std::min<uint64_t>(kWireChunkBytes, b.bytes - at))) return false;
        } else {
            bool ok = true;
            b.buf->visit(0, b.bytes, [&](const uint8_t* d, size_t n, size_t) { return ok = w(d, n); });
            if (!ok) return false;
        }
        cursor = b.rel + b.bytes;
    }
    if (!w(zeros, (size_t) (p.plan.blob_pool_bytes - cursor))) return false;
    if (w.pos() != p.plan.total_bytes) return refuse(error, "internal: the written bytes disagree with the plan");
    out.bytes = w.pos();
    out.payload_hash = w.hash();
    out.blob_pool_bytes = p.plan.blob_pool_bytes;
    out.blobs = p.blobs.size();
    return true;
}

bool conversation_wire_encode(const SavedConversation& image, WireSink& sink, const WireIdentity& identity,
                              WireEncoded& out, std::string& error) {
    WirePlan plan;
    return conversation_wire_encode(image, sink, identity, kWireMaxCheckpointDepth, plan, out, error);
}

// ------------------------------------------------------------------------------------------------ sinks / sources

bool VectorWireSink::write(const uint8_t* data, size_t bytes) {
    bytes_.insert(bytes_.end(), data, data + bytes);
    return true;
}

SlotWireSink::SlotWireSink(int fd, uint64_t offset, uint64_t capacity) : fd_(fd), at_(offset), capacity_(capacity) {}
SlotWireSink::SlotWireSink(uint8_t* mapping, uint64_t capacity) : map_(mapping), capacity_(capacity) {}

bool SlotWireSink::write(const uint8_t* data, size_t bytes) {
    if (bytes > capacity_ - pos_) {
        error_ = "the payload needs more than the slot's " + num(capacity_) + " bytes; claim a larger tier";
        return false;
    }
    if (map_) {
        std::memcpy(map_ + pos_, data, bytes);
    } else {
        size_t done = 0;
        while (done < bytes) {
            const ssize_t n = ::pwrite(fd_, data + done, bytes - done, (off_t) (at_ + pos_ + done));
            if (n < 0 && errno == EINTR) continue;
            if (n <= 0) {
                error_ = std::string("pwrite into the slot failed: ") + std::strerror(errno);
                return false;
            }
            done += (size_t) n;
        }
    }
    pos_ += bytes;
    return true;
}

bool SpanWireSource::read(uint8_t* dst, uint64_t offset, size_t bytes) const {
    if (offset > n_ || bytes > n_ - offset) return false;
    std::memcpy(dst, p_ + offset, bytes);
    return true;
}
const uint8_t* SpanWireSource::span(uint64_t offset, size_t bytes) const {
    if (offset > n_ || bytes > n_ - offset) return nullptr;
    return p_ + offset;
}

bool FileWireSource::read(uint8_t* dst, uint64_t offset, size_t bytes) const {
    if (offset > n_ || bytes > n_ - offset) return false;
    size_t done = 0;
    while (done < bytes) {
        const ssize_t n = ::pread(fd_, dst + done, bytes - done, (off_t) (at_ + offset + done));
        if (n < 0 && errno == EINTR) continue;
        if (n <= 0) return false;
        done += (size_t) n;
    }
    return true;
}

// ------------------------------------------------------------------------------------------------ decode

namespace {

struct Ref {
    uint64_t bytes = 0, off = 0;
};
struct KvIn {
    int format = 0;
    int64_t cells = 0, heads = 0, head_dim = 0, page_size = 0, pooled_rows = 0, idx_dim = 0;
    Ref refs[5];
};
struct CpIn {
    std::vector<int32_t> ids;
    std::vector<ConversationImageKey> imgs;
    Ref refs[5];
    uint64_t used = 0;
    std::vector<CpIn> parts;
};
struct StageIn {
    int64_t lo = 0, hi = 0;
    CpIn state;
    std::vector<KvIn> kv;
};

void parse_header(const uint8_t* h, WireHeaderRecord& r) {
    r.magic = rd32(h);
    r.fmt_version = rd16(h + 4);
    r.flags = rd16(h + 6);
    for (int i = 0; i < 18; ++i) r.geometry[i] = rd64(h + 8 + 8 * i);
    r.layer_lo = rd64(h + 152);
    r.layer_hi = rd64(h + 160);
    r.n_kv = (int64_t) rd64(h + 168);
    r.n_checkpoints = (int64_t) rd64(h + 176);
    r.n_stage_parts = (int64_t) rd64(h + 184);
    r.live_tokens = (int64_t) rd64(h + 192);
    r.blob_pool_off = rd64(h + 200);
    r.blob_pool_bytes = rd64(h + 208);
    r.geom_hash = rd64(h + 216);
    r.pack_hash = rd64(h + 224);
    r.payload_bytes = rd64(h + 232);
    r.payload_hash = rd64(h + 240);
    r.reserved = rd64(h + 248);
}

/// The checks a header must pass on its own (no geometry, no hashes, no body).
bool header_self_check(const WireHeaderRecord& h, std::string& error) {
    if (h.magic != kWireMagic) return refuse(error, "not an SR4H hand-off payload (magic 0x" + hex16(h.magic) + ")");
    if (h.fmt_version != kWireFormatVersion)
        return refuse(error, "unsupported payload format version " + num(h.fmt_version) + " (this build reads " +
                                 num(kWireFormatVersion) + ")");
    if (h.flags & ~kWireFlagKnown) return refuse(error, "unknown header flag bits 0x" + hex16(h.flags & ~kWireFlagKnown));
    if (h.flags & kWireFlagPartial) return refuse(error, "the payload is marked partial and can never be mounted");
    if (h.payload_hash != 0)
        return refuse(error, "reserved field is not zero: the header's payload_hash must be 0 on the wire");
    if (h.reserved != 0) return refuse(error, "reserved field is not zero: the header's last word must be 0");
    if (h.payload_bytes < kWireHeaderRecordBytes)
        return refuse(error, "the header declares " + num(h.payload_bytes) + " payload bytes, less than itself");
    if (h.blob_pool_off % kWireBlobAlign) return refuse(error, "the blob pool does not start on a 64-byte boundary");
    if (h.blob_pool_off < kWireHeaderRecordBytes || h.blob_pool_off > h.payload_bytes ||
        h.blob_pool_bytes != h.payload_bytes - h.blob_pool_off)
        return refuse(error, "the blob pool does not end the payload (off " + num(h.blob_pool_off) + ", " +
                                 num(h.blob_pool_bytes) + " bytes, payload " + num(h.payload_bytes) + ")");
    if (h.n_kv < 0 || h.n_kv > kWireMaxKvRecords) return refuse(error, "n_kv " + num((uint64_t) h.n_kv) + " is out of range");
    if (h.n_checkpoints < 0 || h.n_checkpoints > kWireMaxCheckpoints)
        return refuse(error, "n_checkpoints " + num((uint64_t) h.n_checkpoints) + " is out of range");
    if (h.n_stage_parts < 0 || h.n_stage_parts > kWireMaxStageParts)
        return refuse(error, "n_stage_parts " + num((uint64_t) h.n_stage_parts) + " is out of range");
    if (h.live_tokens < 0) return refuse(error, "live_tokens is negative");
    if (((h.flags & kWireFlagHasStageParts) != 0) != (h.n_stage_parts > 0))
        return refuse(error, "the has_stage_parts flag disagrees with n_stage_parts");
    return true;
}

class Decoder {
public:
    /// `shape` null: a full decode (blobs copied into a fresh image that replaces the caller's on success).
    /// `shape` set: a shape decode - the image is built in place with every blob left empty and recorded in
    /// `shape` (key -> payload offset and size); no blob byte and no hash is read from the source.
    Decoder(const WireSource& src, const WireExpect& expect, std::string& error,
            wire_detail::BlobTable* shape = nullptr)
        : src_(src), expect_(expect), error_(error), shape_(shape) {}

    bool run(SavedConversation& image, WireDecoded& info) {
        if (src_.size() < kWireHeaderRecordBytes)
            return refuse(error_, "the payload is shorter than the header (" + num(src_.size()) + " of 256 bytes)");
        uint8_t raw[kWireHeaderRecordBytes];
        if (!src_.read(raw, 0, sizeof raw)) return refuse(error_, "the source could not serve the header");
        parse_header(raw, h_);
        if (!header_self_check(h_, error_)) return false;
        if (expect_.max_payload_bytes && h_.payload_bytes > expect_.max_payload_bytes)
            return refuse(error_, "the header declares " + num(h_.payload_bytes) + " bytes, more than the slot's " +
                                      num(expect_.max_payload_bytes));
        if (h_.payload_bytes > src_.size())
            return refuse(error_, "the header declares " + num(h_.payload_bytes) + " payload bytes but only " +
                                      num(src_.size()) + " are available");
        pool_off_ = h_.blob_pool_off;
        pool_bytes_ = h_.blob_pool_bytes;
        if (expect_.stage_parts >= 0 && expect_.stage_parts != h_.n_stage_parts)
            return refuse(error_, "the payload carries " + num((uint64_t) h_.n_stage_parts) +
                                      " layer-split stage parts; this instance has " + num((uint64_t) expect_.stage_parts));
        if (expect_.check_geometry)
            for (int i = 0; i < 18; ++i)
                if ((int64_t) h_.geometry[i] != expect_.geometry[(size_t) i])
                    return refuse(error_, "runtime geometry differs: slot " + num((uint64_t) i) + " is " +
                                              std::to_string((int64_t) h_.geometry[i]) + ", this process has " +
                                              std::to_string(expect_.geometry[(size_t) i]));
        if (expect_.check_hashes) {
            if (h_.geom_hash != expect_.geom_hash)
                return refuse(error_, "geom_hash " + hex16(h_.geom_hash) + " differs from the expected " +
                                          hex16(expect_.geom_hash));
            if (h_.pack_hash != expect_.pack_hash)
                return refuse(error_, "pack_hash " + hex16(h_.pack_hash) + " differs from the expected " +
                                          hex16(expect_.pack_hash));
        }
        if (shape_) {
            if (expect_.check_payload_hash)
                return refuse(error_, "a shape decode never reads the blobs, so it cannot check the payload hash");
            hash_ = 0;
        } else if (!hash_payload()) {
            return false;
        }
        if (expect_.check_payload_hash && hash_ != expect_.payload_hash)
            return refuse(error_, "payload hash " + hex16(hash_) + " differs from the expected " +
                                      hex16(expect_.payload_hash));
        // the records, bounded by the start of the pool
        uint64_t pos = kWireHeaderRecordBytes;
        const uint64_t end = pool_off_;
        std::vector<KvIn> kv((size_t) h_.n_kv);
        for (auto& k : kv) {
            uint64_t body_end = 0;
            if (!record(pos, end, kWireRecordKv, "a KV record in the KV array", body_end) || !kv_body(pos, body_end, k))
                return false;
        }
        CpIn live;
        {
            uint64_t body_end = 0;
            if (!record(pos, end, kWireRecordCheckpoint, "the live CHECKPOINT", body_end) ||
                !checkpoint(pos, body_end, 0, live))
                return false;
        }
        if ((uint64_t) h_.live_tokens != live.ids.size())
            return refuse(error_, "the header's live_tokens " + num((uint64_t) h_.live_tokens) +
                                      " disagrees with the live checkpoint's " + num(live.ids.size()) + " ids");
        std::vector<CpIn> cps((size_t) h_.n_checkpoints);
        for (auto& c : cps) {
            uint64_t body_end = 0;
            if (!record(pos, end, kWireRecordCheckpoint, "a retained CHECKPOINT", body_end) || !checkpoint(pos, body_end, 0, c))
                return false;
        }
        std::vector<StageIn> stages((size_t) h_.n_stage_parts);
        for (auto& s : stages) {
            uint64_t body_end = 0;
            if (!record(pos, end, kWireRecordStage, "a STAGE", body_end) || !stage(pos, body_end, s)) return false;
        }
        uint64_t end_body = 0;
        if (!record(pos, end, kWireRecordEnd, "the END!", end_body)) return false;
        if (align64(pos) != pool_off_) return refuse(error_, "the records do not end where the blob pool begins");
        if (pool_bytes_ != (blobs_ ? align64(cursor_) : 0))
            return refuse(error_, "the blob pool's size disagrees with the blobs it holds");

        // every check passed: build the image (a shape decode builds in place, so the recorded keys stay valid)
        SavedConversation local;
        SavedConversation& out = shape_ ? image : local;
        if (shape_) {
            out = SavedConversation{};
            shape_->clear();
        }
        for (int i = 0; i < 18; ++i) out.geometry[(size_t) i] = (int64_t) h_.geometry[i];
        out.layer_lo = (int64_t) h_.layer_lo;
        out.layer_hi = (int64_t) h_.layer_hi;
        out.cvec = (h_.flags & kWireFlagCvec) != 0;
        out.owner = kNoOwner;
        out.kv.resize(kv.size());
        for (size_t i = 0; i < kv.size(); ++i)
            if (!make_kv(kv[i], out.kv[i])) return false;
        if (!make_checkpoint(live, out.live)) return false;
        out.checkpoints.resize(cps.size());
        for (size_t i = 0; i < cps.size(); ++i)
            if (!make_checkpoint(cps[i], out.checkpoints[i])) return false;
        out.stage_parts.resize(stages.size());
        for (size_t i = 0; i < stages.size(); ++i) {
            ConversationStageSnapshot& s = out.stage_parts[i];
            s.layer_lo = stages[i].lo;
            s.layer_hi = stages[i].hi;
            if (!make_checkpoint(stages[i].state, s.state)) return false;
            s.kv.resize(stages[i].kv.size());
            for (size_t j = 0; j < s.kv.size(); ++j)
                if (!make_kv(stages[i].kv[j], s.kv[j])) return false;
        }
        if (!shape_) image = std::move(out);
        info = WireDecoded{};
        info.bytes = h_.payload_bytes;
        info.payload_hash = hash_;
        info.geom_hash = h_.geom_hash;
        info.pack_hash = h_.pack_hash;
        for (int i = 0; i < 18; ++i) info.geometry[(size_t) i] = (int64_t) h_.geometry[i];
        info.layer_lo = (int64_t) h_.layer_lo;
        info.layer_hi = (int64_t) h_.layer_hi;
        info.n_kv = h_.n_kv;
        info.n_checkpoints = h_.n_checkpoints;
        info.n_stage_parts = h_.n_stage_parts;
        info.live_tokens = h_.live_tokens;
        info.flags = h_.flags;
        info.cvec = (h_.flags & kWireFlagCvec) != 0;
        info.blob_pool_off = pool_off_;
        info.blob_pool_bytes = pool_bytes_;
        info.blobs = blobs_;
        return true;
    }

private:
    /// Read [off, off + n) of the payload; the caller keeps off + n inside its record.
    bool get(uint64_t off, void* dst, size_t n) {
        if (off > h_.payload_bytes || n > h_.payload_bytes - off)
            return refuse(error_, "the payload is shorter than its records claim");
        if (n && !src_.read(static_cast<uint8_t*>(dst), off, n))
            return refuse(error_, "the source could not serve payload bytes [" + num(off) + ", " + num(off + n) + ")");
        return true;
    }
    /// A field of `n` bytes at `pos`, inside the record body ending at `end`.
    bool field(uint64_t& pos, uint64_t end, void* dst, size_t n, const char* rec) {
        if (pos > end || n > end - pos)
            return refuse(error_, std::string("the ") + rec + " record is shorter than its contents");
        if (!get(pos, dst, n)) return false;
        pos += n;
        return true;
    }
    bool u64(uint64_t& pos, uint64_t end, uint64_t& v, const char* rec) {
        uint8_t b[8];
        if (!field(pos, end, b, 8, rec)) return false;
        v = rd64(b);
        return true;
    }
    bool record(uint64_t& pos, uint64_t end, uint32_t want, const char* what, uint64_t& body_end) {
        uint8_t b[kWireRecordHeaderBytes];
        if (pos > end || kWireRecordHeaderBytes > end - pos)
            return refuse(error_, std::string("the payload is shorter than its records claim (") + what + " record)");
        if (!get(pos, b, sizeof b)) return false;
        const uint32_t kind = rd32(b), flags = rd32(b + 4);
        const uint64_t bytes = rd64(b + 8);
        if (kind != want) {
            if (want == kWireRecordEnd)
                return refuse(error_, "the record stream is missing its END! marker (found kind " + num(kind) + ")");
            return refuse(error_, std::string("expected ") + what + " record, found record kind " + num(kind));
        }
        if (flags) return refuse(error_, std::string(what) + " record has non-zero flags " + num(flags));
        if (want == kWireRecordKv && bytes != kKvBody)
            return refuse(error_, "the KV array holds a record of " + num(bytes) + " bytes; a KV record is 136");
        if (want == kWireRecordEnd && bytes != 0) return refuse(error_, "the END! record carries a body");
        pos += kWireRecordHeaderBytes;
        if (bytes > end - pos)
            return refuse(error_, std::string(what) + " record declares more bytes (" + num(bytes) +
                                      ") than the payload holds");
        body_end = pos + bytes;
        return true;
    }
    bool blobref(uint64_t& pos, uint64_t end, Ref& r, const char* rec) {
        if (!u64(pos, end, r.bytes, rec) || !u64(pos, end, r.off, rec)) return false;
        if (r.bytes == 0) {
            if (r.off != 0) return refuse(error_, "a zero-length blob must be referenced as {0,0}");
            return true;
        }
        if (r.off < pool_off_ || (r.off - pool_off_) % kWireBlobAlign)
            return refuse(error_, "a blob reference is not on a 64-byte boundary of the blob pool");
        const uint64_t rel = r.off - pool_off_;
        if (rel > pool_bytes_ || r.bytes > pool_bytes_ - rel)
            return refuse(error_, "a blob reference points past the end of the pool");
        if (rel != align64(cursor_)) return refuse(error_, "a blob reference is out of emission order");
        cursor_ = rel + r.bytes;
        ++blobs_;
        return true;
    }
    bool kv_body(uint64_t& pos, uint64_t end, KvIn& k) {
        uint8_t b[56];
        if (!field(pos, end, b, sizeof b, "KV")) return false;
        k.format = (int) (int32_t) rd32(b);
        if (rd32(b + 4)) return refuse(error_, "reserved field is not zero (the KV record's pad)");
        int64_t* f[6] = {&k.cells, &k.heads, &k.head_dim, &k.page_size, &k.pooled_rows, &k.idx_dim};
        for (int i = 0; i < 6; ++i) *f[i] = (int64_t) rd64(b + 8 + 8 * i);
        for (auto& r : k.refs)
            if (!blobref(pos, end, r, "KV")) return false;
        if (pos != end) return refuse(error_, "a KV record does not end where its header said");
        return true;
    }
    bool checkpoint(uint64_t& pos, uint64_t end, int depth, CpIn& c) {
        if (depth > expect_.max_checkpoint_depth)
            return refuse(error_, "checkpoint stage_parts are nested deeper than " + num((uint64_t) expect_.max_checkpoint_depth) + " levels");
        uint64_t n_ids = 0;
        if (!u64(pos, end, n_ids, "CHECKPOINT")) return false;
        if ((int64_t) n_ids < 0 || n_ids > (end - pos) / 4)
            return refuse(error_, "a checkpoint's id count " + num(n_ids) + " does not fit its record");
        c.ids.resize((size_t) n_ids);
        if (!field(pos, end, c.ids.data(), (size_t) n_ids * 4, "CHECKPOINT")) return false;
        if constexpr (std::endian::native != std::endian::little)   // the wire's int32s are little-endian
            for (auto& id : c.ids) id = (int32_t) rd32(reinterpret_cast<const uint8_t*>(&id));
        if ((n_ids * 4) % 8) {
            uint8_t pad[4];
            if (!field(pos, end, pad, 4, "CHECKPOINT")) return false;
            if (pad[0] | pad[1] | pad[2] | pad[3]) return refuse(error_, "reserved field is not zero (the ids pad)");
        }
        uint64_t n_imgs = 0;
        if (!u64(pos, end, n_imgs, "CHECKPOINT")) return false;
        if ((int64_t) n_imgs < 0 || (int64_t) n_imgs > kWireMaxImages || n_imgs > (end - pos) / 16)
            return refuse(error_, "a checkpoint's image count " + num(n_imgs) + " does not fit its record");
        c.imgs.resize((size_t) n_imgs);
        for (auto& img : c.imgs) {
            uint64_t start = 0, hash = 0;
            if (!u64(pos, end, start, "CHECKPOINT") || !u64(pos, end, hash, "CHECKPOINT")) return false;
            img.start = (int64_t) start;
            img.hash = hash;
        }
        for (auto& r : c.refs)
            if (!blobref(pos, end, r, "CHECKPOINT")) return false;
        uint64_t n_parts = 0;
        if (!u64(pos, end, c.used, "CHECKPOINT") || !u64(pos, end, n_parts, "CHECKPOINT")) return false;
        if ((int64_t) n_parts < 0 || n_parts > (end - pos) / kWireRecordHeaderBytes)
            return refuse(error_, "a checkpoint's stage-part count " + num(n_parts) + " does not fit its record");
        if (n_parts && depth + 1 > expect_.max_checkpoint_depth)
            return refuse(error_, "checkpoint stage_parts are nested deeper than " + num((uint64_t) expect_.max_checkpoint_depth) + " levels");
        c.parts.resize((size_t) n_parts);
        for (auto& p : c.parts) {
            uint64_t body_end = 0;
            if (!record(pos, end, kWireRecordCheckpoint, "a stage-part CHECKPOINT", body_end) ||
                !checkpoint(pos, body_end, depth + 1, p))
                return false;
        }
        if (pos != end)
            return refuse(error_, "a CHECKPOINT record does not end where its header said (" + num(end - pos) +
                                      " bytes unaccounted)");
        return true;
    }
    bool stage(uint64_t& pos, uint64_t end, StageIn& s) {
        uint64_t lo = 0, hi = 0, n_kv = 0;
        if (!u64(pos, end, lo, "STAGE") || !u64(pos, end, hi, "STAGE")) return false;
        s.lo = (int64_t) lo;
        s.hi = (int64_t) hi;
        uint64_t body_end = 0;
        if (!record(pos, end, kWireRecordCheckpoint, "the STAGE's CHECKPOINT", body_end) ||
            !checkpoint(pos, body_end, 0, s.state))
            return false;
        if (!u64(pos, end, n_kv, "STAGE")) return false;
        if ((int64_t) n_kv < 0 || (int64_t) n_kv > kWireMaxKvRecords ||
            n_kv > (end - pos) / (kWireRecordHeaderBytes + kKvBody))
            return refuse(error_, "a STAGE record's KV count " + num(n_kv) + " does not fit its record");
        s.kv.resize((size_t) n_kv);
        for (auto& k : s.kv) {
            uint64_t kv_end = 0;
            if (!record(pos, end, kWireRecordKv, "a KV record in the STAGE's KV array", kv_end) || !kv_body(pos, kv_end, k))
                return false;
        }
        if (pos != end) return refuse(error_, "a STAGE record does not end where its header said");
        return true;
    }
    bool hash_payload() {
        hash_ = kWireHashSeed;
        std::vector<uint8_t> chunk;
        for (uint64_t at = 0; at < h_.payload_bytes;) {
            const size_t n = (size_t) std::min<uint64_t>(kWireChunkBytes, h_.payload_bytes - at);
            const uint8_t* p = src_.span(at, n);
            if (!p) {
                chunk.resize(n);
                if (!src_.read(chunk.data(), at, n))
                    return refuse(error_, "the source could not serve payload bytes [" + num(at) + ", " + num(at + n) + ")");
                p = chunk.data();
            }
            hash_ = fnv1a64(p, n, hash_);
            at += n;
        }
        return true;
    }
    bool copy_out(const Ref& r, uint8_t* dst, size_t n, uint64_t at) {
        for (uint64_t done = 0; done < n;) {
            const size_t piece = (size_t) std::min<uint64_t>(kWireChunkBytes, n - done);
            const uint8_t* p = src_.span(r.off + at + done, piece);
            if (p) std::memcpy(dst + done, p, piece);
            else if (!get(r.off + at + done, dst + done, piece)) return false;
            done += piece;
        }
        return true;
    }
    bool make_buffer(const Ref& r, ConversationBuffer& b) {
        if (shape_) {
            if (r.bytes) (*shape_)[&b] = wire_detail::BlobAt{r.off, r.bytes};
            return true;
        }
        b.resize((size_t) r.bytes);
        bool ok = true;
        b.visit(0, (size_t) r.bytes, [&](uint8_t* p, size_t n, size_t at) { return ok = copy_out(r, p, n, at); });
        return ok;
    }
    bool make_vec(const Ref& r, std::vector<uint8_t>& v) {
        if (shape_) {
            if (r.bytes) (*shape_)[&v] = wire_detail::BlobAt{r.off, r.bytes};
            return true;
        }
        v.resize((size_t) r.bytes);
        return copy_out(r, v.data(), v.size(), 0);
    }
    bool make_kv(const KvIn& in, ConversationKv& k) {
        k.format = in.format;
        k.cells = in.cells;
        k.heads = in.heads;
        k.head_dim = in.head_dim;
        k.page_size = in.page_size;
        k.pooled_rows = in.pooled_rows;
        k.idx_dim = in.idx_dim;
        ConversationBuffer* bufs[5] = {&k.k, &k.v, &k.k_scale, &k.v_scale, &k.pooled};
        for (int i = 0; i < 5; ++i)
            if (!make_buffer(in.refs[i], *bufs[i])) return false;
        return true;
    }
    bool make_checkpoint(const CpIn& in, ConversationCheckpoint& c) {
        c.ids = in.ids;
        c.imgs = in.imgs;
        c.used = in.used;
        std::vector<uint8_t>* vecs[5] = {&c.gdn, &c.ple, &c.tails, &c.dead, &c.block_pos};
        for (int i = 0; i < 5; ++i)
            if (!make_vec(in.refs[i], *vecs[i])) return false;
        c.stage_parts.resize(in.parts.size());
        for (size_t i = 0; i < in.parts.size(); ++i)
            if (!make_checkpoint(in.parts[i], c.stage_parts[i])) return false;
        return true;
    }

    const WireSource& src_;
    const WireExpect& expect_;
    std::string& error_;
    wire_detail::BlobTable* shape_ = nullptr;
    WireHeaderRecord h_{};
    uint64_t pool_off_ = 0, pool_bytes_ = 0, cursor_ = 0, hash_ = 0;
    size_t blobs_ = 0;
};

}  // namespace

bool conversation_wire_decode(const WireSource& source, SavedConversation& image, WireDecoded& info,
                              const WireExpect& expect, std::string& error) {
    Decoder d(source, expect, error);
    return d.run(image, info);
}

namespace wire_detail {
bool decode_shape(const WireSource& source, SavedConversation& image, WireDecoded& info, const WireExpect& expect,
                  BlobTable& blobs, std::string& error) {
    Decoder d(source, expect, error, &blobs);
    return d.run(image, info);
}
}  // namespace wire_detail

bool conversation_wire_decode(const uint8_t* data, uint64_t bytes, SavedConversation& image, WireDecoded& info,
                              const WireExpect& expect, std::string& error) {
    SpanWireSource src(data, bytes);
    return conversation_wire_decode(src, image, info, expect, error);
}

bool conversation_wire_peek(const uint8_t* data, uint64_t bytes, WireHeaderRecord& header, std::string& error) {
    if (!data || bytes < kWireHeaderRecordBytes)
        return refuse(error, "the payload is shorter than the header (" + num(bytes) + " of 256 bytes)");
    WireHeaderRecord h{};
    parse_header(data, h);
    if (!header_self_check(h, error)) return false;
    header = h;
    return true;
}

std::string conversation_wire_describe(const WireHeaderRecord& h) {
    char b[320];
    std::snprintf(b, sizeof b,
                  "SR4H v%u flags=0x%x layers=[%lld,%lld) n_kv=%lld n_checkpoints=%lld n_stage_parts=%lld "
                  "live_tokens=%lld pool=%llu+%llu payload=%llu geom_hash=%016llx pack_hash=%016llx",
                  (unsigned) h.fmt_version, (unsigned) h.flags, (long long) h.layer_lo, (long long) h.layer_hi,
                  (long long) h.n_kv, (long long) h.n_checkpoints, (long long) h.n_stage_parts,
                  (long long) h.live_tokens, (unsigned long long) h.blob_pool_off,
                  (unsigned long long) h.blob_pool_bytes, (unsigned long long) h.payload_bytes,
                  (unsigned long long) h.geom_hash, (unsigned long long) h.pack_hash);
    return b;
}

}  // namespace strata::core
