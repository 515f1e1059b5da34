// conversation_wire_device.cpp - SR4H payloads packed straight from device state
// (include/strata_kv/conversation_wire_device.hpp).
//
// 1. Validate exactly as conversation_snapshot_save does (conversation_snapshot_bytes).
// 2. Build a SHAPE image: the SavedConversation that save would produce, with every metadata field real but
//    every byte buffer empty; a side table maps each buffer to the pieces it is made of (a device stream through
//    a page table, a contiguous device range, or host memory) and so to its byte count.
// 3. Plan the payload from the shape (the encoder's own plan pass, sizes from the side table) and write the
//    header + record stream on the host.
// 4. Per device: one batch of gather launches moves that device's pieces into a zeroed image of the blob pool
//    (the staging buffer, or the destination itself when it is device memory), then one device-to-host copy per
//    run of consecutive pieces; host-resident pieces are copied on the host, sub-16-byte pieces by the copy
//    engine, and every byte of the pool nobody wrote is zeroed.
#include "strata_kv/conversation_wire_device.hpp"
#include "strata_kv/pinned.hpp"

#include "kv_stream_detail.h"
#include "skv_internal.h"
#include "snapshot_detail.hpp"
#include "strata_kv.h"
#include "wire_detail.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <unordered_map>
#include <utility>

namespace strata::core {
namespace {
using namespace snapshot_detail;

constexpr int kHostSide = -1;

/// One contiguous part of a blob.
struct Piece {
    int device = kHostSide;              // kHostSide: `host` holds the bytes
    strata::kv::DeviceStream dev;        // device side: logical bytes [from, from + bytes) of this stream
    uint64_t from = 0;
    const uint8_t* host = nullptr;
    uint64_t rel = 0;                    // offset inside the blob
    uint64_t bytes = 0;
};
struct Source {
    std::vector<Piece> pieces;
    uint64_t bytes = 0;
};
using Side = std::unordered_map<const void*, Source>;

bool pfail(std::string& error, const std::string& why) {
    error = "conversation wire device: " + why;
    return false;
}
bool cuda_ok(cudaError_t e, std::string& error, const char* step) {
    if (e == cudaSuccess) return true;
    (void) cudaGetLastError();
    return pfail(error, std::string(step) + ": " + cudaGetErrorString(e));
}

void add_device(Side& side, const void* key, int device, const strata::kv::DeviceStream& s, uint64_t from,
                uint64_t bytes) {
    if (!bytes) return;
    Source& src = side[key];
    src.pieces.push_back(Piece{device, s, from, nullptr, src.bytes, bytes});
    src.bytes += bytes;
}
void add_host(Side& side, const void* key, const uint8_t* p, uint64_t bytes) {
    if (!bytes) return;
    Source& src = side[key];
    src.pieces.push_back(Piece{kHostSide, {}, 0, p, src.bytes, bytes});
    src.bytes += bytes;
}
strata::kv::DeviceStream flat(const void* p) {
    strata::kv::DeviceStream s;
    s.base = p;
    return s;
}

/// One layer's K/V record and its five streams (the shape twin of enqueue_kv_save, no retained prefix).
bool shape_kv(ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto, bool index,
              int device, Side& side, std::string& error) {
    LayerExtent x;
    if (!layer_extent(st, g, upto, index, x, error) || !layer_usable(st, x, upto, error)) return false;
    image.format = x.format;
    image.cells = x.cells;
    image.heads = g.n_head_kv;
    image.head_dim = g.head_dim;
    image.page_size = x.page_size;
    image.pooled_rows = x.pooled_rows;
    image.idx_dim = g.idx_key_dim;
    const auto src = layer_sources(st);
    const ConversationBuffer* dst[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    for (int i = 0; i < 5; ++i) {
        const uint64_t n = x.bytes[(size_t) i];
        if (!n) continue;
        if (!src[(size_t) i]) return fail(error, "missing state buffer");
        if (i < 4 && st.kv_mode != 0)
            add_host(side, dst[i], static_cast<const uint8_t*>(src[(size_t) i]), n);
        else
            add_device(side, dst[i], device, layer_stream(st, x, i, src[(size_t) i]), 0, n);
    }
    return true;
}

/// A session's running state into checkpoint `c` (whose ids are set): the shape twin of enqueue_checkpoint_save.
bool shape_running(ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g, int device, Side& side,
                   std::string& error) {
    RunningState rs;
    if (!running_state(ss, g, c.ids.size(), rs, error)) return false;
    const ConversationStateSizes& per = rs.per;
    add_device(side, &c.gdn, device, flat(ss.gdn_state), 0, rs.gdn());
    if (rs.keeps_ple) add_device(side, &c.ple, device, flat(ss.ple_hist), 0, rs.ple());
    for (size_t j = 0; j < rs.layers; ++j) {
        const QsaState& st = owned_layer(ss, j);
        add_device(side, &c.tails, device, flat(st.idx_tail), 0, per.tail);
        add_device(side, &c.dead, device, flat(st.idx_dead), 0, per.dead);
        add_device(side, &c.block_pos, device, flat(st.idx_block_pos), 0, per.block_pos);
    }
    return true;
}

/// A retained checkpoint (host data already): metadata copied, its byte vectors referenced in place.
void shape_retained(ConversationCheckpoint& out, const ConversationCheckpoint& c, Side& side) {
    out.ids = c.ids;
    out.imgs = c.imgs;
    out.used = c.used;
    add_host(side, &out.gdn, c.gdn.data(), c.gdn.size());
    add_host(side, &out.ple, c.ple.data(), c.ple.size());
    add_host(side, &out.tails, c.tails.data(), c.tails.size());
    add_host(side, &out.dead, c.dead.data(), c.dead.size());
    add_host(side, &out.block_pos, c.block_pos.data(), c.block_pos.size());
    out.stage_parts.resize(c.stage_parts.size());   // sized before any part registers an address
    for (size_t i = 0; i < c.stage_parts.size(); ++i) shape_retained(out.stage_parts[i], c.stage_parts[i], side);
}

int resolve(int device) {
    if (device >= 0) return device;
    int cur = 0;
    cudaGetDevice(&cur);
    return cur;
}

/// The shape of conversation_snapshot_save's image, in the same order.
bool build_shape(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
                 const ModelGeometry& g, const QsaState& draft, SavedConversation& shape, Side& side,
                 std::string& error) {
    size_t estimate = 0;
    if (!conversation_snapshot_bytes(view, ss, stages, g, draft, estimate, error)) return false;
    shape = SavedConversation{};
    side.clear();
    shape.geometry = geometry_key(g);
    shape.layer_lo = ss.layer_lo;
    shape.layer_hi = ss.layer_hi;
    shape.live.ids = view.ids;
    shape.live.imgs = view.images;
    shape.cvec = view.cvec;
    shape.checkpoints.resize(view.checkpoints.size());
    for (size_t i = 0; i < view.checkpoints.size(); ++i) shape_retained(shape.checkpoints[i], view.checkpoints[i], side);
    const size_t layers = owned_count(ss);
    shape.kv.resize(layers + 1);
    const int64_t upto = (int64_t) view.ids.size();
    const int main_dev = resolve(stages.main_device);
    if (!shape_running(shape.live, ss, g, main_dev, side, error)) return false;
    for (size_t j = 0; j < layers; ++j)
        if (!shape_kv(shape.kv[j], owned_layer(ss, j), g, upto, true, main_dev, side, error)) return false;
    const int draft_dev = stages.empty() ? main_dev : resolve(stages.draft_device);
    if (!shape_kv(shape.kv.back(), draft, g, upto, false, draft_dev, side, error)) return false;
    shape.stage_parts.resize((size_t) stage_count(stages));
    for (int64_t i = 0; i < stage_count(stages); ++i) {
        const ConversationStage& stage = stages.stages[i];
        const SessionState& sss = *stage.session;
        ConversationStageSnapshot& part = shape.stage_parts[(size_t) i];
        part.layer_lo = sss.layer_lo;
        part.layer_hi = sss.layer_hi;
        part.state.ids = view.ids;
        part.kv.resize(owned_count(sss));
        const int dev = resolve(stage.device);
        if (!shape_running(part.state, sss, g, dev, side, error)) return false;
        for (size_t j = 0; j < part.kv.size(); ++j)
            if (!shape_kv(part.kv[j], owned_layer(sss, j), g, upto, true, dev, side, error)) return false;
    }
    return true;
}

wire_detail::SizeOf side_sizes(const Side& side) {
    return [&side](const void* key, uint64_t real) -> uint64_t {
        const auto it = side.find(key);
        return it == side.end() ? real : it->second.bytes;
    };
}

/// A piece placed at its absolute payload offset.
struct Placed {
    const Piece* piece;
    uint64_t at;
};

bool granular(const Piece& p, uint64_t at) {
    if (p.dev.pages) return true;   // paged streams are page-granular by construction
    const uintptr_t src = reinterpret_cast<uintptr_t>(static_cast<const uint8_t*>(p.dev.base) + p.from);
    return ((src | at | p.bytes) & 15u) == 0;
}

skv_segment segment_of(const Piece& p, uint8_t* dst) {
    skv_segment s{};
    const uint8_t* base = static_cast<const uint8_t*>(p.dev.base);
    s.bytes = p.bytes;
    s.dst = dst;
    if (p.dev.pages) {
        s.src = base;
        s.src_pages = p.dev.pages + p.from / p.dev.page_bytes;
        s.page_bytes = p.dev.page_bytes;
        s.src_page_limit = p.dev.page_limit;
    } else {
        s.src = base + p.from;
    }
    return s;
}

bool launch_all(const std::vector<skv_segment>& segs, std::string& error) {
    for (size_t i = 0; i < segs.size(); i += SKV_COPY_MAX_SEGMENTS) {
        const int n = (int) std::min<size_t>(SKV_COPY_MAX_SEGMENTS, segs.size() - i);
        if (skv_copy(segs.data() + i, n, SKV_COPY_AUTO, nullptr) != SKV_OK)
            return pfail(error, std::string("gather: ") + skv_last_error());
    }
    return true;
}

thread_local WireDevicePhases t_last_phases;

/// Host-clock marks of one pack or mount; finish() publishes them as this thread's last phases.  A call that fails
/// publishes nothing (the previous record stays).
class PhaseClock {
public:
    PhaseClock() : t0_(std::chrono::steady_clock::now()), prepared_(t0_), enqueued_(t0_) {}
    void mark_prepared() { prepared_ = enqueued_ = std::chrono::steady_clock::now(); }
    void mark_enqueued() { enqueued_ = std::chrono::steady_clock::now(); }
    void finish() {
        const auto end = std::chrono::steady_clock::now();
        auto ms = [](auto a, auto b) { return std::chrono::duration<double, std::milli>(b - a).count(); };
        t_last_phases = WireDevicePhases{ms(t0_, prepared_), ms(prepared_, enqueued_), ms(enqueued_, end), ms(t0_, end)};
    }

private:
    std::chrono::steady_clock::time_point t0_, prepared_, enqueued_;
};

bool status_clean(int device, std::string& error) {
    uint32_t status = 0;
    if (skv_query_status(device, nullptr, &status) != SKV_OK) return pfail(error, skv_last_error());
    if (status) return pfail(error, "the device refused part of the gather (a page-table entry outside its pool)");
    return true;
}

}  // namespace

// ------------------------------------------------------------------------------------------------ public API

bool conversation_wire_pack_plan(const ConversationView& view, const SessionState& ss,
                                 const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                 WirePlan& plan, std::string& error, const WireDeviceOptions& opt) {
    SavedConversation shape;
    Side side;
    std::vector<wire_detail::PlannedBlob> blobs;
    return build_shape(view, ss, stages, g, draft, shape, side, error) &&
           wire_detail::plan(shape, opt.max_checkpoint_depth, side_sizes(side), plan, blobs, error);
}

bool conversation_wire_pack_plan(const ConversationView& view, const SessionState& ss, const ModelGeometry& g,
                                 const QsaState& draft, WirePlan& plan, std::string& error,
                                 const WireDeviceOptions& opt) {
    return conversation_wire_pack_plan(view, ss, {}, g, draft, plan, error, opt);
}

bool conversation_wire_pack_device(const ConversationView& view, const SessionState& ss,
                                   const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                   const WireIdentity& identity, uint8_t* dst, uint64_t capacity, WirePlan& plan,
                                   WireEncoded& out, std::string& error, const WireDeviceOptions& opt) {
    PhaseClock phases;
    SavedConversation shape;
    Side side;
    std::vector<wire_detail::PlannedBlob> blobs;
    if (!build_shape(view, ss, stages, g, draft, shape, side, error)) return false;
    const wire_detail::SizeOf sizes = side_sizes(side);
    WirePlan p;
    if (!wire_detail::plan(shape, opt.max_checkpoint_depth, sizes, p, blobs, error)) return false;
    if (!dst) return pfail(error, "no destination");
    if (capacity < p.total_bytes)
        return pfail(error, "the payload needs " + std::to_string(p.total_bytes) + " bytes; the destination holds " +
                                std::to_string(capacity));
    cudaPointerAttributes attr{};
    if (!cuda_ok(cudaPointerGetAttributes(&attr, dst), error, "destination attributes")) return false;
    const bool on_device = attr.type == cudaMemoryTypeDevice;
    const int dst_device = on_device ? attr.device : kHostSide;

    // every piece at its absolute offset, in payload order
    std::vector<Placed> placed;
    for (const auto& b : blobs) {
        const auto it = side.find(b.key);
        if (it == side.end()) return pfail(error, "internal: a planned blob has no source");
        for (const Piece& pc : it->second.pieces) placed.push_back(Placed{&pc, p.blob_pool_off + b.rel + pc.rel});
    }
    std::map<int, std::vector<size_t>> by_device;   // kernel-gathered pieces per device
    std::vector<size_t> direct, host;
    for (size_t i = 0; i < placed.size(); ++i) {
        const Piece& pc = *placed[i].piece;
        if (pc.device == kHostSide) host.push_back(i);
        else if (granular(pc, placed[i].at)) by_device[pc.device].push_back(i);
        else direct.push_back(i);
        if (on_device && pc.device != kHostSide && pc.device != dst_device)
            return pfail(error, "a device destination must be on the device of every device-resident blob (blob on " +
                                    std::to_string(pc.device) + ", destination on " + std::to_string(dst_device) + ")");
    }

    // header + records
    std::vector<uint8_t> records;
    uint8_t* rec = dst;
    if (on_device) {
        records.resize((size_t) p.blob_pool_off);
        rec = records.data();
    }
    if (!wire_detail::write_records(shape, identity, p, blobs, sizes, rec, error)) return false;

    if (on_device) {
        const DeviceScope on(dst_device);
        if (!device_sync(error)) return false;   // the session's producers are done before the reads
        phases.mark_prepared();
        // one byte-range launch: the pads between blobs (and after the last; every other pool byte is gathered)
        // and the pieces too short or unaligned for the bulk engines
        std::vector<skv::ByteRange> small;
        uint64_t cursor = p.blob_pool_off;
        for (const Placed& pl : placed) {
            if (pl.at > cursor) small.push_back({dst + cursor, nullptr, pl.at - cursor});
            cursor = std::max(cursor, pl.at + pl.piece->bytes);
        }
        if (p.total_bytes > cursor) small.push_back({dst + cursor, nullptr, p.total_bytes - cursor});
        std::vector<size_t> large;
        for (size_t i : direct) {
            const Piece& pc = *placed[i].piece;
            if (pc.bytes <= skv::kByteRangeMaxBytes)
                small.push_back({dst + placed[i].at, static_cast<const uint8_t*>(pc.dev.base) + pc.from, pc.bytes});
            else
                large.push_back(i);
        }
        if (skv::byte_ranges(small, nullptr) != SKV_OK) return pfail(error, skv_last_error());
        if (!cuda_ok(cudaMemcpyAsync(dst, records.data(), records.size(), cudaMemcpyHostToDevice, nullptr), error,
                     "records"))
            return false;
        if (skv_clear_status(dst_device, nullptr) != SKV_OK) return pfail(error, skv_last_error());
        std::vector<skv_segment> segs;
        for (size_t i : by_device[dst_device]) segs.push_back(segment_of(*placed[i].piece, dst + placed[i].at));
        if (!launch_all(segs, error)) return false;
        for (size_t i : large) {
            const Piece& pc = *placed[i].piece;
            if (!cuda_ok(cudaMemcpyAsync(dst + placed[i].at, static_cast<const uint8_t*>(pc.dev.base) + pc.from,
                                         pc.bytes, cudaMemcpyDeviceToDevice, nullptr),
                         error, "running-state copy"))
                return false;
        }
        for (size_t i : host) {
            const Piece& pc = *placed[i].piece;
            if (!cuda_ok(cudaMemcpyAsync(dst + placed[i].at, pc.host, pc.bytes, cudaMemcpyHostToDevice, nullptr),
                         error, "host blob copy"))
                return false;
        }
        phases.mark_enqueued();
        if (!cuda_ok(cudaStreamSynchronize(nullptr), error, "synchronize") ||
            (!segs.empty() && !status_clean(dst_device, error)))
            return false;
        phases.finish();
        plan = p;
        out.bytes = p.total_bytes;
        out.payload_hash = 0;
        out.blob_pool_bytes = p.blob_pool_bytes;
        out.blobs = blobs.size();
        return true;
    }

    // host destination: mark what each step writes, so every other pool byte is zeroed exactly once
    phases.mark_prepared();
    std::vector<std::pair<uint64_t, uint64_t>> written;   // [begin, end) absolute
    for (auto& [device, idx] : by_device) {
        const DeviceScope on(device);
        if (!device_sync(error)) return false;
        const uint64_t lo = placed[idx.front()].at & ~uint64_t(255);
        const uint64_t hi = placed[idx.back()].at + placed[idx.back()].piece->bytes;
        uint8_t* staging = nullptr;
        if (!strata::kv::transfer_staging(hi - lo, &staging, error, "conversation wire device pack")) return false;
        if (skv_clear_status(device, nullptr) != SKV_OK) return pfail(error, skv_last_error());
        if (!cuda_ok(cudaMemsetAsync(staging, 0, hi - lo, nullptr), error, "staging clear")) return false;
        std::vector<skv_segment> segs;
        segs.reserve(idx.size());
        for (size_t i : idx) segs.push_back(segment_of(*placed[i].piece, staging + (placed[i].at - lo)));
        if (!launch_all(segs, error)) return false;
        // one copy per run: consecutive placed pieces (payload order) that all belong to this device's gather
        for (size_t k = 0; k < idx.size();) {
            size_t e = k;
            while (e + 1 < idx.size() && idx[e + 1] == idx[e] + 1) ++e;
            const uint64_t a = placed[idx[k]].at, b = placed[idx[e]].at + placed[idx[e]].piece->bytes;
            if (!cuda_ok(cudaMemcpyAsync(dst + a, staging + (a - lo), b - a, cudaMemcpyDeviceToHost, nullptr), error,
                         "device-to-host copy"))
                return false;
            written.emplace_back(a, b);
            k = e + 1;
        }
        for (size_t i : direct) {
            const Piece& pc = *placed[i].piece;
            if (pc.device != device) continue;
            if (!cuda_ok(cudaMemcpyAsync(dst + placed[i].at, static_cast<const uint8_t*>(pc.dev.base) + pc.from,
                                         pc.bytes, cudaMemcpyDeviceToHost, nullptr),
                         error, "running-state copy"))
                return false;
            written.emplace_back(placed[i].at, placed[i].at + pc.bytes);
        }
        if (!cuda_ok(cudaStreamSynchronize(nullptr), error, "synchronize") || !status_clean(device, error)) return false;
    }
    for (size_t i : direct) {   // sub-16-byte pieces of a device with nothing to gather
        const Piece& pc = *placed[i].piece;
        if (by_device.count(pc.device)) continue;
        const DeviceScope on(pc.device);
        if (!cuda_ok(cudaMemcpy(dst + placed[i].at, static_cast<const uint8_t*>(pc.dev.base) + pc.from, pc.bytes,
                                cudaMemcpyDeviceToHost),
                     error, "running-state copy"))
            return false;
        written.emplace_back(placed[i].at, placed[i].at + pc.bytes);
    }
    for (size_t i : host) {
        const Piece& pc = *placed[i].piece;
        std::memcpy(dst + placed[i].at, pc.host, pc.bytes);
        written.emplace_back(placed[i].at, placed[i].at + pc.bytes);
    }
    std::sort(written.begin(), written.end());
    uint64_t cursor = p.blob_pool_off;
    for (const auto& [a, b] : written) {
        if (a > cursor) std::memset(dst + cursor, 0, a - cursor);
        cursor = std::max(cursor, b);
    }
    if (p.total_bytes > cursor) std::memset(dst + cursor, 0, p.total_bytes - cursor);
    phases.mark_enqueued();   // the host target's copies wait per device above: they count as enqueue time

    plan = p;
    out.bytes = p.total_bytes;
    out.payload_hash = opt.hash ? fnv1a64(dst, p.total_bytes) : 0;
    out.blob_pool_bytes = p.blob_pool_bytes;
    out.blobs = blobs.size();
    phases.finish();
    return true;
}

bool conversation_wire_pack_device(const ConversationView& view, const SessionState& ss, const ModelGeometry& g,
                                   const QsaState& draft, const WireIdentity& identity, uint8_t* dst,
                                   uint64_t capacity, WirePlan& plan, WireEncoded& out, std::string& error,
                                   const WireDeviceOptions& opt) {
    return conversation_wire_pack_device(view, ss, {}, g, draft, identity, dst, capacity, plan, out, error, opt);
}

// ------------------------------------------------------------------------------------------------ device mount

namespace {

/// A page-locked host block from the recycling pool (strata_kv/pinned.hpp): device-to-host copies into it run at
/// PCIe speed with no staging.
struct PinnedBlock {
    uint8_t* p = nullptr;
    size_t n = 0;
    explicit PinnedBlock(size_t bytes) : p(static_cast<uint8_t*>(strata::kv::pinned_alloc(bytes))), n(bytes) {}
    PinnedBlock(PinnedBlock&& o) noexcept : p(std::exchange(o.p, nullptr)), n(std::exchange(o.n, 0)) {}
    PinnedBlock(const PinnedBlock&) = delete;
    PinnedBlock& operator=(const PinnedBlock&) = delete;
    PinnedBlock& operator=(PinnedBlock&&) = delete;
    ~PinnedBlock() {
        if (p) strata::kv::pinned_free(p, n);
    }
};

/// The records of a device payload, served from a host copy of [0, records); size() is the whole payload's.
class RecordSource final : public WireSource {
public:
    RecordSource(PinnedBlock block, uint64_t records, uint64_t total)
        : block_(std::move(block)), records_(records), total_(total) {}
    uint64_t size() const override { return total_; }
    bool read(uint8_t* dst, uint64_t offset, size_t bytes) const override {
        if (offset > records_ || bytes > records_ - offset) return false;
        std::memcpy(dst, block_.p + offset, bytes);
        return true;
    }
    const uint8_t* span(uint64_t offset, size_t bytes) const override {
        if (offset > records_ || bytes > records_ - offset) return nullptr;
        return block_.p + offset;
    }

private:
    PinnedBlock block_;
    uint64_t records_;
    uint64_t total_;
};

/// The header and record stream of a device payload in one page-locked host block: a first read of
/// kRecordPrefix bytes (the records are a few KiB plus 4 bytes per token id, so most sessions' fit), and a second
/// read of only the rest when they run longer.  Null (and `error` set) on a refusal or a failed copy.
constexpr uint64_t kRecordPrefix = 64 * 1024;
std::unique_ptr<RecordSource> read_records(const uint8_t* payload, uint64_t bytes, std::string& error) {
    try {
        const uint64_t first = std::min<uint64_t>(bytes, kRecordPrefix);
        PinnedBlock block(kRecordPrefix);
        if (!cuda_ok(cudaMemcpy(block.p, payload, first, cudaMemcpyDefault), error, "header copy")) return nullptr;
        WireHeaderRecord h{};
        if (!conversation_wire_peek(block.p, kWireHeaderRecordBytes, h, error)) return nullptr;
        if (h.blob_pool_off < kWireHeaderRecordBytes || h.blob_pool_off > bytes || h.payload_bytes > bytes) {
            pfail(error, "the header's records or payload run past the " + std::to_string(bytes) + " device bytes");
            return nullptr;
        }
        if (h.blob_pool_off > first) {
            PinnedBlock whole((size_t) h.blob_pool_off);
            std::memcpy(whole.p, block.p, (size_t) first);
            if (!cuda_ok(cudaMemcpy(whole.p + first, payload + first, h.blob_pool_off - first, cudaMemcpyDefault),
                         error, "records copy"))
                return nullptr;
            return std::make_unique<RecordSource>(std::move(whole), h.blob_pool_off, bytes);
        }
        return std::make_unique<RecordSource>(std::move(block), h.blob_pool_off, bytes);
    } catch (const std::bad_alloc&) {
        pfail(error, "no host memory for the payload's records");
        return nullptr;
    }
}

/// One device's share of a mount: copy-kernel segments by engine, plain copies for what the kernels cannot take,
/// and work that must follow the writes.
struct MountBatch {
    std::vector<skv_segment> tma, vec;
    struct Plain {
        void* dst;
        const void* src;
        uint64_t bytes;
    };
    std::vector<Plain> plain;                  // copy-engine copies (the host-authoritative K/V of streamed layers)
    std::vector<skv::ByteRange> small;         // device-to-device pieces too short or unaligned for the engines
    std::vector<std::function<bool(std::string&)>> after;

    /// src (device payload) -> dst through `d` (paged or contiguous).
    void add(const uint8_t* src, const strata::kv::DeviceStream& d, uint64_t from, uint64_t bytes) {
        if (!bytes) return;
        skv_segment sg{};
        sg.src = src;
        sg.bytes = bytes;
        if (d.pages) {
            sg.dst = const_cast<void*>(d.base);
            sg.dst_pages = d.pages + from / d.page_bytes;
            sg.page_bytes = d.page_bytes;
            sg.dst_page_limit = d.page_limit;
            (d.page_bytes >= 1024 && d.page_bytes <= 16384 ? tma : vec).push_back(sg);
            return;
        }
        uint8_t* dst = const_cast<uint8_t*>(static_cast<const uint8_t*>(d.base)) + from;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15u) == 0) {
            sg.dst = dst;
            tma.push_back(sg);
        } else {
            add_device(dst, src, bytes);
        }
    }
    /// A device-to-device piece outside the engines' alignment: a byte-range write, or a copy when it is large.
    void add_device(void* dst, const void* src, uint64_t bytes) {
        if (!bytes) return;
        if (bytes <= skv::kByteRangeMaxBytes)
            small.push_back({static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), bytes});
        else
            plain.push_back(Plain{dst, src, bytes});
    }
    void add_plain(void* dst, const void* src, uint64_t bytes) {
        if (bytes) plain.push_back(Plain{dst, src, bytes});
    }

    /// Enqueue everything on `device`'s legacy stream (phases: issue marked after the last enqueue).
    bool issue(int device, std::string& error) {
        const DeviceScope on(device);
        if (skv_clear_status(device, nullptr) != SKV_OK) return pfail(error, skv_last_error());
        for (auto* list : {&tma, &vec}) {
            const int engine = list == &tma ? SKV_COPY_TMA : SKV_COPY_VEC;
            for (size_t i = 0; i < list->size(); i += SKV_COPY_MAX_SEGMENTS) {
                const int n = (int) std::min<size_t>(SKV_COPY_MAX_SEGMENTS, list->size() - i);
                if (skv_copy(list->data() + i, n, engine, nullptr) != SKV_OK)
                    return pfail(error, std::string("mount copy: ") + skv_last_error());
            }
        }
        if (skv::byte_ranges(small, nullptr) != SKV_OK) return pfail(error, std::string("mount copy: ") + skv_last_error());
        for (const Plain& p : plain)
            if (!cuda_ok(cudaMemcpyAsync(p.dst, p.src, p.bytes, cudaMemcpyDefault, nullptr), error, "mount copy"))
                return false;
        for (auto& fn : after)
            if (!fn(error)) return false;
        return true;
    }
    /// Wait for what issue() enqueued and read the device status.
    static bool complete(int device, std::string& error) {
        const DeviceScope on(device);
        if (!cuda_ok(cudaStreamSynchronize(nullptr), error, "synchronize")) return false;
        return status_clean(device, error);
    }
    bool run(int device, std::string& error) { return issue(device, error) && complete(device, error); }
};

/// One layer's K/V from the payload into `st` (validated already): the mount twin of enqueue_kv_restore.
void mount_kv(const ConversationKv& k, const uint8_t* payload, const wire_detail::BlobTable& blobs,
              const QsaState& st, const ModelGeometry& g, int64_t upto, bool index, MountBatch& b) {
    LayerExtent x;
    std::string ignored;
    layer_extent(st, g, upto, index, x, ignored);
    const auto dst = layer_sources(st);
    const ConversationBuffer* bufs[5] = {&k.k, &k.v, &k.k_scale, &k.v_scale, &k.pooled};
    std::array<const uint8_t*, 5> src{};
    for (int i = 0; i < 5; ++i) {
        const auto it = blobs.find(bufs[i]);
        if (it == blobs.end()) continue;
        src[(size_t) i] = payload + it->second.off;
        if (i < 4 && st.kv_mode != 0)   // the authoritative host copy
            b.add_plain(const_cast<void*>(dst[(size_t) i]), src[(size_t) i], it->second.bytes);
        else
            b.add(src[(size_t) i], layer_stream(st, x, i, dst[(size_t) i]), 0, it->second.bytes);
    }
    if (st.kv_mode == 1) {
        const strata::kernels::KvStreamMap map = st.map;
        b.after.push_back([map](std::string& err) {
            if (skv::stream_reset(map, nullptr) == SKV_OK) return true;
            err = std::string("conversation wire device mount: residency reset: ") + skv_last_error();
            return false;
        });
    } else if (st.kv_mode == 2 && x.cells > 0) {
        const int64_t end = x.cells / x.page_size, begin = std::max<int64_t>(0, end - st.n_slots);
        const auto slots = layer_slots(st);
        for (int i = 0; i < 4; ++i) {
            const auto it = blobs.find(bufs[i]);
            if (it == blobs.end()) continue;
            const uint64_t pb = it->second.bytes / (uint64_t) end;
            for (int64_t p = begin; p < end;) {
                const int64_t sl = p % st.n_slots, run = std::min<int64_t>(end - p, st.n_slots - sl);
                strata::kv::DeviceStream ring;
                ring.base = static_cast<const uint8_t*>(slots[(size_t) i]) + (uint64_t) sl * pb;
                b.add(src[(size_t) i] + (uint64_t) p * pb, ring, 0, (uint64_t) run * pb);
                p += run;
            }
        }
    }
}

/// A checkpoint's running state from the payload into `ss` (validated already): the mount twin of
/// conversation_checkpoint_restore, including the indexer's spare row.
void mount_running(const ConversationCheckpoint& c, const uint8_t* payload, const wire_detail::BlobTable& blobs,
                   const SessionState& ss, const ModelGeometry& g, MountBatch& b) {
    ConversationStateSizes z;
    std::string ignored;
    conversation_session_sizes(g, ss, z, ignored);
    auto at = [&](const std::vector<uint8_t>& v) -> const uint8_t* {
        const auto it = blobs.find(&v);
        return it == blobs.end() ? nullptr : payload + it->second.off;
    };
    auto flat = [](const void* p) {
        strata::kv::DeviceStream s;
        s.base = p;
        return s;
    };
    if (const uint8_t* p = at(c.gdn)) b.add(p, flat(ss.gdn_state), 0, z.gdn);
    if (const uint8_t* p = at(c.ple)) b.add(p, flat(ss.ple_hist), 0, z.ple);
    const uint8_t *tails = at(c.tails), *dead = at(c.dead), *pos = at(c.block_pos);
    const uint64_t block = (uint64_t) strata::kernels::qsa_real_shapes().idx_block;
    for (size_t j = 0; j < owned_count(ss); ++j) {
        const QsaState& st = owned_layer(ss, j);
        if (tails) b.add(tails + j * z.tail, flat(st.idx_tail), 0, z.tail);
        if (dead) b.add(dead + j * z.dead, flat(st.idx_dead), 0, z.dead);
        if (pos) b.add_device(st.idx_block_pos, pos + j * z.block_pos, z.block_pos);
        if (dead && !c.ids.empty())   // the indexer's moving spare row is the dead key again
            b.add(dead + j * z.dead, flat(st.idx_pooled + (c.ids.size() / block) * (size_t) g.idx_key_dim), 0, z.dead);
    }
}

/// Retained checkpoints live on the host (the cache keeps them): copy their blobs out of the payload.
bool fill_retained(ConversationCheckpoint& c, const uint8_t* payload, wire_detail::BlobTable& blobs,
                   std::string& error) {
    for (std::vector<uint8_t>* v : {&c.gdn, &c.ple, &c.tails, &c.dead, &c.block_pos}) {
        const auto it = blobs.find(v);
        if (it == blobs.end()) continue;
        v->resize((size_t) it->second.bytes);
        if (!cuda_ok(cudaMemcpy(v->data(), payload + it->second.off, v->size(), cudaMemcpyDefault), error,
                     "retained checkpoint copy"))
            return false;
        blobs.erase(it);
    }
    for (auto& part : c.stage_parts)
        if (!fill_retained(part, payload, blobs, error)) return false;
    return true;
}

}  // namespace

ConversationRestore conversation_wire_mount_device(const uint8_t* payload, uint64_t bytes, SessionState& ss,
                                                   const ConversationStageSet& stages, const ModelGeometry& g,
                                                   const QsaState& draft, const WireExpect& expect,
                                                   SavedConversation& meta, WireDecoded& info, std::string& error) {
    using R = ConversationRestore;
    PhaseClock phases;
    if (!payload || bytes < kWireHeaderRecordBytes) {
        pfail(error, "no payload, or one shorter than its header");
        return R::invalid;
    }
    const std::unique_ptr<RecordSource> records = read_records(payload, bytes, error);
    if (!records) return R::invalid;
    const RecordSource& src = *records;
    wire_detail::BlobTable blobs;
    if (!wire_detail::decode_shape(src, meta, info, expect, blobs, error)) return R::invalid;
    for (auto& c : meta.checkpoints)
        if (!fill_retained(c, payload, blobs, error)) return R::invalid;
    const wire_detail::BlobTable& table = blobs;
    const SizeOf sizes = [&table](const void* key, uint64_t real) -> uint64_t {
        const auto it = table.find(key);
        return it == table.end() ? real : it->second.bytes;
    };
    if (!snapshot_validate_sized(meta, ss, stages, g, draft, error, sizes)) return R::invalid;

    // every check passed: the writes
    const int64_t upto = (int64_t) meta.live.ids.size();
    const int main_dev = resolve(stages.main_device);
    const int draft_dev = stages.empty() ? main_dev : resolve(stages.draft_device);
    {
        // the main session's layers, its running state and - when it lives on the same device - the draft layer
        // in one batch: one set of launches and one wait
        {
            const DeviceScope on(main_dev);
            if (!device_sync(error)) return R::transfer_failed;
        }
        if (draft_dev != main_dev) {
            const DeviceScope on(draft_dev);
            if (!device_sync(error)) return R::transfer_failed;
        }
        phases.mark_prepared();
        MountBatch b, d;
        for (size_t j = 0; j < owned_count(ss); ++j) mount_kv(meta.kv[j], payload, blobs, owned_layer(ss, j), g, upto, true, b);
        mount_running(meta.live, payload, blobs, ss, g, b);
        mount_kv(meta.kv.back(), payload, blobs, draft, g, upto, false, draft_dev == main_dev ? b : d);
        if (!b.issue(main_dev, error)) return R::transfer_failed;
        if (draft_dev != main_dev && !d.issue(draft_dev, error)) return R::transfer_failed;
        phases.mark_enqueued();
        if (!MountBatch::complete(main_dev, error)) return R::transfer_failed;
        if (draft_dev != main_dev && !MountBatch::complete(draft_dev, error)) return R::transfer_failed;
    }
    const size_t n = meta.live.ids.size();
    ss.ple_prev[0] = n >= 2 ? meta.live.ids[n - 2] : -1;
    ss.ple_prev[1] = n >= 1 ? meta.live.ids[n - 1] : -1;
    for (size_t i = 0; i < meta.stage_parts.size(); ++i) {
        const ConversationStage& stage = stages.stages[i];
        const ConversationStageSnapshot& part = meta.stage_parts[i];
        const int dev = resolve(stage.device);
        {
            const DeviceScope on(dev);
            if (!device_sync(error)) return R::transfer_failed;
        }
        MountBatch b;
        for (size_t j = 0; j < part.kv.size(); ++j)
            mount_kv(part.kv[j], payload, blobs, owned_layer(*stage.session, j), g, upto, true, b);
        mount_running(part.state, payload, blobs, *stage.session, g, b);
        if (!b.run(dev, error)) return R::transfer_failed;
        stage.session->ple_prev[0] = n >= 2 ? meta.live.ids[n - 2] : -1;
        stage.session->ple_prev[1] = n >= 1 ? meta.live.ids[n - 1] : -1;
    }
    phases.finish();
    return R::restored;
}

WireDevicePhases conversation_wire_device_last_phases() { return t_last_phases; }

ConversationRestore conversation_wire_mount_device(const uint8_t* payload, uint64_t bytes, SessionState& ss,
                                                   const ModelGeometry& g, const QsaState& draft,
                                                   const WireExpect& expect, SavedConversation& meta,
                                                   WireDecoded& info, std::string& error) {
    return conversation_wire_mount_device(payload, bytes, ss, {}, g, draft, expect, meta, info, error);
}

}  // namespace strata::core
