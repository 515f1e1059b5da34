// snapshot_detail.hpp - shared pieces of the snapshot layer (internal to libstrata_kv.so).
#pragma once

#include "strata_kv/conversation_snapshot.hpp"
#include "transfer.hpp"

#include <array>
#include <functional>
#include <initializer_list>
#include <string>

namespace strata::core::snapshot_detail {

bool fail(std::string& error, const char* message);
bool checked_product(size_t& out, std::initializer_list<uint64_t> factors);
bool checked_add(size_t& total, size_t n);

/// One layer's snapshot extents: cells (whole pages up to `upto`), indexer rows, and the byte size of each of
/// the five streams k, v, k_scale, v_scale, pooled.
struct LayerExtent {
    int format = 0;
    int64_t cells = 0, pooled_rows = 0, page_size = 0;
    std::array<size_t, 5> bytes{};
};
bool layer_extent(const QsaState& st, const ModelGeometry& g, int64_t upto, bool index, LayerExtent& x,
                  std::string& error);
bool layer_usable(const QsaState& st, const LayerExtent& x, int64_t upto, std::string& error);
/// The authoritative source/target of each stream (device pools in mode 0, host pools otherwise).
std::array<const void*, 5> layer_sources(const QsaState& st);
/// The device-resident pools of each stream (a streamed or ring layer's VRAM slots).
std::array<const void*, 5> layer_slots(const QsaState& st);
/// Stream `i` of a layer as the copy kernels address it (paged through page_table for the K/V streams of a
/// block-pool layer, identity otherwise).
strata::kv::DeviceStream layer_stream(const QsaState& st, const LayerExtent& x, int i, const void* base);

/// The 18-entry geometry key every image and payload carries.
std::array<int64_t, 18> geometry_key(const ModelGeometry& g);

/// Make `device` current for a scope (a negative device, or the current one, changes nothing).
struct DeviceScope {
    int previous = -1;
    explicit DeviceScope(int device);
    ~DeviceScope();
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
};
bool device_sync(std::string& error);

size_t owned_count(const SessionState& ss);
const QsaState& owned_layer(const SessionState& ss, size_t j);
int64_t stage_count(const ConversationStageSet& s);
/// One session's running state for a branch of a given length: the per-buffer sizes (the GDN rows already
/// scaled to the session's carve; tail, dead key and block position per owned QSA layer) and what the session owns.
/// Sizing, validation and saving all read their buffer sizes from this one plan.
struct RunningState {
    ConversationStateSizes per;
    size_t layers = 0;        ///< QSA layers the session owns
    bool keeps_ple = false;   ///< the session keeps a PLE history
    size_t gdn() const { return per.gdn; }
    size_t ple() const { return keeps_ple ? per.ple : 0; }
    size_t tails() const { return layers * per.tail; }
    size_t dead() const { return layers * per.dead; }
    size_t block_pos() const { return layers * per.block_pos; }
};
/// The plan of `ss`'s running state for a `tokens`-long branch; refused (error set) when the session cannot hold
/// one that long: a carve outside the model, too few cells, a missing buffer, no spare indexer row.
bool running_state(const SessionState& ss, const ModelGeometry& g, size_t tokens, RunningState& rs, std::string& error);
/// Image start positions strictly increasing and inside [0, tokens).
bool images_ordered(const std::vector<ConversationImageKey>& images, size_t tokens);
/// The main session plus the stages tile [0, n_layers) in order.
bool stages_tile(const ConversationStageSet& stages, const SessionState& main_ss, const ModelGeometry& g,
                 std::string& error);
/// The live branch and every retained checkpoint are consistent prefixes of it.
bool view_ok(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
             const ModelGeometry& g, std::string& error);

/// The byte count validation sees for a buffer or vector of an image: its own size(), or a side table's for a
/// shape image whose bytes live elsewhere (a device payload).  key = the ConversationBuffer / std::vector.
using SizeOf = std::function<uint64_t(const void* key, uint64_t real)>;
inline uint64_t own_size(const void*, uint64_t real) { return real; }
bool kv_validate_sized(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                       bool index, std::string& error, const SizeOf& size_of);
bool checkpoint_validate_sized(const ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g,
                               std::string& error, const SizeOf& size_of);
bool snapshot_validate_sized(const SavedConversation& image, const SessionState& ss, const ConversationStageSet& stages,
                             const ModelGeometry& g, const QsaState& draft, std::string& error, const SizeOf& size_of);

/// Queue one layer's save / restore into a batch (validation happens here, before anything is queued).
bool enqueue_kv_save(ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto, bool index,
                     strata::kv::Transfer& t, std::string& error, int64_t unchanged, size_t* reused_bytes);
bool enqueue_kv_restore(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                        bool index, strata::kv::Transfer& t, std::string& error);

}  // namespace strata::core::snapshot_detail
