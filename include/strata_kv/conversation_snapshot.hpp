// include/strata_kv/conversation_snapshot.hpp - park / mount a conversation between device state and host.
//
// The same functions, signatures and contracts as the reference's
// include/strata/core/conversation_snapshot.hpp:13-141 (per-layer K/V, running-state checkpoints, whole-session
// snapshots with and without a layer split; validate-before-write; transfer_failed after the first write).
//
// What the B200 build changes underneath:
//   * a block-pool layer's K/V is read and written THROUGH QsaState::page_table, so a pool placed by a block
//     allocator (non-identity table) parks and mounts exactly like the reference's identity pool, byte for byte;
//   * the bytes move with the sm_100a copy kernels: one gather launch per device collects every layer's streams
//     and the running state into a device staging image, the copy engine moves it into pinned host segments, and
//     a mount is the reverse (one scatter launch);
//   * the whole-session save / restore issue one batch (and one synchronisation) per device, not one synchronous
//     copy per 16 MiB segment.
// Streamed layers (kv_mode 1 / 2) keep their authoritative K/V in pinned host memory, as in the reference: a park
// copies it, a mount writes it back and then evicts every VRAM block (kv_mode 1, kv_stream_reset) or refills the
// ring's last n_slots pages (kv_mode 2), with the block movers of include/strata_kv/kv_stream.hpp.  A resident
// layer in a block pool (skv_pool_create / skv_pool_wrap) is addressed through its page table; any other resident
// layer is identity-addressed, which is what the reference assumes.
#pragma once

#include "strata_kv/conversation_cache.hpp"
#include "strata_kv/kv_stream.hpp"
#include "strata_kv/types.hpp"

#include <string>

namespace strata::core {

size_t conversation_kv_bytes(const QsaState& state, const ModelGeometry& g, int64_t upto, bool include_index);
bool conversation_kv_save(ConversationKv& image, const QsaState& state, const ModelGeometry& g, int64_t upto,
                          bool include_index, std::string& error, int64_t unchanged_tokens = 0,
                          size_t* reused_bytes = nullptr);
bool conversation_kv_capture_bytes(const ConversationKv& image, const QsaState& state, const ModelGeometry& g,
                                   int64_t upto, bool include_index, size_t& bytes, std::string& error);
bool conversation_kv_validate(const ConversationKv& image, const QsaState& state, const ModelGeometry& g,
                              int64_t upto, bool include_index, std::string& error);
bool conversation_kv_restore(const ConversationKv& image, const QsaState& state, const ModelGeometry& g,
                             int64_t upto, bool include_index, std::string& error);
bool conversation_kv_verify(const ConversationKv& image, const QsaState& state, const ModelGeometry& g,
                            int64_t upto, bool include_index, uint64_t& fingerprint, std::string& error);

struct ConversationStateSizes {
    size_t gdn = 0, ple = 0, tail = 0, dead = 0, block_pos = 0;
};
bool conversation_state_sizes(const ModelGeometry& g, ConversationStateSizes& sizes, std::string& error);
bool conversation_session_sizes(const ModelGeometry& g, const SessionState& session, ConversationStateSizes& sizes,
                                std::string& error);
bool conversation_checkpoint_validate(const ConversationCheckpoint& checkpoint, const SessionState& session,
                                      const ModelGeometry& g, std::string& error);
bool conversation_checkpoint_save(ConversationCheckpoint& checkpoint, const SessionState& session,
                                  const ModelGeometry& g, std::string& error);
bool conversation_checkpoint_restore(const ConversationCheckpoint& checkpoint, SessionState& session,
                                     const ModelGeometry& g, std::string& error);

struct ConversationView {
    const std::vector<int32_t>& ids;
    const std::vector<ConversationImageKey>& images;
    const std::vector<ConversationCheckpoint>& checkpoints;
    bool cvec;
};

struct ConversationStage {
    SessionState* session = nullptr;
    int device = -1;
};
struct ConversationStageSet {
    const ConversationStage* stages = nullptr;
    int64_t count = 0;
    int main_device = -1;
    int draft_device = -1;
    bool empty() const { return stages == nullptr || count <= 0; }
};

bool conversation_snapshot_bytes(const ConversationView& view, const SessionState& session, const ModelGeometry& g,
                                 const QsaState& draft, size_t& bytes, std::string& error);
bool conversation_snapshot_capture_bytes(const ConversationKvReuse& reuse, const ConversationView& view,
                                         const SessionState& session, const ModelGeometry& g, const QsaState& draft,
                                         size_t& bytes, std::string& error);
bool conversation_snapshot_save(SavedConversation& image, const ConversationView& view, const SessionState& session,
                                const ModelGeometry& g, const QsaState& draft, std::string& error,
                                ConversationKvReuse reuse = {}, size_t* reused_bytes = nullptr);
bool conversation_snapshot_validate(const SavedConversation& image, const SessionState& session,
                                    const ModelGeometry& g, const QsaState& draft, std::string& error);
enum class ConversationRestore { restored, invalid, transfer_failed };
ConversationRestore conversation_snapshot_restore(const SavedConversation& image, SessionState& session,
                                                  const ModelGeometry& g, const QsaState& draft, std::string& error);

bool conversation_snapshot_bytes(const ConversationView& view, const SessionState& session,
                                 const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                 size_t& bytes, std::string& error);
bool conversation_snapshot_capture_bytes(const ConversationKvReuse& reuse, const ConversationView& view,
                                         const SessionState& session, const ConversationStageSet& stages,
                                         const ModelGeometry& g, const QsaState& draft, size_t& bytes,
                                         std::string& error);
bool conversation_snapshot_save(SavedConversation& image, const ConversationView& view, const SessionState& session,
                                const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                std::string& error, ConversationKvReuse reuse = {}, size_t* reused_bytes = nullptr);
bool conversation_snapshot_validate(const SavedConversation& image, const SessionState& session,
                                    const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                    std::string& error);
ConversationRestore conversation_snapshot_restore(const SavedConversation& image, SessionState& session,
                                                  const ConversationStageSet& stages, const ModelGeometry& g,
                                                  const QsaState& draft, std::string& error);

}  // namespace strata::core
