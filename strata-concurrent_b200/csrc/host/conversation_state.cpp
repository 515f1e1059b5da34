// conversation_state.cpp - running-state checkpoints and whole-session snapshots
// (include/strata_kv/conversation_snapshot.hpp; the reference's src/core/conversation_state.cpp:180-507).
//
// Validation and sizing follow the reference's rules (every stage, every checkpoint and the draft are checked
// before the first byte moves; byte estimates count exactly what the image will hold).  Movement is batched per
// device: a park of the main session is ONE transfer batch (running state + every owned layer's K/V: one or two
// gather launches, the device->host copies, one synchronisation), then the draft's device, then each stage's.
#include "snapshot_detail.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <limits>

namespace strata::core {
namespace snapshot_detail {

std::array<int64_t, 18> geometry_key(const ModelGeometry& g) {
    return {g.n_embd,    g.n_layers,       g.qsa_interval,  g.ssm_state_size, g.ssm_k_heads, g.ssm_v_heads,
            g.ssm_d_conv, g.ssm_conv_channels, g.ssm_value_dim, g.n_head,   g.n_head_kv,   g.head_dim,
            g.idx_q_heads, g.idx_key_dim,   g.hc,            g.hc_lr,      g.n_expert,    g.n_ff};
}

DeviceScope::DeviceScope(int device) {
    int cur = 0;
    if (device >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != device && cudaSetDevice(device) == cudaSuccess)
        previous = cur;
}
DeviceScope::~DeviceScope() {
    if (previous >= 0) cudaSetDevice(previous);
}

bool device_sync(std::string& error) {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) return true;
    (void) cudaGetLastError();
    error = std::string("conversation snapshot synchronize: ") + cudaGetErrorString(e);
    return false;
}

size_t owned_count(const SessionState& ss) { return (size_t) std::max<int64_t>(ss.qsa_alloc, 0); }
const QsaState& owned_layer(const SessionState& ss, size_t j) { return ss.qsa_states[(size_t) ss.qsa_ord0 + j]; }
int64_t stage_count(const ConversationStageSet& s) { return s.empty() ? 0 : s.count; }

/// Image starts strictly increasing and inside the token range.
bool images_ordered(const std::vector<ConversationImageKey>& images, size_t tokens) {
    int64_t last = -1;
    for (const auto& im : images) {
        if (im.start < 0 || im.start <= last || (uint64_t) im.start >= tokens) return false;
        last = im.start;
    }
    return true;
}

/// The session can hold a `tokens`-long running state: sizes, pointers, indexer capacity.
bool running_targets(const SessionState& ss, const ModelGeometry& g, size_t tokens, ConversationStateSizes& z,
                     std::string& error) {
    if (!conversation_session_sizes(g, ss, z, error)) return false;
    if (ss.max_cells < 0 || tokens > (uint64_t) ss.max_cells || (z.gdn && !ss.gdn_state) ||
        (owned_count(ss) && !ss.qsa_states))
        return fail(error, "invalid session running-state targets");
    const uint64_t block = (uint64_t) strata::kernels::qsa_real_shapes().idx_block;
    for (size_t j = 0; j < owned_count(ss); ++j) {
        const QsaState& st = owned_layer(ss, j);
        size_t pooled = 0;
        if (!st.idx_tail || !st.idx_dead || !st.idx_block_pos || !st.idx_pooled || st.max_cells < 0 ||
            tokens > (uint64_t) st.max_cells ||
            (tokens && tokens / block >= (uint64_t) std::max<int64_t>(0, st.idx_pooled_rows)) ||
            !checked_product(pooled, {tokens / block + 1, (uint64_t) g.idx_key_dim, sizeof(float)}))
            return fail(error, "invalid indexer running-state target");
    }
    return true;
}

/// The main session plus the stages tile [0, n_layers) in order, each stage's carve consistent.
bool stages_tile(const ConversationStageSet& stages, const SessionState& main_ss, const ModelGeometry& g,
                 std::string& error) {
    if (stages.empty()) return true;
    if (stages.count > (int64_t) (std::numeric_limits<size_t>::max() / sizeof(ConversationStageSnapshot)))
        return fail(error, "too many layer-split stages");
    const int64_t n_qsa = g.n_qsa_layers();
    int64_t next = main_ss.layer_hi;
    for (int64_t i = 0; i < stages.count; ++i) {
        const SessionState* ss = stages.stages[i].session;
        if (!ss) return fail(error, "layer-split stage has no session");
        ConversationStateSizes z;
        if (!conversation_session_sizes(g, *ss, z, error)) return false;
        if (ss->layer_lo != next || ss->layer_lo >= ss->layer_hi || ss->layer_hi > g.n_layers)
            return fail(error, "layer-split stages do not tile the model");
        if (ss->qsa_ord0 < ss->layer_lo / std::max<int64_t>(g.qsa_interval, 1))
            return fail(error, "layer-split stage carve starts before its layer range");
        if (ss->qsa_alloc > n_qsa - ss->qsa_ord0) return fail(error, "layer-split stage carve past the last QSA layer");
        next = ss->layer_hi;
    }
    if (next != g.n_layers) return fail(error, "layer-split stages do not cover the whole model");
    return true;
}

/// A later stage's share of a snapshot estimate.
bool stage_estimate(const SessionState& ss, const ModelGeometry& g, int64_t upto, size_t& total, std::string& error) {
    ConversationStateSizes z;
    if (!conversation_session_sizes(g, ss, z, error) || !running_targets(ss, g, (size_t) upto, z, error)) return false;
    const size_t layers = owned_count(ss);
    size_t dir = 0, tails = 0, dead = 0, pos = 0, ids = 0;
    if (!checked_product(dir, {layers, sizeof(ConversationKv)}) || !checked_product(tails, {layers, z.tail}) ||
        !checked_product(dead, {layers, z.dead}) || !checked_product(pos, {layers, z.block_pos}) ||
        !checked_product(ids, {(uint64_t) upto, sizeof(int32_t)}))
        return fail(error, "stage byte count overflow");
    for (size_t n : {dir, ids, tails, dead, pos, z.gdn, ss.ple_hist ? z.ple : (size_t) 0})
        if (!checked_add(total, n)) return fail(error, "stage byte count overflow");
    for (size_t j = 0; j < layers; ++j) {
        const size_t n = conversation_kv_bytes(owned_layer(ss, j), g, upto, true);
        if (!n || !checked_add(total, n)) return fail(error, "invalid or overflowing stage K/V byte estimate");
    }
    return true;
}

/// The live branch and every retained checkpoint are prefixes of it, with the right per-stage parts.
bool view_ok(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
             const ModelGeometry& g, std::string& error) {
    ConversationStateSizes z;
    if (!running_targets(ss, g, view.ids.size(), z, error)) return false;
    if (view.ids.empty() || !images_ordered(view.images, view.ids.size()) ||
        std::any_of(view.ids.begin(), view.ids.end(), [](int32_t id) { return id < 0; }))
        return fail(error, "invalid live token/image metadata");
    for (const auto& c : view.checkpoints) {
        if (c.ids.empty() || c.ids.size() > view.ids.size() || !std::equal(c.ids.begin(), c.ids.end(), view.ids.begin()))
            return fail(error, "checkpoint is not a live token prefix");
        if ((int64_t) c.stage_parts.size() != stage_count(stages))
            return fail(error, stages.empty() ? "layer-split parking is not supported"
                                              : "checkpoint is missing a layer-split stage part");
        if (!conversation_checkpoint_validate(c, ss, g, error)) return false;
        for (size_t i = 0; i < c.stage_parts.size(); ++i) {
            const ConversationCheckpoint& part = c.stage_parts[i];
            if (part.ids.size() != c.ids.size() || !part.imgs.empty() || !part.stage_parts.empty())
                return fail(error, "layer-split checkpoint part is not a live token prefix");
            if (!conversation_checkpoint_validate(part, *stages.stages[i].session, g, error)) return false;
        }
        size_t k = 0;
        for (const auto& key : view.images) {
            if ((uint64_t) key.start >= c.ids.size()) break;
            if (k >= c.imgs.size() || !(c.imgs[k++] == key)) return fail(error, "checkpoint image identity differs");
        }
        if (k != c.imgs.size()) return fail(error, "checkpoint image prefix differs");
    }
    return true;
}

bool checkpoint_meta_bytes(const ConversationCheckpoint& c, size_t& total) {
    size_t ids = 0, imgs = 0, parts = 0;
    if (!checked_product(ids, {c.ids.size(), sizeof(int32_t)}) ||
        !checked_product(imgs, {c.imgs.size(), sizeof(ConversationImageKey)}))
        return false;
    for (size_t n : {ids, imgs, c.gdn.size(), c.ple.size(), c.tails.size(), c.dead.size(), c.block_pos.size()})
        if (!checked_add(total, n)) return false;
    if (!checked_product(parts, {c.stage_parts.capacity(), sizeof(ConversationCheckpoint)}) || !checked_add(total, parts))
        return false;
    for (const auto& p : c.stage_parts)
        if (!checkpoint_meta_bytes(p, total)) return false;
    return true;
}

/// The main session's share: its running state, metadata, every owned layer's K/V and the draft's.
bool main_estimate(const ConversationView& view, const SessionState& ss, const ModelGeometry& g, const QsaState& draft,
                   size_t& bytes, std::string& error) {
    ConversationStateSizes z;
    if (!conversation_session_sizes(g, ss, z, error)) return false;
    const uint64_t qsa = owned_count(ss);
    size_t ids = 0, imgs = 0, cps = 0, layers = 0, tails = 0, dead = 0, pos = 0;
    if (!checked_product(ids, {view.ids.size(), sizeof(int32_t)}) ||
        !checked_product(imgs, {view.images.size(), sizeof(ConversationImageKey)}) ||
        !checked_product(cps, {view.checkpoints.size(), sizeof(ConversationCheckpoint)}) ||
        !checked_product(layers, {qsa + 1, sizeof(ConversationKv)}) || !checked_product(tails, {qsa, z.tail}) ||
        !checked_product(dead, {qsa, z.dead}) || !checked_product(pos, {qsa, z.block_pos}))
        return fail(error, "snapshot metadata byte count overflow");
    for (size_t n : {ids, imgs, cps, layers, tails, dead, pos, z.gdn, ss.ple_hist ? z.ple : (size_t) 0})
        if (!checked_add(bytes, n)) return fail(error, "snapshot byte count overflow");
    for (const auto& c : view.checkpoints)
        if (!checkpoint_meta_bytes(c, bytes)) return fail(error, "checkpoint byte count overflow");
    const int64_t upto = (int64_t) view.ids.size();
    for (uint64_t i = 0; i <= qsa; ++i) {
        const QsaState& st = i == qsa ? draft : owned_layer(ss, (size_t) i);
        const size_t n = conversation_kv_bytes(st, g, upto, i != qsa);
        if (!n || !checked_add(bytes, n)) return fail(error, "invalid or overflowing K/V byte estimate");
    }
    return true;
}

/// Queue a checkpoint's running state (save direction) into `t`.
bool enqueue_checkpoint_save(ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g,
                             strata::kv::Transfer& t, std::string& error) {
    ConversationStateSizes z;
    if (!running_targets(ss, g, c.ids.size(), z, error)) return false;
    const size_t layers = owned_count(ss);
    c.gdn.resize(z.gdn);
    c.ple.resize(ss.ple_hist ? z.ple : 0);
    c.tails.resize(layers * z.tail);
    c.dead.resize(layers * z.dead);
    c.block_pos.resize(layers * z.block_pos);
    auto dev = [](const void* p) {
        strata::kv::DeviceStream s;
        s.base = p;
        return s;
    };
    if (!c.gdn.empty()) t.save(dev(ss.gdn_state), 0, c.gdn.size(), c.gdn.data());
    if (!c.ple.empty()) t.save(dev(ss.ple_hist), 0, c.ple.size(), c.ple.data());
    for (size_t j = 0; j < layers; ++j) {
        const QsaState& st = owned_layer(ss, j);
        t.save(dev(st.idx_tail), 0, z.tail, c.tails.data() + j * z.tail);
        t.save(dev(st.idx_dead), 0, z.dead, c.dead.data() + j * z.dead);
        t.save(dev(st.idx_block_pos), 0, z.block_pos, c.block_pos.data() + j * z.block_pos);
    }
    return true;
}

}  // namespace snapshot_detail

using namespace snapshot_detail;

// ------------------------------------------------------------------------------------------------ sizes

bool conversation_state_sizes(const ModelGeometry& g, ConversationStateSizes& z, std::string& error) {
    z = {};
    const auto key = geometry_key(g);
    for (size_t i = 0; i < key.size(); ++i)
        if (key[i] < 0 || (i != 1 && key[i] == 0)) return fail(error, "invalid model geometry");
    size_t recurrence = 0, convolution = 0;
    if (!checked_product(recurrence, {(uint64_t) g.ssm_state_size, (uint64_t) g.ssm_v_heads, (uint64_t) g.ssm_state_size}) ||
        !checked_product(convolution, {(uint64_t) g.ssm_conv_channels, (uint64_t) (g.ssm_d_conv - 1)}) ||
        !checked_add(recurrence, convolution) ||
        !checked_product(z.gdn, {(uint64_t) g.n_gdn_layers(), recurrence, sizeof(float)}) ||
        !checked_product(z.ple, {(uint64_t) strata::kernels::NG_HIST, (uint64_t) strata::kernels::NG_HC_DIM, sizeof(float)}) ||
        !checked_product(z.tail, {(uint64_t) (strata::kernels::qsa_real_shapes().idx_block - 1), (uint64_t) g.idx_key_dim,
                                  sizeof(float)}) ||
        !checked_product(z.dead, {(uint64_t) g.idx_key_dim, sizeof(float)}))
        return fail(error, "running-state byte count overflow");
    z.block_pos = sizeof(int32_t);
    size_t all = 0;
    if (!checked_product(all, {(uint64_t) g.n_qsa_layers(), z.tail}) ||
        !checked_product(all, {(uint64_t) g.n_qsa_layers(), z.dead}) ||
        !checked_product(all, {(uint64_t) g.n_qsa_layers(), z.block_pos}))
        return fail(error, "indexer byte count overflow");
    return true;
}

bool conversation_session_sizes(const ModelGeometry& g, const SessionState& ss, ConversationStateSizes& z,
                                std::string& error) {
    if (!conversation_state_sizes(g, z, error)) return false;
    const int64_t n_gdn = g.n_gdn_layers(), n_qsa = g.n_qsa_layers();
    if (ss.gdn_alloc < 0 || ss.gdn_alloc > n_gdn || ss.qsa_ord0 < 0 || ss.qsa_alloc < 0 || ss.qsa_ord0 > n_qsa ||
        ss.qsa_alloc > n_qsa - ss.qsa_ord0)
        return fail(error, "invalid session layer carve");
    z.gdn = n_gdn > 0 ? z.gdn / (size_t) n_gdn * (size_t) ss.gdn_alloc : 0;
    return true;
}

// ------------------------------------------------------------------------------------------------ checkpoints

bool conversation_checkpoint_validate(const ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g,
                                      std::string& error) {
    return checkpoint_validate_sized(c, ss, g, error, own_size);
}

bool snapshot_detail::checkpoint_validate_sized(const ConversationCheckpoint& c, const SessionState& ss,
                                                const ModelGeometry& g, std::string& error, const SizeOf& size_of) {
    ConversationStateSizes z;
    if (!running_targets(ss, g, c.ids.size(), z, error)) return false;
    const size_t layers = owned_count(ss);
    auto n = [&](const std::vector<uint8_t>& v) { return size_of(&v, v.size()); };
    if (n(c.gdn) != z.gdn || n(c.ple) != (ss.ple_hist ? z.ple : 0) || n(c.tails) != layers * z.tail ||
        n(c.dead) != layers * z.dead || n(c.block_pos) != layers * z.block_pos || !images_ordered(c.imgs, c.ids.size()))
        return fail(error, "invalid checkpoint running-state payload");
    return true;
}

bool conversation_checkpoint_save(ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g,
                                  std::string& error) {
    strata::kv::Transfer t;
    if (!enqueue_checkpoint_save(c, ss, g, t, error)) return false;
    return t.run(error, "conversation snapshot running-state copy");
}

bool conversation_checkpoint_restore(const ConversationCheckpoint& c, SessionState& ss, const ModelGeometry& g,
                                     std::string& error) {
    if (!conversation_checkpoint_validate(c, ss, g, error)) return false;
    ConversationStateSizes z;
    if (!conversation_session_sizes(g, ss, z, error)) return false;
    auto dev = [](const void* p) {
        strata::kv::DeviceStream s;
        s.base = p;
        return s;
    };
    strata::kv::Transfer t;
    if (!c.gdn.empty()) t.restore(c.gdn.data(), 0, c.gdn.size(), dev(ss.gdn_state));
    if (!c.ple.empty()) t.restore(c.ple.data(), 0, c.ple.size(), dev(ss.ple_hist));
    const uint64_t block = (uint64_t) strata::kernels::qsa_real_shapes().idx_block;
    for (size_t j = 0; j < owned_count(ss); ++j) {
        const QsaState& st = owned_layer(ss, j);
        t.restore(c.tails.data() + j * z.tail, 0, z.tail, dev(st.idx_tail));
        t.restore(c.dead.data() + j * z.dead, 0, z.dead, dev(st.idx_dead));
        t.restore(c.block_pos.data() + j * z.block_pos, 0, z.block_pos, dev(st.idx_block_pos));
        if (!c.ids.empty()) {
            // the indexer's moving spare row is the dead key again (the row the next block will pool into)
            const size_t row = c.ids.size() / block;
            t.restore(c.dead.data() + j * z.dead, 0, z.dead, dev(st.idx_pooled + row * (size_t) g.idx_key_dim));
        }
    }
    if (!t.run(error, "conversation snapshot running-state copy")) return false;
    const size_t n = c.ids.size();
    ss.ple_prev[0] = n >= 2 ? c.ids[n - 2] : -1;
    ss.ple_prev[1] = n >= 1 ? c.ids[n - 1] : -1;
    return device_sync(error);
}

// ------------------------------------------------------------------------------------------------ snapshots

bool conversation_snapshot_bytes(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
                                 const ModelGeometry& g, const QsaState& draft, size_t& bytes, std::string& error) {
    bytes = 0;
    if (!stages_tile(stages, ss, g, error) || !view_ok(view, ss, stages, g, error) ||
        !main_estimate(view, ss, g, draft, bytes, error))
        return false;
    if (!stages.empty()) {
        size_t dir = 0;
        if (!checked_product(dir, {(uint64_t) stages.count, sizeof(ConversationStageSnapshot)}) || !checked_add(bytes, dir))
            return fail(error, "layer-split stage directory overflow");
    }
    for (int64_t i = 0; i < stage_count(stages); ++i)
        if (!stage_estimate(*stages.stages[i].session, g, (int64_t) view.ids.size(), bytes, error)) return false;
    return true;
}

bool conversation_snapshot_bytes(const ConversationView& view, const SessionState& ss, const ModelGeometry& g,
                                 const QsaState& draft, size_t& bytes, std::string& error) {
    return conversation_snapshot_bytes(view, ss, {}, g, draft, bytes, error);
}

bool conversation_snapshot_capture_bytes(const ConversationKvReuse& reuse, const ConversationView& view,
                                         const SessionState& ss, const ConversationStageSet& stages,
                                         const ModelGeometry& g, const QsaState& draft, size_t& bytes,
                                         std::string& error) {
    if (!conversation_snapshot_bytes(view, ss, stages, g, draft, bytes, error)) return false;
    if (reuse.kv.empty()) return true;
    const size_t layers = owned_count(ss) + 1;   // the main session's layers and the draft; never a stage's
    if (reuse.kv.size() != layers || reuse.unchanged_tokens < 0 || reuse.unchanged_tokens > reuse.captured_tokens ||
        reuse.unchanged_tokens > (int64_t) view.ids.size())
        return fail(error, "invalid retained K/V prefix");
    for (size_t i = 0; i < layers; ++i) {
        const bool index = i + 1 != layers;
        const QsaState& st = index ? owned_layer(ss, i) : draft;
        if (!conversation_kv_validate(reuse.kv[i], st, g, reuse.captured_tokens, index, error)) return false;
        const size_t fresh = conversation_kv_bytes(st, g, (int64_t) view.ids.size(), index);
        size_t retained = 0;
        if (!conversation_kv_capture_bytes(reuse.kv[i], st, g, (int64_t) view.ids.size(), index, retained, error))
            return false;
        bytes -= fresh;
        if (!checked_add(bytes, retained)) return fail(error, "retained K/V allocation overflow");
    }
    size_t dir = 0;
    if (!checked_product(dir, {reuse.kv.capacity() - layers, sizeof(ConversationKv)}) || !checked_add(bytes, dir))
        return fail(error, "retained K/V directory overflow");
    return true;
}

bool conversation_snapshot_capture_bytes(const ConversationKvReuse& reuse, const ConversationView& view,
                                         const SessionState& ss, const ModelGeometry& g, const QsaState& draft,
                                         size_t& bytes, std::string& error) {
    return conversation_snapshot_capture_bytes(reuse, view, ss, {}, g, draft, bytes, error);
}

bool conversation_snapshot_save(SavedConversation& image, const ConversationView& view, const SessionState& ss,
                                const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                std::string& error, ConversationKvReuse reuse, size_t* reused_bytes) {
    size_t estimate = 0;
    if (!conversation_snapshot_capture_bytes(reuse, view, ss, stages, g, draft, estimate, error)) return false;
    SavedConversation captured;   // built aside: a failure publishes nothing
    captured.geometry = geometry_key(g);
    captured.layer_lo = ss.layer_lo;
    captured.layer_hi = ss.layer_hi;
    captured.live.ids = view.ids;
    captured.live.imgs = view.images;
    captured.cvec = view.cvec;
    captured.checkpoints = view.checkpoints;
    const int64_t unchanged = reuse.kv.empty() ? 0 : reuse.unchanged_tokens;
    captured.kv = std::move(reuse.kv);
    const size_t layers = owned_count(ss);
    captured.kv.resize(layers + 1);
    const int64_t upto = (int64_t) view.ids.size();
    {
        const DeviceScope on(stages.main_device);
        if (!device_sync(error)) return false;
        strata::kv::Transfer t;
        if (!enqueue_checkpoint_save(captured.live, ss, g, t, error)) return false;
        for (size_t j = 0; j < layers; ++j)
            if (!enqueue_kv_save(captured.kv[j], owned_layer(ss, j), g, upto, true, t, error, unchanged, reused_bytes))
                return false;
        if (!t.run(error, "conversation snapshot copy")) return false;
    }
    {
        // the draft lives on the last stage's device when the model is split; its final cell may not have been
        // computed when the output cap was reached, so that page is refreshed even on an unchanged prefix
        const DeviceScope on(stages.empty() ? -1 : stages.draft_device);
        if (!stages.empty() && !device_sync(error)) return false;
        strata::kv::Transfer t;
        if (!enqueue_kv_save(captured.kv.back(), draft, g, upto, false, t, error, std::max<int64_t>(0, unchanged - 1),
                             reused_bytes) ||
            !t.run(error, "conversation snapshot copy"))
            return false;
    }
    captured.stage_parts.resize((size_t) stage_count(stages));
    for (int64_t i = 0; i < stage_count(stages); ++i) {
        const ConversationStage& stage = stages.stages[i];
        const SessionState& sss = *stage.session;
        ConversationStageSnapshot& part = captured.stage_parts[(size_t) i];
        part.layer_lo = sss.layer_lo;
        part.layer_hi = sss.layer_hi;
        part.state.ids = view.ids;
        part.kv.resize(owned_count(sss));
        const DeviceScope on(stage.device);
        if (!device_sync(error)) return false;
        strata::kv::Transfer t;
        if (!enqueue_checkpoint_save(part.state, sss, g, t, error)) return false;
        for (size_t j = 0; j < part.kv.size(); ++j)
            if (!enqueue_kv_save(part.kv[j], owned_layer(sss, j), g, upto, true, t, error, 0, nullptr)) return false;
        if (!t.run(error, "conversation snapshot copy")) return false;
    }
    image = std::move(captured);
    return true;
}

bool conversation_snapshot_save(SavedConversation& image, const ConversationView& view, const SessionState& ss,
                                const ModelGeometry& g, const QsaState& draft, std::string& error,
                                ConversationKvReuse reuse, size_t* reused_bytes) {
    return conversation_snapshot_save(image, view, ss, {}, g, draft, error, std::move(reuse), reused_bytes);
}

bool conversation_snapshot_validate(const SavedConversation& image, const SessionState& ss,
                                    const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                    std::string& error) {
    return snapshot_validate_sized(image, ss, stages, g, draft, error, own_size);
}

bool snapshot_detail::snapshot_validate_sized(const SavedConversation& image, const SessionState& ss,
                                              const ConversationStageSet& stages, const ModelGeometry& g,
                                              const QsaState& draft, std::string& error, const SizeOf& size_of) {
    if (!stages_tile(stages, ss, g, error)) return false;
    if (!image.live.stage_parts.empty()) return fail(error, "layer-split parking is not supported");
    if ((int64_t) image.stage_parts.size() != stage_count(stages))
        return fail(error, stages.empty() ? "layer-split parking is not supported"
                                          : "snapshot is missing a layer-split stage part");
    if (image.geometry != geometry_key(g)) return fail(error, "incompatible runtime geometry");
    if (image.layer_lo != ss.layer_lo || image.layer_hi != ss.layer_hi)
        return fail(error, "snapshot from another session layer range");
    const ConversationView view{image.live.ids, image.live.imgs, image.checkpoints, image.cvec};
    if (!view_ok(view, ss, stages, g, error) || !checkpoint_validate_sized(image.live, ss, g, error, size_of))
        return false;
    const size_t layers = owned_count(ss);
    if (image.kv.size() != layers + 1) return fail(error, "invalid K/V layer count");
    const int64_t upto = (int64_t) image.live.ids.size();
    for (size_t j = 0; j < layers; ++j)
        if (!kv_validate_sized(image.kv[j], owned_layer(ss, j), g, upto, true, error, size_of)) return false;
    if (!kv_validate_sized(image.kv.back(), draft, g, upto, false, error, size_of)) return false;
    for (size_t i = 0; i < image.stage_parts.size(); ++i) {
        const ConversationStageSnapshot& part = image.stage_parts[i];
        const SessionState& sss = *stages.stages[i].session;
        if (part.layer_lo != sss.layer_lo || part.layer_hi != sss.layer_hi)
            return fail(error, "layer-split stage part from another session layer range");
        if (!part.state.imgs.empty() || !part.state.stage_parts.empty() ||
            part.state.ids.size() != image.live.ids.size() ||
            !std::equal(part.state.ids.begin(), part.state.ids.end(), image.live.ids.begin()))
            return fail(error, "layer-split stage part is not a live token prefix");
        if (!checkpoint_validate_sized(part.state, sss, g, error, size_of)) return false;
        if (part.kv.size() != owned_count(sss)) return fail(error, "invalid layer-split stage K/V layer count");
        for (size_t j = 0; j < part.kv.size(); ++j)
            if (!kv_validate_sized(part.kv[j], owned_layer(sss, j), g, upto, true, error, size_of)) return false;
    }
    return true;
}

bool conversation_snapshot_validate(const SavedConversation& image, const SessionState& ss, const ModelGeometry& g,
                                    const QsaState& draft, std::string& error) {
    return conversation_snapshot_validate(image, ss, {}, g, draft, error);
}

ConversationRestore conversation_snapshot_restore(const SavedConversation& image, SessionState& ss,
                                                  const ConversationStageSet& stages, const ModelGeometry& g,
                                                  const QsaState& draft, std::string& error) {
    if (!conversation_snapshot_validate(image, ss, stages, g, draft, error)) return ConversationRestore::invalid;
    const int64_t upto = (int64_t) image.live.ids.size();
    {
        const DeviceScope on(stages.main_device);
        if (!device_sync(error)) return ConversationRestore::transfer_failed;
        strata::kv::Transfer t;
        for (size_t j = 0; j < owned_count(ss); ++j)
            if (!enqueue_kv_restore(image.kv[j], owned_layer(ss, j), g, upto, true, t, error))
                return ConversationRestore::transfer_failed;
        if (!t.run(error, "conversation snapshot copy")) return ConversationRestore::transfer_failed;
    }
    {
        const DeviceScope on(stages.empty() ? -1 : stages.draft_device);
        strata::kv::Transfer t;
        if (!enqueue_kv_restore(image.kv.back(), draft, g, upto, false, t, error) ||
            !t.run(error, "conversation snapshot copy"))
            return ConversationRestore::transfer_failed;
    }
    {
        const DeviceScope on(stages.main_device);
        if (!conversation_checkpoint_restore(image.live, ss, g, error)) return ConversationRestore::transfer_failed;
    }
    for (size_t i = 0; i < image.stage_parts.size(); ++i) {
        const ConversationStage& stage = stages.stages[i];
        const ConversationStageSnapshot& part = image.stage_parts[i];
        const DeviceScope on(stage.device);
        strata::kv::Transfer t;
        for (size_t j = 0; j < part.kv.size(); ++j)
            if (!enqueue_kv_restore(part.kv[j], owned_layer(*stage.session, j), g, upto, true, t, error))
                return ConversationRestore::transfer_failed;
        if (!t.run(error, "conversation snapshot copy")) return ConversationRestore::transfer_failed;
        if (!conversation_checkpoint_restore(part.state, *stage.session, g, error))
            return ConversationRestore::transfer_failed;
    }
    return ConversationRestore::restored;
}

ConversationRestore conversation_snapshot_restore(const SavedConversation& image, SessionState& ss,
                                                  const ModelGeometry& g, const QsaState& draft, std::string& error) {
    return conversation_snapshot_restore(image, ss, {}, g, draft, error);
}

}  // namespace strata::core
