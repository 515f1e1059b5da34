// conversation_state.cpp - running-state checkpoints and whole-session snapshots
// (include/strata_kv/conversation_snapshot.hpp; the C++ API of the reference's src/core/conversation_state.cpp).
//
// Accounting and refusals.  Every question this file answers about a session - can it hold a branch of T tokens,
// how big is its share of an image, does an image's running state fit it - is read off ONE plan of that session's
// running state (RunningState, built by running_state) and summed in ONE checked byte ledger (Ledger).  Sizing
// adds plan entries to a ledger, validation compares an image's buffers with the same entries, and a save sizes
// its buffers from them, so the three cannot disagree about a buffer.  The refusal set is the reference's: any
// failed check refuses the whole call before the first byte moves.  The reasons are this file's own words.
//
// Movement is batched per device: a park of the main session is ONE transfer batch (running state + every owned
// layer's K/V: one or two gather launches, the device->host copies, one synchronisation), then the draft's device,
// then each later stage's.
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
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess && strata::kv::transfer_fault(strata::kv::TransferStep::device_sync)) e = cudaErrorUnknown;
    if (e == cudaSuccess) return true;
    (void) cudaGetLastError();
    error = std::string("conversation snapshot synchronize: ") + cudaGetErrorString(e);
    return false;
}

size_t owned_count(const SessionState& ss) { return (size_t) std::max<int64_t>(ss.qsa_alloc, 0); }
const QsaState& owned_layer(const SessionState& ss, size_t j) { return ss.qsa_states[(size_t) ss.qsa_ord0 + j]; }
int64_t stage_count(const ConversationStageSet& s) { return s.empty() ? 0 : s.count; }

namespace {

/// A byte total that goes sour on the first overflowing or invalid term and stays sour.
class Ledger {
public:
    /// `count` entries of `each` bytes.
    Ledger& add(uint64_t count, uint64_t each) {
        size_t n = 0;
        if (!checked_product(n, {count, each})) ok_ = false;
        return add(n);
    }
    Ledger& add(size_t n) {
        if (ok_ && !checked_add(total_, n)) ok_ = false;
        return *this;
    }
    /// A term whose 0 means "invalid" (a K/V estimate of a layer that cannot be parked).
    Ledger& add_estimate(size_t n) {
        if (n == 0) ok_ = false;
        return add(n);
    }
    bool ok() const { return ok_; }
    size_t total() const { return total_; }

private:
    size_t total_ = 0;
    bool ok_ = true;
};

/// Why one owned QSA layer's indexer cannot carry a `tokens`-long branch (its buffers, its cell capacity, the
/// pooled rows the branch fills plus the spare row the next block pools into), or null when it can.
const char* indexer_fault(const QsaState& st, const ModelGeometry& g, uint64_t tokens) {
    if (!st.idx_tail || !st.idx_dead || !st.idx_block_pos || !st.idx_pooled) return "an indexer buffer is missing";
    if (st.max_cells < 0 || tokens > (uint64_t) st.max_cells) return "a QSA layer holds fewer cells than the branch";
    const uint64_t rows_used = tokens / (uint64_t) strata::kernels::qsa_real_shapes().idx_block;
    if (tokens > 0 && rows_used + 1 > (uint64_t) std::max<int64_t>(st.idx_pooled_rows, 0))
        return "the indexer has no spare pooled row past the branch";
    size_t pooled = 0;
    if (!checked_product(pooled, {rows_used + 1, (uint64_t) g.idx_key_dim, sizeof(float)}))
        return "the indexer's pooled rows overflow a byte count";
    return nullptr;
}

/// Why checkpoint `c` cannot sit beside the live branch of `view` in an image with `stages` later stages, as far
/// as its own shape tells (the running-state sizes are checked against the sessions separately), or null.
const char* checkpoint_shape_fault(const ConversationCheckpoint& c, const ConversationView& view, int64_t stages) {
    const bool live_prefix = !c.ids.empty() && c.ids.size() <= view.ids.size() &&
                             std::equal(c.ids.begin(), c.ids.end(), view.ids.begin());
    if (!live_prefix) return "a retained checkpoint is not a prefix of the live branch";
    if ((int64_t) c.stage_parts.size() != stages)
        return stages ? "a retained checkpoint lacks a part for every later stage"
                      : "a retained checkpoint carries stage parts but the session is not split";
    for (const ConversationCheckpoint& part : c.stage_parts)
        if (part.ids.size() != c.ids.size() || !part.imgs.empty() || !part.stage_parts.empty())
            return "a checkpoint's stage part does not cover exactly the checkpoint's tokens";
    if (!conversation_match_detail::images_agree(c, view.images, c.ids.size()))
        return "a retained checkpoint's images are not the live branch's images over its tokens";
    return nullptr;
}

/// A session's share of an image of an `upto`-token branch: its running state, the token ids, the K/V directory
/// and every owned layer's K/V, and `draft` (the main session's draft layer) when given.
bool add_session_share(Ledger& ledger, const SessionState& ss, const ModelGeometry& g, int64_t upto,
                       const QsaState* draft, std::string& error) {
    RunningState rs;
    if (!running_state(ss, g, (size_t) upto, rs, error)) return false;
    ledger.add(rs.gdn()).add(rs.ple()).add(rs.tails()).add(rs.dead()).add(rs.block_pos());
    ledger.add((uint64_t) upto, sizeof(int32_t));
    ledger.add(rs.layers + (draft ? 1 : 0), sizeof(ConversationKv));
    for (size_t j = 0; j < rs.layers; ++j) ledger.add_estimate(conversation_kv_bytes(owned_layer(ss, j), g, upto, true));
    if (draft) ledger.add_estimate(conversation_kv_bytes(*draft, g, upto, false));
    return true;
}

/// What a copy of retained checkpoint `c` adds to an image (its own vectors and, recursively, its stage parts).
void add_checkpoint_copy(Ledger& ledger, const ConversationCheckpoint& c) {
    ledger.add(c.ids.size(), sizeof(int32_t)).add(c.imgs.size(), sizeof(ConversationImageKey));
    for (const std::vector<uint8_t>* v : {&c.gdn, &c.ple, &c.tails, &c.dead, &c.block_pos}) ledger.add(v->size());
    ledger.add(c.stage_parts.capacity(), sizeof(ConversationCheckpoint));
    for (const ConversationCheckpoint& part : c.stage_parts) add_checkpoint_copy(ledger, part);
}

}  // namespace

bool images_ordered(const std::vector<ConversationImageKey>& images, size_t tokens) {
    for (size_t i = 0; i < images.size(); ++i) {
        const int64_t start = images[i].start;
        if (start < 0 || (uint64_t) start >= tokens || (i > 0 && start <= images[i - 1].start)) return false;
    }
    return true;
}

bool running_state(const SessionState& ss, const ModelGeometry& g, size_t tokens, RunningState& rs,
                   std::string& error) {
    rs = {};
    if (!conversation_session_sizes(g, ss, rs.per, error)) return false;
    rs.layers = owned_count(ss);
    rs.keeps_ple = ss.ple_hist != nullptr;
    if (ss.max_cells < 0 || tokens > (uint64_t) ss.max_cells)
        return fail(error, "the session holds fewer cells than the branch");
    if ((rs.per.gdn && !ss.gdn_state) || (rs.layers && !ss.qsa_states))
        return fail(error, "the session lacks a running-state buffer its carve needs");
    for (size_t j = 0; j < rs.layers; ++j)
        if (const char* why = indexer_fault(owned_layer(ss, j), g, tokens)) return fail(error, why);
    return true;
}

bool stages_tile(const ConversationStageSet& stages, const SessionState& main_ss, const ModelGeometry& g,
                 std::string& error) {
    if (stages.empty()) return true;
    if (stages.count > (int64_t) (std::numeric_limits<size_t>::max() / sizeof(ConversationStageSnapshot)))
        return fail(error, "the stage set is larger than an image can index");
    const int64_t n_qsa = g.n_qsa_layers(), interval = std::max<int64_t>(g.qsa_interval, 1);
    int64_t covered = main_ss.layer_hi;   // the layers [0, covered) belong to the main session and earlier stages
    for (int64_t i = 0; i < stages.count; ++i) {
        const SessionState* ss = stages.stages[i].session;
        if (!ss) return fail(error, "a later stage has no session");
        ConversationStateSizes unused;
        if (!conversation_session_sizes(g, *ss, unused, error)) return false;
        if (ss->layer_lo != covered || ss->layer_hi <= ss->layer_lo || ss->layer_hi > g.n_layers)
            return fail(error, "the later stages do not continue the layer range in order");
        if (ss->qsa_ord0 < ss->layer_lo / interval || ss->qsa_alloc > n_qsa - ss->qsa_ord0)
            return fail(error, "a later stage's QSA carve lies outside its layers");
        covered = ss->layer_hi;
    }
    if (covered != g.n_layers) return fail(error, "the later stages stop short of the last layer");
    return true;
}

bool view_ok(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
             const ModelGeometry& g, std::string& error) {
    RunningState rs;
    if (!running_state(ss, g, view.ids.size(), rs, error)) return false;
    if (view.ids.empty()) return fail(error, "the live branch is empty");
    if (std::any_of(view.ids.begin(), view.ids.end(), [](int32_t id) { return id < 0; }))
        return fail(error, "the live branch has a negative token id");
    if (!images_ordered(view.images, view.ids.size()))
        return fail(error, "the live branch's images are out of order or past its tokens");
    const int64_t n_stages = stage_count(stages);
    for (const ConversationCheckpoint& c : view.checkpoints) {
        if (const char* why = checkpoint_shape_fault(c, view, n_stages)) return fail(error, why);
        if (!conversation_checkpoint_validate(c, ss, g, error)) return false;
        for (int64_t i = 0; i < n_stages; ++i)
            if (!conversation_checkpoint_validate(c.stage_parts[(size_t) i], *stages.stages[i].session, g, error))
                return false;
    }
    return true;
}

/// Queue a checkpoint's running state (save direction) into `t`, its buffers sized from the session's plan.
bool enqueue_checkpoint_save(ConversationCheckpoint& c, const SessionState& ss, const ModelGeometry& g,
                             strata::kv::Transfer& t, std::string& error) {
    RunningState rs;
    if (!running_state(ss, g, c.ids.size(), rs, error)) return false;
    c.gdn.resize(rs.gdn());
    c.ple.resize(rs.ple());
    c.tails.resize(rs.tails());
    c.dead.resize(rs.dead());
    c.block_pos.resize(rs.block_pos());
    auto dev = [](const void* p) {
        strata::kv::DeviceStream s;
        s.base = p;
        return s;
    };
    if (!c.gdn.empty()) t.save(dev(ss.gdn_state), 0, c.gdn.size(), c.gdn.data());
    if (!c.ple.empty()) t.save(dev(ss.ple_hist), 0, c.ple.size(), c.ple.data());
    const ConversationStateSizes& per = rs.per;
    for (size_t j = 0; j < rs.layers; ++j) {
        const QsaState& st = owned_layer(ss, j);
        t.save(dev(st.idx_tail), 0, per.tail, c.tails.data() + j * per.tail);
        t.save(dev(st.idx_dead), 0, per.dead, c.dead.data() + j * per.dead);
        t.save(dev(st.idx_block_pos), 0, per.block_pos, c.block_pos.data() + j * per.block_pos);
    }
    return true;
}

}  // namespace snapshot_detail

using namespace snapshot_detail;

// ------------------------------------------------------------------------------------------------ sizes

bool conversation_state_sizes(const ModelGeometry& g, ConversationStateSizes& z, std::string& error) {
    z = {};
    std::array<int64_t, 18> dims = geometry_key(g);
    const int64_t layers = dims[1];
    dims[1] = 1;   // a geometry may have no layers; every other dimension must be positive
    if (layers < 0 || *std::min_element(dims.begin(), dims.end()) <= 0)
        return fail(error, "the model geometry has a non-positive dimension");
    const uint64_t idx_block = (uint64_t) strata::kernels::qsa_real_shapes().idx_block;
    size_t state = 0, conv = 0, row = 0;
    bool ok = checked_product(state, {(uint64_t) g.ssm_state_size, (uint64_t) g.ssm_v_heads, (uint64_t) g.ssm_state_size}) &&
              checked_product(conv, {(uint64_t) g.ssm_conv_channels, (uint64_t) (g.ssm_d_conv - 1)});
    row = state;
    ok = ok && checked_add(row, conv) &&
         checked_product(z.gdn, {(uint64_t) g.n_gdn_layers(), row, sizeof(float)}) &&
         checked_product(z.ple, {(uint64_t) strata::kernels::NG_HIST, (uint64_t) strata::kernels::NG_HC_DIM, sizeof(float)}) &&
         checked_product(z.tail, {idx_block - 1, (uint64_t) g.idx_key_dim, sizeof(float)}) &&
         checked_product(z.dead, {(uint64_t) g.idx_key_dim, sizeof(float)});
    z.block_pos = sizeof(int32_t);
    // every QSA layer's share must be countable too (a full carve owns all of them)
    size_t whole = 0;
    const uint64_t n_qsa = (uint64_t) g.n_qsa_layers();
    ok = ok && checked_product(whole, {n_qsa, z.tail}) && checked_product(whole, {n_qsa, z.dead}) &&
         checked_product(whole, {n_qsa, z.block_pos});
    if (!ok) return fail(error, "the running state's byte counts overflow");
    return true;
}

bool conversation_session_sizes(const ModelGeometry& g, const SessionState& ss, ConversationStateSizes& z,
                                std::string& error) {
    if (!conversation_state_sizes(g, z, error)) return false;
    const int64_t n_gdn = g.n_gdn_layers(), n_qsa = g.n_qsa_layers();
    const bool gdn_carve = 0 <= ss.gdn_alloc && ss.gdn_alloc <= n_gdn;
    const bool qsa_carve = 0 <= ss.qsa_ord0 && ss.qsa_ord0 <= n_qsa && 0 <= ss.qsa_alloc && ss.qsa_alloc <= n_qsa - ss.qsa_ord0;
    if (!gdn_carve || !qsa_carve) return fail(error, "the session's layer carve lies outside the model");
    // the GDN rows are per layer: a session carries only the rows of the layers it owns
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
    RunningState rs;
    if (!running_state(ss, g, c.ids.size(), rs, error)) return false;
    auto holds = [&](const std::vector<uint8_t>& v, size_t want) { return size_of(&v, v.size()) == want; };
    if (!holds(c.gdn, rs.gdn()) || !holds(c.ple, rs.ple()) || !holds(c.tails, rs.tails()) || !holds(c.dead, rs.dead()) ||
        !holds(c.block_pos, rs.block_pos()))
        return fail(error, "a checkpoint's running-state buffers are not the size the session needs");
    if (!images_ordered(c.imgs, c.ids.size())) return fail(error, "a checkpoint's images are out of order or past its tokens");
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
    RunningState rs;
    if (!running_state(ss, g, c.ids.size(), rs, error)) return false;
    auto dev = [](const void* p) {
        strata::kv::DeviceStream s;
        s.base = p;
        return s;
    };
    strata::kv::Transfer t;
    if (!c.gdn.empty()) t.restore(c.gdn.data(), 0, c.gdn.size(), dev(ss.gdn_state));
    if (!c.ple.empty()) t.restore(c.ple.data(), 0, c.ple.size(), dev(ss.ple_hist));
    const ConversationStateSizes& per = rs.per;
    // the pooled row the next indexer block accumulates into starts as the dead key again
    const size_t spare_row = c.ids.size() / (size_t) strata::kernels::qsa_real_shapes().idx_block;
    for (size_t j = 0; j < rs.layers; ++j) {
        const QsaState& st = owned_layer(ss, j);
        const uint8_t* dead = c.dead.data() + j * per.dead;
        t.restore(c.tails.data() + j * per.tail, 0, per.tail, dev(st.idx_tail));
        t.restore(dead, 0, per.dead, dev(st.idx_dead));
        t.restore(c.block_pos.data() + j * per.block_pos, 0, per.block_pos, dev(st.idx_block_pos));
        if (!c.ids.empty()) t.restore(dead, 0, per.dead, dev(st.idx_pooled + spare_row * (size_t) g.idx_key_dim));
    }
    if (!t.run(error, "conversation snapshot running-state copy")) return false;
    // the PLE history's two previous tokens are the branch's last two ids, oldest first (-1 before the start)
    const size_t n = c.ids.size();
    for (size_t k = 0; k < 2; ++k) {
        const size_t back = 2 - k;
        ss.ple_prev[k] = n >= back ? c.ids[n - back] : -1;
    }
    return device_sync(error);
}

// ------------------------------------------------------------------------------------------------ snapshots

bool conversation_snapshot_bytes(const ConversationView& view, const SessionState& ss, const ConversationStageSet& stages,
                                 const ModelGeometry& g, const QsaState& draft, size_t& bytes, std::string& error) {
    bytes = 0;
    if (!stages_tile(stages, ss, g, error) || !view_ok(view, ss, stages, g, error)) return false;
    const int64_t upto = (int64_t) view.ids.size();
    Ledger ledger;
    if (!add_session_share(ledger, ss, g, upto, &draft, error)) return false;
    ledger.add(view.images.size(), sizeof(ConversationImageKey)).add(view.checkpoints.size(), sizeof(ConversationCheckpoint));
    for (const ConversationCheckpoint& c : view.checkpoints) add_checkpoint_copy(ledger, c);
    if (!stages.empty()) ledger.add((uint64_t) stages.count, sizeof(ConversationStageSnapshot));
    for (int64_t i = 0; i < stage_count(stages); ++i)
        if (!add_session_share(ledger, *stages.stages[i].session, g, upto, nullptr, error)) return false;
    if (!ledger.ok()) return fail(error, "the snapshot's byte count overflows, or a layer's K/V cannot be sized");
    bytes = ledger.total();
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
    // only the main session's layers and its draft are ever reused, never a later stage's
    const size_t reused = owned_count(ss) + 1;
    const int64_t upto = (int64_t) view.ids.size();
    const bool prefix_ok = reuse.kv.size() == reused && reuse.unchanged_tokens >= 0 &&
                           reuse.unchanged_tokens <= reuse.captured_tokens && reuse.unchanged_tokens <= upto;
    if (!prefix_ok) return fail(error, "the retained K/V does not describe a prefix of this session's layers");
    // each reused layer's fresh estimate gives way to what its retained buffers grow to
    size_t rest = bytes;
    Ledger grown;
    for (size_t i = 0; i < reused; ++i) {
        const bool is_draft = i + 1 == reused;
        const QsaState& st = is_draft ? draft : owned_layer(ss, i);
        if (!conversation_kv_validate(reuse.kv[i], st, g, reuse.captured_tokens, !is_draft, error)) return false;
        size_t kept = 0;
        if (!conversation_kv_capture_bytes(reuse.kv[i], st, g, upto, !is_draft, kept, error)) return false;
        rest -= conversation_kv_bytes(st, g, upto, !is_draft);
        grown.add(kept);
    }
    grown.add(reuse.kv.capacity() - reused, sizeof(ConversationKv)).add(rest);
    if (!grown.ok()) return fail(error, "the capture's byte count overflows");
    bytes = grown.total();
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

namespace {
/// One session's part of an image fits that session: its running-state checkpoint, and one K/V image per owned
/// layer (then the draft's, for the main session) each valid for its layer at `upto` tokens.
bool session_part_fits(const ConversationCheckpoint& state, const std::vector<ConversationKv>& kv,
                       const SessionState& ss, const QsaState* draft, const ModelGeometry& g, int64_t upto,
                       std::string& error, const SizeOf& size_of) {
    if (!checkpoint_validate_sized(state, ss, g, error, size_of)) return false;
    const size_t layers = owned_count(ss);
    if (kv.size() != layers + (draft ? 1 : 0)) return fail(error, "the image holds another number of K/V layers than the session");
    for (size_t j = 0; j < layers; ++j)
        if (!kv_validate_sized(kv[j], owned_layer(ss, j), g, upto, true, error, size_of)) return false;
    return !draft || kv_validate_sized(kv.back(), *draft, g, upto, false, error, size_of);
}
}  // namespace

bool snapshot_detail::snapshot_validate_sized(const SavedConversation& image, const SessionState& ss,
                                              const ConversationStageSet& stages, const ModelGeometry& g,
                                              const QsaState& draft, std::string& error, const SizeOf& size_of) {
    if (!stages_tile(stages, ss, g, error)) return false;
    const int64_t n_stages = stage_count(stages);
    if (!image.live.stage_parts.empty() || (int64_t) image.stage_parts.size() != n_stages)
        return fail(error, n_stages ? "the image lacks a part for every later stage"
                                    : "the image was parked from a split session and this one is not split");
    if (image.geometry != geometry_key(g)) return fail(error, "the image was parked under another model geometry");
    if (image.layer_lo != ss.layer_lo || image.layer_hi != ss.layer_hi)
        return fail(error, "the image covers other layers than the session");
    const ConversationView view{image.live.ids, image.live.imgs, image.checkpoints, image.cvec};
    const int64_t upto = (int64_t) image.live.ids.size();
    if (!view_ok(view, ss, stages, g, error) ||
        !session_part_fits(image.live, image.kv, ss, &draft, g, upto, error, size_of))
        return false;
    for (int64_t i = 0; i < n_stages; ++i) {
        const ConversationStageSnapshot& part = image.stage_parts[(size_t) i];
        const SessionState& stage = *stages.stages[i].session;
        if (part.layer_lo != stage.layer_lo || part.layer_hi != stage.layer_hi)
            return fail(error, "a stage part covers other layers than its stage");
        const bool whole_branch = part.state.imgs.empty() && part.state.stage_parts.empty() &&
                                  part.state.ids == image.live.ids;
        if (!whole_branch) return fail(error, "a stage part's running state is not for the whole live branch");
        if (!session_part_fits(part.state, part.kv, stage, nullptr, g, upto, error, size_of)) return false;
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
