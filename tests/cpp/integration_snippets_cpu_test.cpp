// tests/cpp/integration_snippets_cpu_test.cpp - the calls a maintainer adds to the reference engine to bind this
// library (park_current, the mount hook, the split-role publish and mount), written as functions over the
// engine's own objects, so that a change of a header that breaks a documented call breaks this build.  Compiled
// (syntax and types, warnings as errors) by tests/test_cpp_cpu.py; nothing here is run.
#include "strata_kv.h"
#include "strata_kv/conversation_snapshot.hpp"
#include "strata_kv/conversation_wire_device.hpp"
#include "strata_kv/handoff_device.hpp"

#include <string>
#include <vector>

using namespace strata::core;

// 1. one QSA layer's K and V through its page table into a host or staging image
bool park_layer(const QsaState& st, void* k_image, void* v_image, uint64_t data_bytes, uint32_t page_bytes,
                void* stream, std::string& error) {
    skv_segment seg[2] = {
        {st.k_pool, k_image, st.page_table, nullptr, data_bytes, page_bytes, 0, st.n_pages, 0},
        {st.v_pool, v_image, st.page_table, nullptr, data_bytes, page_bytes, 0, st.n_pages, 0},
    };
    if (skv_copy(seg, 2, SKV_COPY_AUTO, stream) != SKV_OK) {
        error = std::string("conversation snapshot copy: ") + skv_last_error();
        return false;
    }
    return true;
}

// 2. the block table in the reference page_table format
void place_layer(skv_pool* pool, int32_t n_blocks, int32_t* k_page_table, int32_t* v_page_table) {
    std::vector<int32_t> blocks((size_t) n_blocks);
    skv_alloc_blocks(pool, n_blocks, blocks.data());
    skv_expand_block_table(blocks.data(), n_blocks, 64, 128, 0, k_page_table);
    skv_expand_block_table(blocks.data(), n_blocks, 64, 128, 64, v_page_table);
}

// 3. the pull hand-off between a prefill and a decode GPU
void pull(uint64_t* ready_flag, uint64_t* done_flag, uint64_t seq_no, const skv_segment* segs, int n, void* stream) {
    skv_signal(ready_flag, seq_no, stream);
    skv_wait_flag(ready_flag, seq_no, 2'000'000'000, stream);
    skv_copy(segs, n, SKV_COPY_TMA, stream);
    skv_signal(done_flag, seq_no, stream);
}
void pull_gated(uint64_t* ready_flag, uint64_t* done_flag, uint64_t seq_no, const skv_segment* segs, int n,
                void* stream) {
    skv_copy_gated(segs, n, ready_flag, seq_no, 2'000'000'000, done_flag, seq_no, stream);
}

// 3. one GPU of a pushed chain
void chain_hop(int k, const skv_segment* chunks, int n_chunks, const uint64_t* my_flags, uint64_t* next_flags,
               uint64_t seq_no, void* stream) {
    skv_copy_chained(chunks, n_chunks, k ? my_flags : nullptr, next_flags, seq_no, 2'000'000'000, stream);
}

// 3. a decode GPU's share of a many-to-many batch
void phased(const uint64_t* bytes_pre_to_dec, int n_pre, int n_dec, int me, const skv_segment* const* flow,
            const int* n_flow, uint64_t* my_flags, uint64_t* const* peer_flags, uint64_t step, void* stream) {
    const int n = n_pre > n_dec ? n_pre : n_dec;
    const int max_runs = n * n;
    std::vector<skv_sched_run> runs((size_t) (n_dec * max_runs));
    std::vector<int> n_runs((size_t) n_dec);
    uint64_t bound = 0;
    int phases = 0;
    skv_schedule_phases(bytes_pre_to_dec, n_pre, n_dec, runs.data(), max_runs, n_runs.data(), &bound, &phases);
    skv_segment pieces[64];
    int n_pieces = 0;
    for (int j = 0; j < n_runs[(size_t) me]; ++j) {
        const skv_sched_run& r = runs[(size_t) (me * max_runs + j)];
        skv_slice_segments(flow[r.src], n_flow[r.src], r.lo, r.hi, pieces, 64, &n_pieces);
        skv_copy_gated(pieces, n_pieces, r.wait >= 0 ? &my_flags[r.wait] : nullptr, step, 2'000'000'000,
                       r.signal_dst >= 0 ? &peer_flags[r.signal_dst][r.signal_idx] : nullptr, step, stream);
    }
}

// 3, the same with the hand-overs as launches of their own
void phased_launches(const skv_sched_run* runs, int n, const skv_segment* const* flow, const int* n_flow,
                     uint64_t* my_flags, uint64_t* const* peer_flags, uint64_t step, void* stream) {
    skv_segment pieces[64];
    int n_pieces = 0;
    for (int j = 0; j < n; ++j) {
        const skv_sched_run& r = runs[j];
        if (r.wait >= 0) skv_wait_flag(&my_flags[r.wait], step, 2'000'000'000, stream);
        skv_slice_segments(flow[r.src], n_flow[r.src], r.lo, r.hi, pieces, 64, &n_pieces);
        skv_copy(pieces, n_pieces, SKV_COPY_TMA, stream);
        if (r.signal_dst >= 0) skv_signal(&peer_flags[r.signal_dst][r.signal_idx], step, stream);
    }
}

// 3b. parking straight to the SR4H wire format
bool pack(const ConversationView& view, const SessionState& session, const ModelGeometry& g, const QsaState& draft,
          uint64_t geom_hash, uint64_t pack_hash, uint8_t* dst, WireEncoded& enc, std::string& err) {
    WirePlan plan;
    if (!conversation_wire_pack_plan(view, session, g, draft, plan, err)) return false;
    return conversation_wire_pack_device(view, session, g, draft, {geom_hash, pack_hash}, dst, plan.total_bytes, plan,
                                         enc, err);
}

// 3c. the split roles with a device descriptor in the slot
bool prefill_side(HandoffArena& arena, uint32_t tier, uint64_t client_id, uint64_t request_id,
                  const ConversationView& view, const SessionState& session, const ConversationStageSet& stages,
                  const ModelGeometry& g, const QsaState& draft, uint64_t geom_hash, uint64_t pack_hash,
                  uint8_t* payload_buf, uint64_t payload_cap, const uint8_t ipc_handle[64], std::string& err) {
    HandoffClaim claim;
    WireEncoded enc;
    if (!arena.claim(tier, client_id, request_id, claim, err)) return false;
    return handoff_device_publish(arena, claim, view, session, stages, g, draft, {geom_hash, pack_hash}, payload_buf,
                                  payload_cap, ipc_handle, 0, enc, err);
}

ConversationRestore decode_side(HandoffArena& arena, DevicePayloadImports& imports, int slot, uint64_t nonce,
                                uint64_t client_id, SessionState& session, const ConversationStageSet& stages,
                                const ModelGeometry& g, const QsaState& draft, const WireExpect& expect,
                                SavedConversation& meta, WireDecoded& info, std::string& err) {
    HandoffPayload payload;
    if (!arena.read_slot(slot, nonce, client_id, payload, err)) return ConversationRestore::invalid;
    if (handoff_device_is_descriptor(payload.data, payload.payload_bytes))
        return handoff_device_mount(payload, imports, session, stages, g, draft, expect, meta, info, err);
    return ConversationRestore::invalid;   // an SR4H payload: conversation_wire_decode + _restore, as today
}
