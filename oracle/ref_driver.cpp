// oracle/ref_driver.cpp - TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// A thin extern "C" driver around the REFERENCE's own park/resume and wire-codec code, compiled from the
// reference's sources by oracle/Makefile into oracle/_ref/libstrata_ref.so.  Nothing here restates the
// reference: every byte this produces comes out of the reference's functions
//   * conversation_snapshot_save / _restore   (src/core/conversation_state.cpp:360-507)
//   * conversation_kv_save / _restore         (src/core/conversation_snapshot.cpp:139-219)
//   * conversation_wire_encode / _decode      (src/core/conversation_wire.cpp:1006-1040)
// run against HOST buffers laid out the way the reference's device pools are (identity page table,
// kv_mode 0).  cudaMemcpy / cudaDeviceSynchronize / cudaGetLastError are link-wrapped to host
// operations exactly the way the reference builds its own conversation_transfer_test
// (CMakeLists.txt:333-340), so no GPU is touched.
//
// Only tests/, tests/golden/make_golden.py, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
// this library.
#include "strata/core/conversation_snapshot.hpp"
#include "strata/core/conversation_wire.hpp"
#include "strata/core/pinned.hpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace strata::core;

// ---------------------------------------------------------------- link-wrapped CUDA (host backend)
namespace {
int g_fail_copy_at = 0;   // 1-based index of the copy that fails; 0 = never
int g_copy_calls = 0;
}  // namespace

extern "C" __attribute__((visibility("default"))) cudaError_t __wrap_cudaMemcpy(void* dst, const void* src, size_t n,
                                                                                 cudaMemcpyKind) {
    if (++g_copy_calls == g_fail_copy_at) return cudaErrorInvalidValue;
    std::memcpy(dst, src, n);
    return cudaSuccess;
}
extern "C" __attribute__((visibility("default"))) cudaError_t __wrap_cudaDeviceSynchronize() { return cudaSuccess; }
extern "C" __attribute__((visibility("default"))) cudaError_t __wrap_cudaGetLastError() { return cudaSuccess; }

// ---------------------------------------------------------------- the reference's FNV-1a symbol
// The reference defines fnv1a64 in src/core/pinned.cu:594-601, a CUDA translation unit that also drags in the
// expert arena.  The codec only needs the hash, so this supplies the public FNV-1a 64 algorithm (offset basis
// 1469598103934665603, prime 1099511628211) under the reference's declared signature
// (include/strata/core/pinned.hpp:173).
namespace strata::core {
uint64_t fnv1a64(const uint8_t* p, uint64_t n, uint64_t seed) {
    uint64_t h = seed;
    for (uint64_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}
}  // namespace strata::core

// ---------------------------------------------------------------- mode-1/2 entry points mode 0 never calls
namespace strata::kernels {
void kv_stream_reset(const KvStreamMap&, void*) {
    std::fprintf(stderr, "ref_driver: kv_stream_reset reached (kv_mode 1 is not built into the oracle)\n");
    std::abort();
}
void kv_ring_restore(const QsaAttnPools&, const KvHostPools&, int, int64_t, int64_t, int64_t, const QsaShapes&, void*) {
    std::fprintf(stderr, "ref_driver: kv_ring_restore reached (kv_mode 2 is not built into the oracle)\n");
    std::abort();
}
}  // namespace strata::kernels
namespace strata::core {
strata::kernels::QsaAttnPools qsa_attn_pools(const QsaState&) {
    std::fprintf(stderr, "ref_driver: qsa_attn_pools reached (kv_mode 2 is not built into the oracle)\n");
    std::abort();
}
}  // namespace strata::core

// ---------------------------------------------------------------- the flat session description
extern "C" {

#define REF_MAX_QSA 64

/// A synthetic session held in host memory in the reference's device layout.  Index n_qsa of the K/V
/// arrays is the draft (MTP) layer; the indexer arrays have n_qsa entries.  ple_hist may be null (the
/// reference then saves no PLE history, src/core/conversation_state.cpp:231).
typedef struct RefSession {
    int64_t n_layers, qsa_interval, n_head_kv, head_dim;
    int64_t ssm_state_size, ssm_v_heads, ssm_d_conv, ssm_conv_channels, idx_key_dim;
    int64_t max_cells;        // cells every pool holds (a multiple of the 4-cell page)
    int64_t idx_pooled_rows;  // rows of each idx_pooled buffer
    void* k_pool[REF_MAX_QSA + 1];
    void* v_pool[REF_MAX_QSA + 1];
    void* idx_pooled[REF_MAX_QSA];
    void* idx_tail[REF_MAX_QSA];
    void* idx_dead[REF_MAX_QSA];
    void* idx_block_pos[REF_MAX_QSA];
    void* gdn_state;
    void* ple_hist;
} RefSession;

}  // extern "C"

namespace {

ModelGeometry geometry(const RefSession& r) {
    ModelGeometry g;
    g.n_layers = r.n_layers;
    g.qsa_interval = r.qsa_interval;
    g.n_head_kv = r.n_head_kv;
    g.head_dim = r.head_dim;
    g.ssm_state_size = r.ssm_state_size;
    g.ssm_v_heads = r.ssm_v_heads;
    g.ssm_d_conv = r.ssm_d_conv;
    g.ssm_conv_channels = r.ssm_conv_channels;
    g.idx_key_dim = r.idx_key_dim;
    return g;
}

/// The reference's session objects over the flat description.  Identity page tables, kv_mode 0, one GPU.
struct Bound {
    ModelGeometry g;
    std::vector<QsaState> qsa;
    std::vector<std::vector<int32_t>> tables;
    QsaState draft;
    SessionState ss;
    int64_t n_qsa = 0;

    bool bind(const RefSession& r, std::string& error) {
        g = geometry(r);
        n_qsa = g.n_qsa_layers();
        if (n_qsa > REF_MAX_QSA || r.max_cells % 4 != 0) { error = "ref_driver: unsupported session shape"; return false; }
        const int64_t pages = r.max_cells / 4;
        tables.assign((size_t) n_qsa + 1, std::vector<int32_t>((size_t) pages));
        for (auto& t : tables)
            for (int64_t p = 0; p < pages; ++p) t[(size_t) p] = (int32_t) p;
        auto layer = [&](QsaState& st, int64_t j, bool index) {
            st = QsaState{};
            st.k_pool = static_cast<uint16_t*>(r.k_pool[j]);
            st.v_pool = static_cast<uint16_t*>(r.v_pool[j]);
            st.page_table = tables[(size_t) j].data();
            st.n_pages = pages;
            st.n_slots = pages;
            st.max_cells = r.max_cells;
            st.kv_mode = 0;
            if (index) {
                st.idx_pooled_rows = r.idx_pooled_rows;
                st.idx_pooled = static_cast<float*>(r.idx_pooled[j]);
                st.idx_tail = static_cast<float*>(r.idx_tail[j]);
                st.idx_dead = static_cast<float*>(r.idx_dead[j]);
                st.idx_block_pos = static_cast<int32_t*>(r.idx_block_pos[j]);
            } else {
                st.idx_pooled_rows = 2;
            }
        };
        qsa.resize((size_t) n_qsa);
        for (int64_t j = 0; j < n_qsa; ++j) layer(qsa[(size_t) j], j, true);
        layer(draft, n_qsa, false);
        ss = SessionState{};
        ss.max_cells = r.max_cells;
        ss.gdn_state = static_cast<float*>(r.gdn_state);
        ss.qsa_states = qsa.empty() ? nullptr : qsa.data();
        ss.layer_lo = 0;
        ss.layer_hi = g.n_layers;
        ss.qsa_ord0 = 0;
        ss.qsa_alloc = n_qsa;
        ss.gdn_ord0 = 0;
        ss.gdn_alloc = g.n_gdn_layers();
        ss.ple_hist = static_cast<float*>(r.ple_hist);
        return true;
    }
};

void set_error(char* out, size_t cap, const std::string& e) {
    if (out && cap) std::snprintf(out, cap, "%s", e.c_str());
}

uint8_t* copy_out(const std::vector<uint8_t>& bytes) {
    uint8_t* p = static_cast<uint8_t*>(std::malloc(bytes.size() ? bytes.size() : 1));
    if (p && !bytes.empty()) std::memcpy(p, bytes.data(), bytes.size());
    return p;
}

}  // namespace

extern "C" {

/// conversation_snapshot_save over `r` for the first `tokens` tokens (ids given), then
/// conversation_wire_encode of the result into a malloc'd buffer.  Returns 0 on success.
__attribute__((visibility("default"))) int ref_snapshot_encode(const RefSession* r, int64_t tokens, const int32_t* ids,
                                                               uint64_t geom_hash, uint64_t pack_hash,
                                                               uint8_t** out, uint64_t* out_bytes, uint64_t* out_hash,
                                                               char* err, size_t err_cap) {
    std::string error;
    Bound b;
    if (!b.bind(*r, error)) { set_error(err, err_cap, error); return 1; }
    std::vector<int32_t> live(ids, ids + tokens);
    std::vector<ConversationImageKey> images;
    std::vector<ConversationCheckpoint> checkpoints;
    const ConversationView view{live, images, checkpoints, true};
    SavedConversation image;
    if (!conversation_snapshot_save(image, view, b.ss, b.g, b.draft, error)) { set_error(err, err_cap, error); return 2; }
    VectorWireSink sink;
    WireEncoded enc;
    if (!conversation_wire_encode(image, sink, {geom_hash, pack_hash}, enc, error)) { set_error(err, err_cap, error); return 3; }
    *out = copy_out(sink.data());
    *out_bytes = enc.bytes;
    *out_hash = enc.payload_hash;
    return 0;
}

/// conversation_wire_decode of `payload`, then conversation_snapshot_restore into `r`.
/// Returns 0 on success, 4 when the payload is refused, 5 when validation refuses (invalid),
/// 6 when a transfer failed after the first write.
__attribute__((visibility("default"))) int ref_decode_restore(const RefSession* r, const uint8_t* payload, uint64_t bytes,
                                                              char* err, size_t err_cap) {
    std::string error;
    Bound b;
    if (!b.bind(*r, error)) { set_error(err, err_cap, error); return 1; }
    SavedConversation image;
    WireDecoded info;
    WireExpect expect;
    if (!conversation_wire_decode(payload, bytes, image, info, expect, error)) { set_error(err, err_cap, error); return 4; }
    const auto status = conversation_snapshot_restore(image, b.ss, b.g, b.draft, error);
    if (status == ConversationRestore::invalid) { set_error(err, err_cap, error); return 5; }
    if (status == ConversationRestore::transfer_failed) { set_error(err, err_cap, error); return 6; }
    return 0;
}

/// The byte count conversation_snapshot_bytes prices a park at (src/core/conversation_state.cpp:320-333).
__attribute__((visibility("default"))) int ref_snapshot_bytes(const RefSession* r, int64_t tokens, const int32_t* ids,
                                                              uint64_t* bytes, char* err, size_t err_cap) {
    std::string error;
    Bound b;
    if (!b.bind(*r, error)) { set_error(err, err_cap, error); return 1; }
    std::vector<int32_t> live(ids, ids + tokens);
    std::vector<ConversationImageKey> images;
    std::vector<ConversationCheckpoint> checkpoints;
    size_t n = 0;
    if (!conversation_snapshot_bytes({live, images, checkpoints, true}, b.ss, b.g, b.draft, n, error)) {
        set_error(err, err_cap, error);
        return 2;
    }
    *bytes = n;
    return 0;
}

/// The reference's host park/resume, timed: `reps` times conversation_snapshot_save from `src` then
/// conversation_snapshot_restore into `dst`.  Writes per-rep milliseconds (save, restore) into the arrays.
__attribute__((visibility("default"))) int ref_time_park_resume(const RefSession* src, const RefSession* dst, int64_t tokens,
                                                                const int32_t* ids, int reps, double* save_ms,
                                                                double* restore_ms, char* err, size_t err_cap) {
    std::string error;
    Bound a, b;
    if (!a.bind(*src, error) || !b.bind(*dst, error)) { set_error(err, err_cap, error); return 1; }
    std::vector<int32_t> live(ids, ids + tokens);
    std::vector<ConversationImageKey> images;
    std::vector<ConversationCheckpoint> checkpoints;
    const ConversationView view{live, images, checkpoints, true};
    for (int i = 0; i < reps; ++i) {
        SavedConversation image;
        const auto t0 = std::chrono::steady_clock::now();
        if (!conversation_snapshot_save(image, view, a.ss, a.g, a.draft, error)) { set_error(err, err_cap, error); return 2; }
        const auto t1 = std::chrono::steady_clock::now();
        if (conversation_snapshot_restore(image, b.ss, b.g, b.draft, error) != ConversationRestore::restored) {
            set_error(err, err_cap, error);
            return 3;
        }
        const auto t2 = std::chrono::steady_clock::now();
        save_ms[i] = std::chrono::duration<double, std::milli>(t1 - t0).count();
        restore_ms[i] = std::chrono::duration<double, std::milli>(t2 - t1).count();
    }
    return 0;
}

/// The reference's codec round trip, timed: encode (with its streaming FNV-1a) then decode.
__attribute__((visibility("default"))) int ref_time_wire(const uint8_t* payload, uint64_t bytes, int reps, double* encode_ms,
                                                         double* decode_ms, char* err, size_t err_cap) {
    std::string error;
    SavedConversation image;
    WireDecoded info;
    if (!conversation_wire_decode(payload, bytes, image, info, WireExpect{}, error)) { set_error(err, err_cap, error); return 1; }
    for (int i = 0; i < reps; ++i) {
        VectorWireSink sink(bytes);
        WireEncoded enc;
        const auto t0 = std::chrono::steady_clock::now();
        if (!conversation_wire_encode(image, sink, {info.geom_hash, info.pack_hash}, enc, error)) {
            set_error(err, err_cap, error);
            return 2;
        }
        const auto t1 = std::chrono::steady_clock::now();
        SavedConversation back;
        WireDecoded got;
        WireExpect expect;
        expect.payload_hash = enc.payload_hash;
        expect.check_payload_hash = true;
        if (!conversation_wire_decode(sink.data().data(), sink.data().size(), back, got, expect, error)) {
            set_error(err, err_cap, error);
            return 3;
        }
        const auto t2 = std::chrono::steady_clock::now();
        encode_ms[i] = std::chrono::duration<double, std::milli>(t1 - t0).count();
        decode_ms[i] = std::chrono::duration<double, std::milli>(t2 - t1).count();
    }
    return 0;
}

/// The reference's conversation_wire_payload_hash (FNV-1a over the payload as written).
__attribute__((visibility("default"))) uint64_t ref_payload_hash(const uint8_t* data, uint64_t bytes) {
    return conversation_wire_payload_hash(data, bytes);
}

/// Make the Nth link-wrapped cudaMemcpy fail (0 = never); resets the call counter.
__attribute__((visibility("default"))) void ref_fail_copy_at(int n) {
    g_fail_copy_at = n;
    g_copy_calls = 0;
}

__attribute__((visibility("default"))) void ref_free(void* p) { std::free(p); }

}  // extern "C"
