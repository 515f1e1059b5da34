// include/strata_kv/types.hpp - the session types the handoff / park path reads, under the reference's names.
//
// The reference's own definitions live in its engine headers (ModelGeometry: include/strata/core/layout.hpp:27-60;
// QsaState: include/strata/core/layer.hpp:203-261; SessionState: include/strata/core/session.hpp:30-88;
// KvHostPools / KvStreamMap: include/strata/kernels/kv_stream.hpp:32-59).  Those headers pull in the whole
// engine (weights, kernels, the PLE run), so this build restates only the FIELDS this path reads, with the same
// names, types and defaults.  Code written against these compiles unchanged against the reference headers:
// define STRATA_KV_REFERENCE_HEADERS and put the reference's include directory on the path, and this header
// includes the reference's definitions instead.
#pragma once

#if defined(STRATA_KV_REFERENCE_HEADERS)
#include "strata/core/layer.hpp"
#include "strata/core/session.hpp"
#include "strata/kernels/kv_q4.hpp"
#else

#include <cstdint>

namespace strata::kernels {

/// The host copy of a streamed layer's K/V (identity layout, pinned and device-mapped).  Null when resident.
struct KvHostPools {
    uint16_t* k_pool = nullptr;
    uint16_t* v_pool = nullptr;
    int8_t* k_q = nullptr;
    int8_t* v_q = nullptr;
    uint16_t* k_scale = nullptr;
    uint16_t* v_scale = nullptr;
    uint8_t* k_q4 = nullptr;
    uint8_t* v_q4 = nullptr;
    bool present() const { return k_pool != nullptr || k_q != nullptr || k_q4 != nullptr; }
};

/// The residency map of a streamed layer (device arrays at fixed addresses).
struct KvStreamMap {
    int32_t* page_table = nullptr;
    int32_t* slot_block = nullptr;
    int32_t* slot_stamp = nullptr;
    int32_t* slot_ref = nullptr;
    int32_t* ctl = nullptr;
    int32_t* miss_block = nullptr;
    int32_t* miss_slot = nullptr;
    int64_t n_blocks = 0;
    int64_t n_slots = 0;
};

enum KvFormat : int { kKvF16 = 0, kKvInt8 = 1, kKvQ4 = 2 };

/// The QSA shapes (include/strata/kernels/qsa.hpp:96-117): zero by default, the real artifact's from
/// qsa_real_shapes().
struct QsaShapes {
    int64_t n_head = 0;
    int64_t n_head_kv = 0;
    int64_t head_dim = 0;
    int64_t n_rot = 0;
    int64_t idx_n_head = 0;
    int64_t idx_dim = 0;
    int64_t idx_block = 0;   ///< the indexer pools one key per idx_block cells
    int64_t idx_top_k = 0;
    int64_t page_size = 0;   ///< KV page granule in cells
};
inline QsaShapes qsa_real_shapes() {
    QsaShapes s;
    s.n_head = 24;
    s.n_head_kv = 2;
    s.head_dim = 256;
    s.n_rot = 64;
    s.idx_n_head = 4;
    s.idx_dim = 128;
    s.idx_block = 4;
    s.idx_top_k = 2048;
    s.page_size = 4;
    return s;
}

/// The per-query step record of the capturable QSA kernels (include/strata/kernels/qsa.hpp:156-162): the
/// selection width of query q is steps[q * kStepCount + kStepWidth].
enum QsaStep : int { kStepWidth = 3, kStepCount = 4 };

/// The pools a QSA reader addresses through `page_table` (include/strata/kernels/qsa_decode_attn.hpp:23-33).
struct QsaAttnPools {
    const uint16_t* k_pool = nullptr;
    const uint16_t* v_pool = nullptr;
    const int8_t* k_q = nullptr;
    const int8_t* v_q = nullptr;
    const uint16_t* k_scale = nullptr;
    const uint16_t* v_scale = nullptr;
    const uint8_t* k_q4 = nullptr;
    const uint8_t* v_q4 = nullptr;
    const int32_t* page_table = nullptr;
};

/// INT8 KV: one fp16 scale per 64 values (include/strata/kernels/kv_q8.hpp:22).
inline constexpr int KV_Q8_GROUP = 64;

/// The streaming map's control words: [0] epoch [1] hand [2] misses of the last call [3] overflow, u64 counters at
/// [4] misses, [6] lookups, [8] calls (include/strata/kernels/kv_stream.hpp:61).
inline constexpr int kKvCtlInts = 16;
inline uint64_t kv_stream_map_bytes(int64_t n_slots) { return (uint64_t) n_slots * 4 * 5 + kKvCtlInts * 4; }

/// Q4_0 rotated KV: 18-byte blocks of 32 values (include/strata/kernels/kv_q4.hpp:33).
inline uint64_t kv_q4_bytes_per_head(int head_dim) { return (uint64_t) (head_dim / 32) * 18u; }

/// PLE history rows and width (include/strata/kernels/ngram.hpp:39-40).
inline constexpr int NG_HC_DIM = 10240;
inline constexpr int NG_HIST = 9;

}  // namespace strata::kernels

namespace strata::core {

struct ModelGeometry {
    int64_t n_embd = 2560;
    int64_t n_layers = 48;
    int64_t qsa_interval = 4;
    int64_t ssm_state_size = 128;
    int64_t ssm_k_heads = 16;
    int64_t ssm_v_heads = 48;
    int64_t ssm_d_conv = 4;
    int64_t ssm_conv_channels = 10240;
    int64_t ssm_value_dim = 6144;
    int64_t n_head = 24;
    int64_t n_head_kv = 2;
    int64_t head_dim = 256;
    int64_t idx_q_heads = 4;
    int64_t idx_key_dim = 128;
    int64_t hc = 4;
    int64_t hc_lr = 320;
    int64_t n_expert = 512;
    int64_t n_ff = 640;

    int64_t n_qsa_layers() const { return n_layers / qsa_interval; }
    int64_t n_gdn_layers() const { return n_layers - n_qsa_layers(); }
};

/// One QSA layer's persistent state: the paged K/V pools with their page table, and the indexer rows.
/// A resident (kv_mode 0) layer whose pools lie inside a block pool created with skv_pool_create / skv_pool_wrap is
/// parked and mounted THROUGH `page_table` (device int32, logical page -> physical page), so a block-allocator
/// placement works; any other resident layer is identity-addressed, exactly as the reference assumes in mode 0.
struct QsaState {
    uint16_t* k_pool = nullptr;
    uint16_t* v_pool = nullptr;
    bool kv_int8 = false;
    int8_t* k_q = nullptr;
    int8_t* v_q = nullptr;
    uint16_t* k_scale = nullptr;
    uint16_t* v_scale = nullptr;
    bool kv_q4 = false;
    uint8_t* k_q4 = nullptr;
    uint8_t* v_q4 = nullptr;
    bool kv_hybrid = false;
    int32_t* page_table = nullptr;
    int64_t n_pages = 0;
    int64_t max_cells = 0;
    int kv_mode = 0;
    int64_t n_slots = 0;
    strata::kernels::KvHostPools host;
    strata::kernels::KvStreamMap map;
    int64_t idx_pooled_rows = 0;
    float* idx_tail = nullptr;
    float* idx_dead = nullptr;
    float* idx_pooled = nullptr;
    int32_t* idx_block_pos = nullptr;
};

inline int qsa_kv_format(const QsaState& st) {
    return st.kv_q4 ? strata::kernels::kKvQ4 : st.kv_int8 ? strata::kernels::kKvInt8 : strata::kernels::kKvF16;
}

/// The pools a reader of this layer addresses (the reference's src/core/layer.cpp:710-718).
inline strata::kernels::QsaAttnPools qsa_attn_pools(const QsaState& st) {
    strata::kernels::QsaAttnPools p;
    p.page_table = st.page_table;
    if (st.kv_hybrid) {
        p.k_q = st.k_q;
        p.k_scale = st.k_scale;
        p.v_q4 = st.v_q4;
    } else if (st.kv_q4) {
        p.k_q4 = st.k_q4;
        p.v_q4 = st.v_q4;
    } else if (st.kv_int8) {
        p.k_q = st.k_q;
        p.v_q = st.v_q;
        p.k_scale = st.k_scale;
        p.v_scale = st.v_scale;
    } else {
        p.k_pool = st.k_pool;
        p.v_pool = st.v_pool;
    }
    return p;
}

/// The per-sequence state a session owns: GDN rows, the QSA states of its layer carve, the PLE history.
struct SessionState {
    int64_t max_cells = 0;
    float* gdn_state = nullptr;
    QsaState* qsa_states = nullptr;
    int64_t layer_lo = 0, layer_hi = 0;
    int64_t qsa_ord0 = 0;
    int64_t qsa_alloc = 0;
    int64_t gdn_ord0 = 0;
    int64_t gdn_alloc = 0;
    int32_t ple_prev[2] = {-1, -1};
    int32_t ple_token = -1;
    float* ple_hist = nullptr;
};

}  // namespace strata::core

#endif
