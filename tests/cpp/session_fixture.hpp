// tests/cpp/session_fixture.hpp - the device sessions the C++ GPU test programs park, mount and hand off.
//
// Config 1 of the benchmark (full geometry; 12 QSA layers of fp16 K/V, 36 GDN rows, ids) placed into a block
// pool at seed-random slots: K pages and V pages of a 256-token block in the same slot (v_pool = k_pool + 64
// pages, one table for both).  The synthetic content comes from the test oracle's seeded generators
// (oracle/kv_oracle.c), the same calls tests/golden/make_golden.py made.
#pragma once

#include "strata_kv.h"
#include "strata_kv/conversation_snapshot.hpp"

extern "C" {
#include "kv_oracle.h"
}

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace fixture {

using namespace strata::core;

inline int checks = 0;
inline void check(bool ok, const char* label) {
    ++checks;
    if (!ok) {
        std::fprintf(stderr, "FAIL: %s\n", label);
        std::exit(1);
    }
}
inline void check_ok(bool ok, const std::string& err, const char* label) {
    ++checks;
    if (!ok) {
        std::fprintf(stderr, "FAIL: %s -> %s\n", label, err.c_str());
        std::exit(1);
    }
}
inline void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        std::fprintf(stderr, "FAIL: %s: %s\n", what, cudaGetErrorString(e));
        std::exit(1);
    }
}

/// The oracle's per-buffer seed rule (oracle/oracle.py layer_seed).
inline uint64_t layer_seed(uint64_t seed, uint64_t layer, uint64_t which) { return seed * 1000003ull + layer * 7919ull + which * 104729ull; }

constexpr int64_t kPageCells = 4, kBlockTokens = 256, kPagesPerBlock = kBlockTokens / kPageCells, kSlotPages = 128;

/// One session resident on the CURRENT device: every QSA layer (and the draft) paged into a block pool at seed-random
/// slots, K pages and V pages of a block in the same slot (v_pool = k_pool + 64 pages, one table for both).
struct DeviceSession {
    ModelGeometry g;
    int64_t tokens = 0, pages = 0, blocks = 0, page_bytes = 0;
    skv_pool* pool = nullptr;
    uint8_t* base = nullptr;
    int64_t pool_blocks = 0;
    std::vector<QsaState> qsa;     // n_qsa main layers
    QsaState draft;
    std::vector<std::vector<int32_t>> slots;       // per layer (main..., draft): block -> slot
    std::vector<std::vector<int32_t>> tables;      // per layer: host copy of the page table
    std::vector<int32_t*> dev_tables;
    std::vector<void*> allocations;
    float* gdn = nullptr;
    SessionState ss;

    template <class T>
    T* dev_alloc(size_t bytes) {
        void* p = nullptr;
        cuda(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
        cuda(cudaMemset(p, 0, bytes ? bytes : 16), "cudaMemset");
        allocations.push_back(p);
        return static_cast<T*>(p);
    }

    DeviceSession(const ModelGeometry& geometry, int64_t t, int64_t n_blocks, uint64_t placement_seed) : g(geometry), tokens(t) {
        pages = (t + kPageCells - 1) / kPageCells;
        blocks = (t + kBlockTokens - 1) / kBlockTokens;
        page_bytes = g.n_head_kv * kPageCells * g.head_dim * 2;
        pool_blocks = n_blocks;
        int device = 0;
        cuda(cudaGetDevice(&device), "cudaGetDevice");
        check(skv_pool_create(device, n_blocks, (uint64_t) (kSlotPages * page_bytes), &pool) == SKV_OK, "pool created");
        base = static_cast<uint8_t*>(skv_pool_base(pool));
        cuda(cudaMemset(base, 0, (size_t) n_blocks * kSlotPages * page_bytes), "pool zeroed");
        check(skv_pool_scramble(pool, placement_seed) == SKV_OK, "pool scrambled");
        const int64_t n_qsa = g.n_qsa_layers();
        const int64_t max_cells = blocks * kBlockTokens;
        const int64_t pooled_rows = max_cells / 4 + 2;
        auto make_layer = [&](QsaState& st, bool index) {
            std::vector<int32_t> s((size_t) blocks), table((size_t) (blocks * kPagesPerBlock));
            check(skv_alloc_blocks(pool, blocks, s.data()) == SKV_OK, "blocks allocated");
            check(skv_expand_block_table(s.data(), blocks, kPagesPerBlock, kSlotPages, 0, table.data()) == SKV_OK,
                  "table expanded");
            int32_t* dt = dev_alloc<int32_t>(table.size() * 4);
            cuda(cudaMemcpy(dt, table.data(), table.size() * 4, cudaMemcpyHostToDevice), "table upload");
            st = QsaState{};
            st.k_pool = reinterpret_cast<uint16_t*>(base);
            st.v_pool = reinterpret_cast<uint16_t*>(base + kPagesPerBlock * page_bytes);
            st.page_table = dt;
            st.n_pages = blocks * kPagesPerBlock;
            st.max_cells = max_cells;
            st.kv_mode = 0;
            st.n_slots = n_blocks * kSlotPages - kPagesPerBlock;   // pages addressable from k_pool AND from v_pool
            if (index) {
                st.idx_pooled_rows = pooled_rows;
                st.idx_pooled = dev_alloc<float>((size_t) pooled_rows * g.idx_key_dim * 4);
                st.idx_tail = dev_alloc<float>(3 * (size_t) g.idx_key_dim * 4);
                st.idx_dead = dev_alloc<float>((size_t) g.idx_key_dim * 4);
                st.idx_block_pos = dev_alloc<int32_t>(4);
            } else {
                st.idx_pooled_rows = 2;
            }
            slots.push_back(s);
            tables.push_back(table);
            dev_tables.push_back(dt);
        };
        qsa.resize((size_t) n_qsa);
        for (auto& st : qsa) make_layer(st, true);
        make_layer(draft, false);
        const size_t row = (size_t) (g.ssm_state_size * g.ssm_v_heads * g.ssm_state_size +
                                     g.ssm_conv_channels * (g.ssm_d_conv - 1));
        gdn = dev_alloc<float>((size_t) g.n_gdn_layers() * row * 4);
        ss = SessionState{};
        ss.max_cells = max_cells;
        ss.gdn_state = gdn;
        ss.qsa_states = qsa.data();
        ss.layer_hi = g.n_layers;
        ss.qsa_alloc = n_qsa;
        ss.gdn_alloc = g.n_gdn_layers();
    }
    ~DeviceSession() {
        for (void* p : allocations) cudaFree(p);
        skv_pool_destroy(pool);
    }
    const QsaState& layer(size_t j) const { return j < qsa.size() ? qsa[j] : draft; }

    /// Upload a layer's logical K or V image (pages * page_bytes) through its slots.
    void put(size_t j, int kv, const std::vector<uint8_t>& logical) {
        const int64_t block_bytes = kPagesPerBlock * page_bytes;
        for (int64_t b = 0; b < blocks; ++b) {
            const int64_t n = std::min<int64_t>(block_bytes, (int64_t) logical.size() - b * block_bytes);
            if (n <= 0) break;
            uint8_t* dst = base + ((int64_t) slots[j][(size_t) b] * kSlotPages + kv * kPagesPerBlock) * page_bytes;
            cuda(cudaMemcpy(dst, logical.data() + b * block_bytes, (size_t) n, cudaMemcpyHostToDevice), "page upload");
        }
    }
    /// Read a layer's logical K or V image back through its slots.
    std::vector<uint8_t> get(size_t j, int kv) const {
        std::vector<uint8_t> out((size_t) (pages * page_bytes));
        const int64_t block_bytes = kPagesPerBlock * page_bytes;
        for (int64_t b = 0; b < blocks; ++b) {
            const int64_t n = std::min<int64_t>(block_bytes, (int64_t) out.size() - b * block_bytes);
            if (n <= 0) break;
            const uint8_t* src = base + ((int64_t) slots[j][(size_t) b] * kSlotPages + kv * kPagesPerBlock) * page_bytes;
            cuda(cudaMemcpy(out.data() + b * block_bytes, src, (size_t) n, cudaMemcpyDeviceToHost), "page read");
        }
        return out;
    }
};

template <class T>
std::vector<uint8_t> as_bytes(const std::vector<T>& v) {
    std::vector<uint8_t> b(v.size() * sizeof(T));
    std::memcpy(b.data(), v.data(), b.size());
    return b;
}
inline std::vector<uint8_t> read_buffer(const ConversationBuffer& b) {
    std::vector<uint8_t> out(b.size());
    check(b.read(out.data(), 0, out.size()), "buffer readable");
    return out;
}
template <class T>
std::vector<T> from_device(const T* p, size_t n) {
    std::vector<T> v(n);
    cuda(cudaMemcpy(v.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost), "read back");
    return v;
}

/// The synthetic content of config 1 (oracle/oracle.py make_sequence).
struct Content {
    std::vector<std::vector<uint8_t>> k, v;                     // per layer incl. the draft
    std::vector<std::vector<float>> pooled, tail, dead;         // per QSA layer
    std::vector<int32_t> block_pos;
    std::vector<float> gdn;
    std::vector<int32_t> ids;
};
inline Content make_content(const DeviceSession& s, uint64_t seed) {
    Content c;
    const ModelGeometry& g = s.g;
    const uint64_t n16 = (uint64_t) (s.pages * s.page_bytes / 2);
    for (int64_t j = 0; j <= g.n_qsa_layers(); ++j) {
        std::vector<uint8_t> k(n16 * 2), v(n16 * 2);
        orc_fill_f16_normal(reinterpret_cast<uint16_t*>(k.data()), n16, layer_seed(seed, (uint64_t) j, 1), 0);
        orc_fill_f16_normal(reinterpret_cast<uint16_t*>(v.data()), n16, layer_seed(seed, (uint64_t) j, 2), 0);
        c.k.push_back(std::move(k));
        c.v.push_back(std::move(v));
    }
    const uint64_t cap_rows = (uint64_t) s.pages + 2;
    for (int64_t j = 0; j < g.n_qsa_layers(); ++j) {
        std::vector<float> p(cap_rows * (uint64_t) g.idx_key_dim), t(3 * (size_t) g.idx_key_dim), d((size_t) g.idx_key_dim);
        orc_fill_f32_normal(p.data(), p.size(), layer_seed(seed, (uint64_t) j, 3), 0, 1.0f);
        orc_fill_f32_normal(t.data(), t.size(), layer_seed(seed, (uint64_t) j, 4), 0, 1.0f);
        orc_fill_f32_normal(d.data(), d.size(), layer_seed(seed, (uint64_t) j, 5), 0, 1.0f);
        c.pooled.push_back(std::move(p));
        c.tail.push_back(std::move(t));
        c.dead.push_back(std::move(d));
        c.block_pos.push_back((int32_t) (s.tokens / 4));
    }
    const size_t row = (size_t) (g.ssm_state_size * g.ssm_v_heads * g.ssm_state_size + g.ssm_conv_channels * (g.ssm_d_conv - 1));
    c.gdn.resize((size_t) g.n_gdn_layers() * row);
    orc_fill_f32_normal(c.gdn.data(), c.gdn.size(), layer_seed(seed, 999, 6), 0, 0.02f);
    c.ids.resize((size_t) s.tokens);
    orc_fill_ids(c.ids.data(), c.ids.size(), layer_seed(seed, 999, 8), 151936);
    return c;
}

inline void upload(DeviceSession& s, const Content& c) {
    for (size_t j = 0; j < c.k.size(); ++j) {
        s.put(j, 0, c.k[j]);
        s.put(j, 1, c.v[j]);
    }
    for (size_t j = 0; j < s.qsa.size(); ++j) {
        const QsaState& st = s.qsa[j];
        const size_t rows = std::min<size_t>(c.pooled[j].size(), (size_t) st.idx_pooled_rows * (size_t) s.g.idx_key_dim);
        cuda(cudaMemcpy(st.idx_pooled, c.pooled[j].data(), rows * 4, cudaMemcpyHostToDevice), "pooled upload");
        cuda(cudaMemcpy(st.idx_tail, c.tail[j].data(), c.tail[j].size() * 4, cudaMemcpyHostToDevice), "tail upload");
        cuda(cudaMemcpy(st.idx_dead, c.dead[j].data(), c.dead[j].size() * 4, cudaMemcpyHostToDevice), "dead upload");
        cuda(cudaMemcpy(st.idx_block_pos, &c.block_pos[j], 4, cudaMemcpyHostToDevice), "block_pos upload");
    }
    cuda(cudaMemcpy(s.gdn, c.gdn.data(), c.gdn.size() * 4, cudaMemcpyHostToDevice), "gdn upload");
}

inline double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace fixture
