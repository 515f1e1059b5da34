// tests/cpp/device_mount_formats_gpu_test.cpp - the device mount agrees with the host mount for every KV format
// and residency mode.
//
// For each format (fp16, int8 + scales, q4_0, hybrid K8V4) and each residency mode a format allows (resident,
// streamed, ring), a small whole-model session (one QSA layer, a ring-buffered draft, the running state) is filled
// with seeded bytes and parked (image A), encoded into an SR4H payload, and the payload is copied to device
// memory.  The session is then overwritten with other bytes and mounted from the DEVICE payload with
// conversation_wire_mount_device; a fresh park must equal A buffer for buffer.  The same round trip through the
// host path (conversation_snapshot_restore) must agree too, and a streamed layer's residency map must be evicted.
//
// Usage: device_mount_formats_gpu_test      (exit 0 = pass)
#include "strata_kv/conversation_snapshot.hpp"
#include "strata_kv/conversation_wire.hpp"
#include "strata_kv/conversation_wire_device.hpp"

#include <cuda_runtime.h>

#include <array>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace strata::core;
using namespace strata::kernels;

namespace {

int checks = 0;
void check(bool ok, const std::string& label) {
    ++checks;
    if (!ok) {
        std::fprintf(stderr, "FAIL: %s\n", label.c_str());
        std::exit(1);
    }
}
void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        std::fprintf(stderr, "FAIL: %s: %s\n", what, cudaGetErrorString(e));
        std::exit(1);
    }
}

/// Device and pinned allocations of one layer, freed together.
struct Allocs {
    std::vector<void*> dev, host;
    ~Allocs() {
        for (void* p : dev) cudaFree(p);
        for (void* p : host) cudaFreeHost(p);
    }
    template <class T>
    T* device(size_t bytes) {
        void* p = nullptr;
        cuda(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
        cuda(cudaMemset(p, 0, bytes ? bytes : 16), "cudaMemset");
        dev.push_back(p);
        return static_cast<T*>(p);
    }
    template <class T>
    T* pinned(size_t bytes) {
        void* p = nullptr;
        cuda(cudaHostAlloc(&p, bytes ? bytes : 16, cudaHostAllocMapped), "cudaHostAlloc");
        std::memset(p, 0, bytes ? bytes : 16);
        host.push_back(p);
        void* d = nullptr;
        cuda(cudaHostGetDevicePointer(&d, p, 0), "device pointer");
        return static_cast<T*>(d);
    }
};

constexpr int kHybrid = 3;

/// One QSA layer of `fmt` in residency `mode`: `pages` logical pages; `slots` VRAM pages when streamed or ring.
struct Layer {
    QsaState st;
    std::vector<std::pair<void*, size_t>> streams;   // every byte array the layer's state lives in (for filling)

    Layer(Allocs& a, const ModelGeometry& g, int fmt, int mode, int64_t pages, int64_t slots, bool index) {
        st.kv_mode = mode;
        st.kv_int8 = fmt == kKvInt8;
        st.kv_q4 = fmt == kKvQ4;
        st.kv_hybrid = fmt == kHybrid;
        st.n_pages = pages;
        st.n_slots = mode ? slots : pages;
        st.max_cells = pages * 4;
        const size_t rows = (size_t) (g.n_head_kv * 4);
        const size_t q4 = kv_q4_bytes_per_head((int) g.head_dim), scale = (size_t) (g.head_dim / KV_Q8_GROUP) * 2;
        const size_t f16 = (size_t) g.head_dim * 2, i8 = (size_t) g.head_dim;
        auto pool = [&](size_t per_row, size_t n_pages) { return rows * per_row * n_pages; };
        const size_t resident = (size_t) st.n_slots;
        auto both = [&](auto& dev_ptr, auto& host_ptr, size_t per_row) {
            using T = std::remove_pointer_t<std::remove_reference_t<decltype(dev_ptr)>>;
            dev_ptr = a.device<T>(pool(per_row, resident));
            streams.push_back({dev_ptr, pool(per_row, resident)});
            if (mode) {
                host_ptr = a.pinned<T>(pool(per_row, (size_t) pages));
                streams.push_back({host_ptr, pool(per_row, (size_t) pages)});
            }
        };
        if (fmt == kHybrid) {
            st.k_q = a.device<int8_t>(pool(i8, (size_t) pages));
            st.v_q4 = a.device<uint8_t>(pool(q4, (size_t) pages));
            st.k_scale = a.device<uint16_t>(pool(scale, (size_t) pages));
            streams.push_back({st.k_q, pool(i8, (size_t) pages)});
            streams.push_back({st.v_q4, pool(q4, (size_t) pages)});
            streams.push_back({st.k_scale, pool(scale, (size_t) pages)});
        } else if (fmt == kKvQ4) {
            both(st.k_q4, st.host.k_q4, q4);
            both(st.v_q4, st.host.v_q4, q4);
        } else if (fmt == kKvInt8) {
            both(st.k_q, st.host.k_q, i8);
            both(st.v_q, st.host.v_q, i8);
            both(st.k_scale, st.host.k_scale, scale);
            both(st.v_scale, st.host.v_scale, scale);
        } else {
            both(st.k_pool, st.host.k_pool, f16);
            both(st.v_pool, st.host.v_pool, f16);
        }
        st.idx_pooled_rows = index ? st.max_cells / 4 + 2 : 2;
        st.idx_pooled = a.device<float>((size_t) st.idx_pooled_rows * (size_t) g.idx_key_dim * 4);
        streams.push_back({st.idx_pooled, (size_t) st.idx_pooled_rows * (size_t) g.idx_key_dim * 4});
        st.page_table = a.device<int32_t>((size_t) pages * 4);
        if (mode == 1) {
            KvStreamMap& m = st.map;
            m.page_table = st.page_table;
            m.n_blocks = pages;
            m.n_slots = slots;
            m.slot_block = a.device<int32_t>((size_t) slots * 4);
            m.slot_stamp = a.device<int32_t>((size_t) slots * 4);
            m.slot_ref = a.device<int32_t>((size_t) slots * 4);
            m.miss_block = a.device<int32_t>((size_t) slots * 4);
            m.miss_slot = a.device<int32_t>((size_t) slots * 4);
            m.ctl = a.device<int32_t>(kKvCtlInts * 4);
        } else if (mode == 2) {
            kv_ring_table(st.page_table, pages, slots, nullptr);
        }
        if (index) {
            st.idx_tail = a.device<float>(3 * (size_t) g.idx_key_dim * 4);
            st.idx_dead = a.device<float>((size_t) g.idx_key_dim * 4);
            st.idx_block_pos = a.device<int32_t>(4);
            streams.push_back({st.idx_tail, 3 * (size_t) g.idx_key_dim * 4});
            streams.push_back({st.idx_dead, (size_t) g.idx_key_dim * 4});
            streams.push_back({st.idx_block_pos, 4});
        }
    }
};

void fill(const std::vector<std::pair<void*, size_t>>& arrays, uint8_t salt) {
    for (size_t i = 0; i < arrays.size(); ++i) {
        std::vector<uint8_t> bytes(arrays[i].second);
        for (size_t j = 0; j < bytes.size(); ++j) bytes[j] = (uint8_t) (salt * 131 + i * 29 + j * 7 + (j >> 9));
        cuda(cudaMemcpy(arrays[i].first, bytes.data(), bytes.size(), cudaMemcpyDefault), "fill");
    }
}

bool same_kv(const ConversationKv& a, const ConversationKv& b) {
    return a.format == b.format && a.cells == b.cells && a.k == b.k && a.v == b.v && a.k_scale == b.k_scale &&
           a.v_scale == b.v_scale && a.pooled == b.pooled;
}
bool same_state(const ConversationCheckpoint& a, const ConversationCheckpoint& b) {
    return a.ids == b.ids && a.gdn == b.gdn && a.ple == b.ple && a.tails == b.tails && a.dead == b.dead &&
           a.block_pos == b.block_pos;
}

void round_trip(int fmt, int mode) {
    const std::string tag = " (format " + std::to_string(fmt) + ", mode " + std::to_string(mode) + ")";
    ModelGeometry g;
    g.n_layers = 4;   // one QSA layer, three GDN layers
    g.ssm_state_size = 2;
    g.ssm_v_heads = 2;
    g.ssm_conv_channels = 8;
    Allocs a;
    Layer main(a, g, fmt, mode, 24, 6, true);
    Layer draft(a, g, fmt == kHybrid ? kKvInt8 : fmt, 2, 24, 6, false);
    SessionState ss;
    ss.max_cells = 96;
    ss.qsa_states = &main.st;
    ss.layer_hi = g.n_layers;
    ss.qsa_alloc = g.n_qsa_layers();
    ss.gdn_alloc = g.n_gdn_layers();
    std::string err;
    ConversationStateSizes z;
    check(conversation_state_sizes(g, z, err), "sizes" + tag);
    ss.gdn_state = a.device<float>(z.gdn);
    ss.ple_hist = a.device<float>(z.ple);
    std::vector<std::pair<void*, size_t>> all = main.streams;
    all.insert(all.end(), draft.streams.begin(), draft.streams.end());
    all.push_back({ss.gdn_state, z.gdn});
    all.push_back({ss.ple_hist, z.ple});
    std::vector<int32_t> ids(65);
    for (size_t i = 0; i < ids.size(); ++i) ids[i] = (int32_t) (i * 3 + 1);
    const std::vector<ConversationImageKey> images;
    std::vector<ConversationCheckpoint> checkpoints;
    fill(all, 11);
    // the indexer keeps its moving spare row equal to the dead key
    cuda(cudaMemcpy(main.st.idx_pooled + (ids.size() / 4) * (size_t) g.idx_key_dim, main.st.idx_dead, z.dead,
                    cudaMemcpyDefault),
         "spare row");
    {
        ConversationCheckpoint cp;   // a retained checkpoint travels in the payload too
        cp.ids.assign(ids.begin(), ids.begin() + 9);
        check(conversation_checkpoint_save(cp, ss, g, err), "retained checkpoint" + tag + ": " + err);
        checkpoints.push_back(std::move(cp));
    }
    const ConversationView view{ids, images, checkpoints, true};
    SavedConversation A;
    check(conversation_snapshot_save(A, view, ss, g, draft.st, err), "park A" + tag + ": " + err);
    VectorWireSink sink;
    WireEncoded enc;
    check(conversation_wire_encode(A, sink, {1, 2}, enc, err), "encode" + tag);
    uint8_t* payload = nullptr;
    cuda(cudaMalloc(&payload, sink.data().size()), "payload");
    cuda(cudaMemcpy(payload, sink.data().data(), sink.data().size(), cudaMemcpyHostToDevice), "payload upload");

    // device mount over other bytes
    fill(all, 77);
    SavedConversation meta;
    WireDecoded info;
    WireExpect ex;
    check(conversation_wire_mount_device(payload, sink.data().size(), ss, g, draft.st, ex, meta, info, err) ==
              ConversationRestore::restored,
          "device mount" + tag + ": " + err);
    check(meta.checkpoints.size() == 1 && same_state(meta.checkpoints[0], A.checkpoints[0]),
          "the retained checkpoint comes back to the host" + tag);
    if (mode == 1) {
        std::vector<int32_t> table(24);
        cuda(cudaMemcpy(table.data(), main.st.page_table, 96, cudaMemcpyDeviceToHost), "table");
        bool evicted = true;
        for (int32_t x : table) evicted &= x == -1;
        check(evicted, "a streamed layer's residency map is evicted" + tag);
    }
    SavedConversation B;
    check(conversation_snapshot_save(B, view, ss, g, draft.st, err), "park after the device mount" + tag + ": " + err);
    check(same_kv(B.kv[0], A.kv[0]) && same_kv(B.kv.back(), A.kv.back()) && same_state(B.live, A.live),
          "device mount then park equals the original park" + tag);
    uint64_t fp = 0;
    check(conversation_kv_verify(A.kv.back(), draft.st, g, (int64_t) ids.size(), false, fp, err),
          "the ring draft verifies after the device mount" + tag + ": " + err);

    // the host mount of the same image agrees
    fill(all, 201);
    check(conversation_snapshot_restore(A, ss, g, draft.st, err) == ConversationRestore::restored,
          "host mount" + tag + ": " + err);
    SavedConversation C;
    check(conversation_snapshot_save(C, view, ss, g, draft.st, err), "park after the host mount" + tag);
    check(same_kv(C.kv[0], B.kv[0]) && same_kv(C.kv.back(), B.kv.back()) && same_state(C.live, B.live),
          "host mount and device mount leave the same state" + tag);
    cudaFree(payload);
}

}  // namespace

int main() {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) return 77;
    cuda(cudaSetDevice(0), "cudaSetDevice");
    for (int fmt : {kKvF16, kKvInt8, kKvQ4})
        for (int mode : {0, 1, 2}) round_trip(fmt, mode);
    round_trip(kHybrid, 0);
    std::printf("device_mount_formats_gpu_test: %d checks passed\n", checks);
    return 0;
}
