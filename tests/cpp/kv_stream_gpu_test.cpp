// tests/cpp/kv_stream_gpu_test.cpp - the block movers of streamed and ring layers on a real device, against the
// test oracle (oracle/kv_oracle.c orc_stream_resolve, the reference's residency policy restated sequentially).
//
// * kv_stream_reset clears a map filled with garbage;
// * 40 kv_stream_resolve calls with seeded selections (1-4 queries, ascending cell ids with locality, some calls
//   naming more distinct blocks than there are slots) leave the page table, every slot array, the control words
//   and the miss lists bit-identical to the oracle's after each call, for rings of 20, 96 and 1,500 slots and for
//   the fp16 and int8 formats; every resident slot holds its block's bytes from the host copy;
// * kv_ring_table, kv_ring_restore (wrapping ranges), kv_stage_from_host, kv_block_bytes, kv_stream_counters.
//
// Usage: kv_stream_gpu_test      (exit 0 = pass)
#include "strata_kv/kv_stream.hpp"

extern "C" {
#include "kv_oracle.h"
}

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

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
template <class T>
T* dev(size_t n) {
    void* p = nullptr;
    cuda(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
    return static_cast<T*>(p);
}
template <class T>
std::vector<T> down(const T* p, size_t n) {
    std::vector<T> v(n);
    cuda(cudaMemcpy(v.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost), "read back");
    return v;
}
template <class T>
void up(T* p, const std::vector<T>& v) {
    cuda(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
}

/// One streamed layer: the host copy (pinned, mapped), the VRAM slots and the residency map.
struct Layer {
    int fmt;
    int64_t n_blocks, n_slots;
    QsaShapes s = qsa_real_shapes();
    std::vector<uint32_t> len;          // per array, bytes per block
    std::vector<uint8_t*> host, slots;  // per array: the host copy as the device addresses it, the VRAM slots
    std::vector<const uint8_t*> mine;   // per array: the host copy as this process reads it
    KvHostPools hp;
    QsaAttnPools sp;
    KvStreamMap m;

    Layer(int format, int64_t blocks, int64_t n_slot, uint64_t seed) : fmt(format), n_blocks(blocks), n_slots(n_slot) {
        const uint32_t rows = (uint32_t) (s.n_head_kv * s.page_size);
        if (fmt == kKvInt8) len = {rows * (uint32_t) s.head_dim, rows * (uint32_t) s.head_dim,
                                   rows * (uint32_t) (s.head_dim / KV_Q8_GROUP) * 2, rows * (uint32_t) (s.head_dim / KV_Q8_GROUP) * 2};
        else len = {rows * (uint32_t) s.head_dim * 2, rows * (uint32_t) s.head_dim * 2};
        for (size_t a = 0; a < len.size(); ++a) {
            void* h = nullptr;
            cuda(cudaHostAlloc(&h, (size_t) (n_blocks * len[a]), cudaHostAllocMapped), "host copy");
            std::vector<uint16_t> fill((size_t) (n_blocks * len[a] / 2));
            orc_fill_f16_normal(fill.data(), fill.size(), seed * 31 + a, 0);
            std::memcpy(h, fill.data(), (size_t) (n_blocks * len[a]));
            mine.push_back(static_cast<const uint8_t*>(h));
            void* hd = nullptr;
            cuda(cudaHostGetDevicePointer(&hd, h, 0), "mapped pointer");
            host.push_back(static_cast<uint8_t*>(hd));
            slots.push_back(dev<uint8_t>((size_t) (n_slots * len[a])));
            cuda(cudaMemset(slots.back(), 0, (size_t) (n_slots * len[a])), "slots zero");
        }
        if (fmt == kKvInt8) {
            hp.k_q = (int8_t*) host[0]; hp.v_q = (int8_t*) host[1]; hp.k_scale = (uint16_t*) host[2]; hp.v_scale = (uint16_t*) host[3];
            sp.k_q = (int8_t*) slots[0]; sp.v_q = (int8_t*) slots[1]; sp.k_scale = (uint16_t*) slots[2]; sp.v_scale = (uint16_t*) slots[3];
        } else {
            hp.k_pool = (uint16_t*) host[0]; hp.v_pool = (uint16_t*) host[1];
            sp.k_pool = (uint16_t*) slots[0]; sp.v_pool = (uint16_t*) slots[1];
        }
        m.page_table = dev<int32_t>((size_t) n_blocks);
        m.slot_block = dev<int32_t>((size_t) n_slots);
        m.slot_stamp = dev<int32_t>((size_t) n_slots);
        m.slot_ref = dev<int32_t>((size_t) n_slots);
        m.ctl = dev<int32_t>(kKvCtlInts);
        m.miss_block = dev<int32_t>((size_t) n_slots);
        m.miss_slot = dev<int32_t>((size_t) n_slots);
        m.n_blocks = n_blocks;
        m.n_slots = n_slots;
        sp.page_table = m.page_table;
    }

    /// Every resident slot holds its block's bytes, in every array.
    bool slots_hold_their_blocks() const {
        const auto sb = down(m.slot_block, (size_t) n_slots);
        for (size_t a = 0; a < len.size(); ++a) {
            const auto got = down(slots[a], (size_t) (n_slots * len[a]));
            for (int64_t sl = 0; sl < n_slots; ++sl) {
                if (sb[(size_t) sl] < 0) continue;
                if (std::memcmp(got.data() + sl * len[a], mine[a] + (uint64_t) sb[(size_t) sl] * len[a], len[a]) != 0)
                    return false;
            }
        }
        return true;
    }
};

void resolve_series(int fmt, int64_t n_blocks, int64_t n_slots, uint64_t seed) {
    Layer L(fmt, n_blocks, n_slots, seed);
    const std::string tag = " (fmt " + std::to_string(fmt) + ", " + std::to_string(n_slots) + " slots)";
    // garbage, then a reset
    up(L.m.page_table, std::vector<int32_t>((size_t) n_blocks, 12345));
    up(L.m.ctl, std::vector<int32_t>(kKvCtlInts, 77));
    kv_stream_reset(L.m, nullptr);
    cuda(cudaDeviceSynchronize(), "reset");
    std::vector<int32_t> table = down(L.m.page_table, (size_t) n_blocks), sb = down(L.m.slot_block, (size_t) n_slots),
                         st = down(L.m.slot_stamp, (size_t) n_slots), rf = down(L.m.slot_ref, (size_t) n_slots),
                         ctl = down(L.m.ctl, kKvCtlInts);
    check(std::all_of(table.begin(), table.end(), [](int32_t x) { return x == -1; }) &&
              std::all_of(sb.begin(), sb.end(), [](int32_t x) { return x == -1; }) &&
              std::all_of(st.begin(), st.end(), [](int32_t x) { return x == -1; }) &&
              std::all_of(rf.begin(), rf.end(), [](int32_t x) { return x == 0; }) &&
              std::all_of(ctl.begin(), ctl.end(), [](int32_t x) { return x == 0; }),
          "reset evicts everything" + tag);
    std::vector<int32_t> mb((size_t) n_slots, 0), ms((size_t) n_slots, 0);
    std::mt19937_64 rng(seed);
    const int64_t cap = 512;
    int32_t* d_ids = dev<int32_t>(4 * cap);
    int32_t* d_steps = dev<int32_t>(16);
    for (int call = 0; call < 40; ++call) {
        const int n_q = 1 + (int) (rng() % 4);
        std::vector<int32_t> ids((size_t) (4 * cap), 0), steps(16, 0);
        for (int q = 0; q < n_q; ++q) {
            // a few runs of consecutive cells at random places: locality like a real selection
            std::vector<int32_t> cells;
            const int runs = 1 + (int) (rng() % 3);
            const int64_t span = (call % 7 == 6) ? n_blocks * 4 : std::min<int64_t>(n_blocks * 4, 8 * n_slots);
            for (int r = 0; r < runs; ++r) {
                const int64_t start = (int64_t) (rng() % (uint64_t) span);
                const int64_t n = 1 + (int64_t) (rng() % (uint64_t) std::max<int64_t>(4, n_slots));
                for (int64_t c = start; c < std::min<int64_t>(start + n, n_blocks * 4); ++c) cells.push_back((int32_t) c);
            }
            std::sort(cells.begin(), cells.end());
            cells.erase(std::unique(cells.begin(), cells.end()), cells.end());
            if ((int64_t) cells.size() > cap) cells.resize((size_t) cap);
            std::copy(cells.begin(), cells.end(), ids.begin() + q * cap);
            steps[(size_t) (q * kStepCount + kStepWidth)] = (int32_t) cells.size();
        }
        up(d_ids, ids);
        up(d_steps, steps);
        kv_stream_resolve(L.m, L.sp, L.hp, fmt, d_ids, d_steps, n_q, cap, L.s, nullptr);
        cuda(cudaDeviceSynchronize(), "resolve");
        const int64_t placed = orc_stream_resolve(table.data(), sb.data(), st.data(), rf.data(), ctl.data(), mb.data(),
                                                  ms.data(), n_blocks, n_slots, ids.data(), steps.data(), n_q, cap,
                                                  L.s.page_size);
        const std::string at = " after call " + std::to_string(call) + tag;
        check(down(L.m.page_table, (size_t) n_blocks) == table, "page table equals the oracle's" + at);
        check(down(L.m.slot_block, (size_t) n_slots) == sb, "slot -> block equals the oracle's" + at);
        check(down(L.m.slot_stamp, (size_t) n_slots) == st, "slot stamps equal the oracle's" + at);
        check(down(L.m.slot_ref, (size_t) n_slots) == rf, "reference bits equal the oracle's" + at);
        check(down(L.m.ctl, kKvCtlInts) == ctl, "control words equal the oracle's" + at);
        const auto gmb = down(L.m.miss_block, (size_t) n_slots), gms = down(L.m.miss_slot, (size_t) n_slots);
        check(std::equal(gmb.begin(), gmb.begin() + placed, mb.begin()) &&
                  std::equal(gms.begin(), gms.begin() + placed, ms.begin()),
              "the placed misses and their slots equal the oracle's" + at);
        check(L.slots_hold_their_blocks(), "every resident slot holds its block's bytes" + at);
    }
    const KvStreamCounters c = kv_stream_counters(L.m);
    uint64_t u[3];
    std::memcpy(u, ctl.data() + 4, sizeof u);
    check(c.misses == u[0] && c.lookups == u[1] && c.calls == 40 && c.overflow == (ctl[3] != 0),
          "kv_stream_counters reads the control words" + tag);
    std::printf("  resolve%s: %llu misses placed over %llu lookups, overflow %d\n", tag.c_str(),
                (unsigned long long) c.misses, (unsigned long long) c.lookups, (int) c.overflow);
}

void ring_and_stage() {
    const int64_t n_blocks = 50, n_slots = 8;
    Layer L(kKvF16, n_blocks, n_slots, 99);
    kv_ring_table(L.m.page_table, n_blocks, n_slots, nullptr);
    const auto table = down(L.m.page_table, (size_t) n_blocks);
    bool ring = true;
    for (int64_t b = 0; b < n_blocks; ++b) ring &= table[(size_t) b] == (int32_t) (b % n_slots);
    check(ring, "kv_ring_table is block % n_slots");
    for (auto [b0, b1] : std::vector<std::pair<int64_t, int64_t>>{{0, 5}, {37, 45}, {42, 50}, {3, 3}}) {
        kv_ring_restore(L.sp, L.hp, kKvF16, b0, b1, n_slots, L.s, nullptr);
        cuda(cudaDeviceSynchronize(), "ring restore");
        bool ok = true;
        for (size_t a = 0; a < L.len.size(); ++a) {
            const auto got = down(L.slots[a], (size_t) (n_slots * L.len[a]));
            for (int64_t b = b0; b < b1; ++b)
                ok &= std::memcmp(got.data() + (b % n_slots) * L.len[a], L.mine[a] + (uint64_t) b * L.len[a], L.len[a]) == 0;
        }
        check(ok, "kv_ring_restore [" + std::to_string(b0) + ", " + std::to_string(b1) + ") lands in slots b % n_slots");
    }
    // stage: the first n blocks of the host copy into an identity-layout pool
    std::vector<uint8_t*> stage;
    QsaAttnPools sp;
    for (size_t a = 0; a < L.len.size(); ++a) stage.push_back(dev<uint8_t>((size_t) (n_blocks * L.len[a])));
    sp.k_pool = (const uint16_t*) stage[0];
    sp.v_pool = (const uint16_t*) stage[1];
    kv_stage_from_host(sp, L.hp, kKvF16, 33, L.s, nullptr);
    cuda(cudaDeviceSynchronize(), "stage");
    bool ok = true;
    for (size_t a = 0; a < L.len.size(); ++a) {
        const auto got = down(stage[a], (size_t) (33 * L.len[a]));
        ok &= std::memcmp(got.data(), L.mine[a], got.size()) == 0;
    }
    check(ok, "kv_stage_from_host copies the first blocks");
    const QsaShapes s = qsa_real_shapes();
    check(kv_block_bytes(s, kKvF16) == 2 * 8 * 256 * 2 && kv_block_bytes(s, kKvInt8) == 2 * 8 * 256 + 2 * 8 * 4 * 2 &&
              kv_block_bytes(s, kKvQ4) == 2 * 8 * 144,
          "kv_block_bytes per format");
}

}  // namespace

int main() {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) return 77;
    cuda(cudaSetDevice(0), "cudaSetDevice");
    resolve_series(kKvF16, 400, 96, 1);
    resolve_series(kKvF16, 300, 20, 2);
    resolve_series(kKvInt8, 3000, 1500, 3);
    ring_and_stage();
    std::printf("kv_stream_gpu_test: %d checks passed\n", checks);
    return 0;
}
