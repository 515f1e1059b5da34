// skv_copy.cu - the sm_100a kernels of the KV handoff path.
//
// Every byte the path moves goes through ONE of two copy engines, driven by the same segment/tile plan:
//
//   copy_tma_kernel  a ring of shared-memory tiles per CTA (geometry in the plan; by default 3 CTAs per SM,
//                    each 4 stages x 16 KiB, so three issuing warps per SM overlap their table loads).  One warp issues
//                    cp.async.bulk global->shared loads tracked by an mbarrier per stage, then
//                    cp.async.bulk shared->global stores tracked by bulk groups.  Table lookups are done
//                    32 pages at a time by the warp's lanes, and consecutive pages (the 64 pages of one
//                    256-token block are consecutive in a pool slot) merge into ONE bulk operation, so a
//                    tile of K is one load and one store however the block table is permuted.
//   copy_vec_kernel  16-byte vector loads (non-coherent, no L1 allocation) and stores, 4 in flight per
//                    thread, for destinations the bulk engine is not used on: peer memory (the P2P push
//                    over NVLink) and mapped pinned host memory (the direct park), and for page granules
//                    below 1 KiB.
//
// Both are pure data movement: HBM (or NVLink / PCIe) bound, no tensor-core work exists on this path.
// The address rule is the reference's reader/writer rule applied to whole pages
// (src/kernels/cuda/qsa.cu:121-142, 405-423): logical page p lives at base + table[p] * page_bytes.
//
// Every wait in these kernels is bounded by device time; a wait that runs out sets
// SKV_STATUS_WAIT_TIMEOUT in the status word, drains what this CTA has in flight (again bounded) and
// returns.  No trap, no assert, no unbounded spin.
#include "skv_internal.h"

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

namespace skv {
namespace {

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;   // 2 s of device time for any in-kernel wait

// ---------------------------------------------------------------- PTX helpers (sm_90+/sm_100a)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
/// Bounded wait for `phase` of `bar`; false when kWaitTimeoutNs of device time passed first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, phase)) return true;
        if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitTimeoutNs) return false;
    }
}
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st_plain(void* p, const uint4& v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------- the plan

/// The segment holding global tile `t` (binary search over the inclusive prefix sums).
__device__ __forceinline__ int locate(const CopyPlan& plan, uint64_t t) {
    int lo = 0, hi = plan.n_segs - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (t < plan.tile_end[mid]) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

struct Tile {
    const SegDev* sg;
    uint64_t local;   // tile index inside the segment
};
__device__ __forceinline__ Tile tile_of(const CopyPlan& plan, uint64_t t) {
    const int s = locate(plan, t);
    const uint64_t first = s ? plan.tile_end[s - 1] : 0;
    return {&plan.seg[s], t - first};
}

/// Validated table entries of `lane`'s page in a paged tile; contiguous sides use the identity.
struct LanePage {
    int64_t s, d;
    bool good;
};
__device__ __forceinline__ LanePage lane_page(const SegDev& sg, uint64_t page, bool in_tile, uint32_t* status) {
    LanePage r{0, 0, false};
    if (!in_tile) return r;
    r.s = sg.src_pages ? (int64_t) __ldg(sg.src_pages + page) : (int64_t) page;
    r.d = sg.dst_pages ? (int64_t) __ldg(sg.dst_pages + page) : (int64_t) page;
    const bool bad_s = sg.src_pages && (r.s < 0 || r.s >= sg.src_page_limit);
    const bool bad_d = sg.dst_pages && (r.d < 0 || r.d >= sg.dst_page_limit);
    if (bad_s) atomicOr(status, SKV_STATUS_BAD_SRC_PAGE);
    if (bad_d) atomicOr(status, SKV_STATUS_BAD_DST_PAGE);
    r.good = !bad_s && !bad_d;
    return r;
}

// ---------------------------------------------------------------- flag waits inside a copy launch

/// Lane 0 reads `flag` once (relaxed, system scope); the whole warp gets `flag >= value`.
__device__ __forceinline__ bool warp_flag_set(const uint64_t* flag, uint64_t value, int lane) {
    int ok = 0;
    if (lane == 0) {
        uint64_t v;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
        ok = v >= value;
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

/// Lane 0 polls `flag` >= value for at most timeout_ns with relaxed loads and a growing back-off (every CTA of the
/// grid may be polling the same word).  Returns the verdict to the whole warp.
__device__ __forceinline__ bool warp_wait_flag(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, int lane) {
    int ok = 1;
    if (lane == 0) {
        const uint64_t t0 = global_timer_ns();
        uint32_t pause = 32;
        for (;;) {
            uint64_t v;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
            if (v >= value) break;
            if (global_timer_ns() - t0 > timeout_ns) {
                ok = 0;
                break;
            }
            __nanosleep(pause);
            pause = min(pause * 2u, 1024u);
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

/// After a flag was seen set: an acquire read of it (lane 0; the flag only grows, so this read sees it set too),
/// then every lane orders its later bulk (async-proxy) loads after that acquire.
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* flag) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    return v;
}
__device__ __forceinline__ void warp_acquire_flag(const uint64_t* flag, int lane) {
    if (lane == 0) (void) ld_acquire_sys(flag);
    __syncwarp();
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- TMA bulk engine

/// Per-stage store instructions prepared at load time: lane l issues a bulk store of store_len[l] bytes
/// from smem offset l*page_bytes to store_addr[l] (0 length: nothing).
struct StageStash {
    uint8_t* store_addr[32];
    uint32_t store_len[32];
    uint32_t smem_off[32];
};

/// Warp-cooperative: issue the bulk loads of tile `t` into `buf`, arm `bar`, stash the stores.
__device__ __forceinline__ void tma_issue_load(const CopyPlan& plan, uint64_t t, uint8_t* buf, uint64_t* bar,
                                               StageStash& stash, int lane) {
    const Tile tl = tile_of(plan, t);
    const SegDev& sg = *tl.sg;
    if (sg.page_bytes == 0) {
        // both sides contiguous: one load, one store
        const uint64_t off = tl.local * sg.tile_bytes;
        const uint32_t len = (uint32_t) min(sg.tile_bytes, sg.bytes - off);
        if (lane == 0) {
            mbar_arrive_expect_tx(bar, len);
            bulk_load(buf, sg.src + off, len, bar);
            stash.store_addr[0] = sg.dst + off;
            stash.store_len[0] = len;
            stash.smem_off[0] = 0;
        } else {
            stash.store_len[lane] = 0;
        }
        return;
    }
    const uint64_t pb = sg.page_bytes;
    const uint64_t page0 = tl.local * sg.pages_per_tile;
    const uint64_t total_pages = sg.bytes / pb;
    const uint32_t np = (uint32_t) min((uint64_t) sg.pages_per_tile, total_pages - page0);
    const LanePage lp = lane_page(sg, page0 + lane, (uint32_t) lane < np, plan.status);
    const unsigned full = 0xffffffffu;
    const uint32_t good = __ballot_sync(full, lp.good);
    const int64_t prev_s = __shfl_up_sync(full, lp.s, 1);
    const int64_t prev_d = __shfl_up_sync(full, lp.d, 1);
    const bool prev_good = lane > 0 && ((good >> (lane - 1)) & 1u);
    // a lane continues the run of the lane before it when both are good and both sides advance by one page
    const bool cont_s = lp.good && prev_good && lp.s == prev_s + 1;
    const bool cont_d = lp.good && prev_good && lp.d == prev_d + 1;
    const uint32_t cs = __ballot_sync(full, cont_s);
    const uint32_t cd = __ballot_sync(full, cont_d);
    const uint32_t after = lane < 31 ? (full << (lane + 1)) : 0u;
    const uint32_t end_s = ~cs & after, end_d = ~cd & after;
    const uint32_t run_s = (end_s ? (uint32_t) (__ffs(end_s) - 1) : 32u) - (uint32_t) lane;
    const uint32_t run_d = (end_d ? (uint32_t) (__ffs(end_d) - 1) : 32u) - (uint32_t) lane;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t) __popc(good) * (uint32_t) pb);
    __syncwarp();
    if (lp.good && !cont_s) bulk_load(buf + (uint64_t) lane * pb, sg.src + (uint64_t) lp.s * pb, run_s * (uint32_t) pb, bar);
    const bool store_start = lp.good && !cont_d;
    stash.store_addr[lane] = store_start ? sg.dst + (uint64_t) lp.d * pb : nullptr;
    stash.store_len[lane] = store_start ? run_d * (uint32_t) pb : 0u;
    stash.smem_off[lane] = (uint32_t) lane * (uint32_t) pb;
}

/// The TMA engine's work for one CTA: a grid-stride share of the tiles through its ring.  Gated (copy_tma_gated_kernel):
/// the CTA first waits for the gate's flag (bounded; a wait that runs out moves nothing), and after its last store has
/// landed it reports to the gate's counters; the last CTA to report raises the done flag if every CTA moved all of
/// its tiles, then zeroes the counters for the next gated launch in stream order.
template <bool Gated>
__device__ __forceinline__ void tma_copy_body(const CopyPlan& plan, uint64_t total_tiles, const GateArgs& gate) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int stages = plan.tma_stages;
    const uint32_t tile = plan.tma_tile;
    uint8_t* ring = smem;
    StageStash* stash = reinterpret_cast<StageStash*>(smem + (size_t) stages * tile);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stash + stages);
    const int lane = (int) threadIdx.x;

    if (lane == 0)
        for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_proxy_async_smem();
    __syncwarp();

    const uint64_t first = blockIdx.x, step = gridDim.x;
    uint64_t mine = first < total_tiles ? (total_tiles - first + step - 1) / step : 0;
    [[maybe_unused]] bool gate_open = true;
    if constexpr (Gated) {
        if (gate.wait_flag) {
            if (warp_flag_set(gate.wait_flag, gate.wait_value, lane) ||
                warp_wait_flag(gate.wait_flag, gate.wait_value, gate.timeout_ns, lane)) {
                warp_acquire_flag(gate.wait_flag, lane);
            } else {
                if (lane == 0) atomicOr(plan.status, SKV_STATUS_WAIT_TIMEOUT);
                gate_open = false;
                mine = 0;
            }
        }
    }
    uint64_t issued = 0;
    for (; issued < mine && issued < (uint64_t) stages; ++issued)
        tma_issue_load(plan, first + issued * step, ring + (issued % stages) * tile, &bars[issued % stages],
                       stash[issued % stages], lane);

    uint64_t k = 0;
    bool timed_out = false;
    for (; k < mine; ++k) {
        const int st = (int) (k % stages);
        const uint32_t phase = (uint32_t) ((k / stages) & 1u);
        // warp-uniform verdict: every lane leaves the loop together, so no later collective splits the warp
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[st], phase))) {
            timed_out = true;
            break;
        }
        fence_proxy_async_smem();
        const uint32_t len = stash[st].store_len[lane];
        if (len) bulk_store(stash[st].store_addr[lane], ring + (size_t) st * tile + stash[st].smem_off[lane], len);
        bulk_commit();
        // refill the stage of tile k-1 once its store has finished reading shared memory
        if (k >= 1 && issued < mine) {
            bulk_wait_read_1();
            __syncwarp();
            const int rs = (int) ((k - 1) % stages);
            tma_issue_load(plan, first + issued * step, ring + (size_t) rs * tile, &bars[rs], stash[rs], lane);
            ++issued;
        }
    }
    if (timed_out) {
        if (lane == 0) atomicOr(plan.status, SKV_STATUS_WAIT_TIMEOUT);
        // drain the loads still in flight into this CTA's shared memory, each wait bounded again
        for (uint64_t j = k; j < issued; ++j)
            (void) mbar_wait_bounded(&bars[j % stages], (uint32_t) ((j / stages) & 1u));
    }
    bulk_wait_all();
    if constexpr (Gated) {
        if (gate.done_flag) {
            // this CTA's bulk stores have landed (wait_group 0); order them before the generic-proxy report
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                if (gate_open && !timed_out)
                    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(gate.counters + 1) : "memory");
                uint32_t before;
                // gpu-scope acq_rel: gathers every CTA's landed stores (and good count) into the last reporter's view
                asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(gate.counters) : "memory");
                if (before + 1 == gridDim.x) {
                    uint32_t good;
                    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(good) : "l"(gate.counters + 1) : "memory");
                    gate.counters[0] = 0;   // zero for the next gated launch (it starts after this one ends)
                    gate.counters[1] = 0;
                    // system-scope release, cumulative over what this thread acquired: a peer GPU that acquires the
                    // flag reads every byte of the copy
                    if (good == gridDim.x)
                        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(gate.done_flag), "l"(gate.done_value)
                                     : "memory");
                }
            }
        }
    }
}

__global__ void __launch_bounds__(32) copy_tma_kernel(const __grid_constant__ CopyPlan plan, uint64_t total_tiles) {
    tma_copy_body<false>(plan, total_tiles, GateArgs{});
}

/// skv_copy_gated: the TMA engine with the hand-off's READY wait before the first load and its DONE release after
/// the last store, inside the one launch.
__global__ void __launch_bounds__(32) copy_tma_gated_kernel(const __grid_constant__ CopyPlan plan, uint64_t total_tiles,
                                                            const __grid_constant__ GateArgs gate) {
    tma_copy_body<true>(plan, total_tiles, gate);
}

// ---------------------------------------------------------------- chained TMA engine
//
// skv_copy_chained: the TMA engine with segment c as chunk c of a pipeline.  CTAs CLAIM tiles (two consecutive
// at a time) from a global counter (not a static stride), so tiles are moved close to their global order and a chunk completes soon after
// its last tile is claimed - a static stride lets fast and slow CTAs drift apart over a long copy, and a chunk is
// only as done as its slowest CTA.  Before loading a tile of a chunk it has not seen released, a CTA checks
// wait_flags[c] >= value; if it is not yet set, the CTA first stores every tile it has loaded, then waits (lane
// 0, relaxed polls with back-off, bounded), then acquires.  When a CTA's next tile lies in a later chunk it waits
// for its bulk stores to land and adds its count for the chunk to landed[c] (gpu-scope release/acquire); the CTA
// that completes the count stores value to signal_flags[c] with release semantics at system scope, so a peer
// GPU that acquires that flag reads every byte of chunk c.  A wait that runs out stops new loads (status
// WAIT_TIMEOUT); loaded tiles are still stored, and a chunk is signalled only if every one of its tiles landed.

constexpr uint32_t kChainClaimBatch = 2;   // consecutive tiles per claim: fewer atomics, chunks still land in order

__global__ void __launch_bounds__(32) copy_tma_chain_kernel(const __grid_constant__ CopyPlan plan, uint64_t total_tiles,
                                                            const ChainArgs chain) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int stages = plan.tma_stages;
    const uint32_t tile = plan.tma_tile;
    uint8_t* ring = smem;
    StageStash* stash = reinterpret_cast<StageStash*>(smem + (size_t) stages * tile);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stash + stages);
    uint64_t* held = bars + stages;   // the global tile index each stage holds
    const int lane = (int) threadIdx.x;
    const unsigned full = 0xffffffffu;
    constexpr uint64_t kNone = ~0ull;

    if (lane == 0)
        for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_proxy_async_smem();
    __syncwarp();

    uint64_t pending = kNone;   // claimed, not yet loaded
    bool exhausted = false;     // the counter ran past the last tile
    uint64_t batch_next = 0, batch_end = 0;   // the rest of the last claimed batch
    auto claim = [&]() {        // warp-uniform, never blocks
        if (pending != kNone || exhausted) return;
        if (batch_next == batch_end) {
            unsigned long long t = 0;
            if (lane == 0) t = atomicAdd(chain.next_tile, (unsigned long long) kChainClaimBatch);
            t = __shfl_sync(full, t, 0);
            if (t >= total_tiles) {
                exhausted = true;
                return;
            }
            batch_next = t;
            batch_end = min((uint64_t) t + kChainClaimBatch, total_tiles);
        }
        pending = batch_next++;
    };
    int cleared = -1;      // the last chunk whose upstream flag this CTA has acquired
    bool stop = false;     // a flag wait ran out: no new loads
    uint64_t issued = 0;   // tiles this CTA has loaded ...
    uint64_t k = 0;        // ... and stored (positions in its own order; stage = position % stages)
    // Load while the ring has room.  The stage a load reuses held the tile at position issued - stages, already
    // stored; its bulk store has finished reading shared memory once at most the newest group is pending.
    auto fill = [&]() {
        while (!stop && issued < k + (uint64_t) stages - (k ? 1u : 0u)) {
            claim();
            if (pending == kNone) return;
            if (chain.wait_flags) {
                const int c = locate(plan, pending);
                if (c > cleared) {
                    const uint64_t* f = chain.wait_flags + c;
                    if (!warp_flag_set(f, chain.value, lane)) {
                        if (issued > k) return;   // not released yet: store what is loaded first
                        if (!warp_wait_flag(f, chain.value, chain.timeout_ns, lane)) {
                            if (lane == 0) atomicOr(plan.status, SKV_STATUS_WAIT_TIMEOUT);
                            stop = true;
                            return;
                        }
                    }
                    warp_acquire_flag(f, lane);
                    cleared = c;
                }
            }
            if (issued >= (uint64_t) stages) bulk_wait_read_1();
            const int st = (int) (issued % stages);
            if (lane == 0) held[st] = pending;
            __syncwarp();
            tma_issue_load(plan, pending, ring + (size_t) st * tile, &bars[st], stash[st], lane);
            pending = kNone;
            ++issued;
        }
    };

    fill();
    uint32_t count = 0;   // tiles of the current chunk this CTA stored and has not yet reported
    bool timed_out = false;
    while (k < issued) {
        const int st = (int) (k % stages);
        const uint32_t phase = (uint32_t) ((k / stages) & 1u);
        if (!__all_sync(full, mbar_wait_bounded(&bars[st], phase))) {
            timed_out = true;
            break;
        }
        fence_proxy_async_smem();
        const uint32_t len = stash[st].store_len[lane];
        if (len) bulk_store(stash[st].store_addr[lane], ring + (size_t) st * tile + stash[st].smem_off[lane], len);
        bulk_commit();
        const uint64_t t = held[st];
        ++k;
        if (chain.signal_flags) {
            const int c = locate(plan, t);
            ++count;
            // the next tile this CTA will store: already loaded, else the next claim (claiming never blocks)
            uint64_t next = kNone;
            if (k < issued) {
                next = held[k % stages];
            } else if (!stop) {
                claim();
                next = pending;
            }
            if (next == kNone || next >= plan.tile_end[c]) {   // leaving chunk c: report it
                bulk_wait_all();   // this CTA's bulk stores have landed
                asm volatile("fence.proxy.async.global;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    // gpu-scope release/acquire on the counter gathers every CTA's stores into the last reporter's
                    // view; its system-scope release store then publishes them (release is cumulative)
                    const uint64_t n_c = plan.tile_end[c] - (c ? plan.tile_end[c - 1] : 0);
                    uint32_t before;
                    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                                 : "=r"(before)
                                 : "l"(chain.landed + c), "r"(count)
                                 : "memory");
                    if ((uint64_t) before + count == n_c)
                        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(chain.signal_flags + c), "l"(chain.value)
                                     : "memory");
                }
                __syncwarp();
                count = 0;
            }
        }
        fill();
    }
    if (timed_out) {
        if (lane == 0) atomicOr(plan.status, SKV_STATUS_WAIT_TIMEOUT);
        for (uint64_t j = k; j < issued; ++j)
            (void) mbar_wait_bounded(&bars[j % stages], (uint32_t) ((j / stages) & 1u));
    }
    bulk_wait_all();
}

// ---------------------------------------------------------------- 16-byte vector engine

constexpr int kVecUnroll = 4;
constexpr uint32_t kVecMaxPages = 512;

__global__ void __launch_bounds__(kVecThreads) copy_vec_kernel(const __grid_constant__ CopyPlan plan, uint64_t total_tiles) {
    __shared__ int64_t s_src[kVecMaxPages];
    __shared__ int64_t s_dst[kVecMaxPages];
    for (uint64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const Tile tl = tile_of(plan, t);
        const SegDev& sg = *tl.sg;
        if (sg.page_bytes == 0) {
            const uint64_t off = tl.local * sg.tile_bytes;
            const uint32_t n16 = (uint32_t) (min(sg.tile_bytes, sg.bytes - off) >> 4);
            const uint8_t* src = sg.src + off;
            uint8_t* dst = sg.dst + off;
            for (uint32_t i = threadIdx.x; i < n16; i += kVecThreads * kVecUnroll) {
                uint4 v[kVecUnroll];
#pragma unroll
                for (int u = 0; u < kVecUnroll; ++u) {
                    const uint32_t e = i + (uint32_t) u * kVecThreads;
                    if (e < n16) v[u] = ld_stream(src + (uint64_t) e * 16);
                }
#pragma unroll
                for (int u = 0; u < kVecUnroll; ++u) {
                    const uint32_t e = i + (uint32_t) u * kVecThreads;
                    if (e < n16) st_plain(dst + (uint64_t) e * 16, v[u]);
                }
            }
            continue;
        }
        const uint32_t pb = sg.page_bytes;
        const uint64_t page0 = tl.local * sg.pages_per_tile;
        const uint32_t np = (uint32_t) min((uint64_t) sg.pages_per_tile, sg.bytes / pb - page0);
        __syncthreads();  // the previous tile's readers are done with s_src / s_dst
        for (uint32_t p = threadIdx.x; p < np; p += kVecThreads) {
            const LanePage lp = lane_page(sg, page0 + p, true, plan.status);
            s_src[p] = lp.good ? lp.s : -1;
            s_dst[p] = lp.good ? lp.d : -1;
        }
        __syncthreads();
        const uint32_t n16 = np * (pb >> 4);
        const uint32_t per_page16 = pb >> 4;
        for (uint32_t i = threadIdx.x; i < n16; i += kVecThreads * kVecUnroll) {
            uint4 v[kVecUnroll];
            int64_t da[kVecUnroll];
#pragma unroll
            for (int u = 0; u < kVecUnroll; ++u) {
                const uint32_t e = i + (uint32_t) u * kVecThreads;
                da[u] = -1;
                if (e < n16) {
                    const uint32_t p = e / per_page16, w = e - p * per_page16;
                    const int64_t s = s_src[p];
                    if (s >= 0) {
                        v[u] = ld_stream(sg.src + (uint64_t) s * pb + (uint64_t) w * 16);
                        da[u] = s_dst[p] * (int64_t) pb + (int64_t) w * 16;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kVecUnroll; ++u)
                if (da[u] >= 0) st_plain(sg.dst + da[u], v[u]);
        }
    }
}

// ---------------------------------------------------------------- completion flags

__global__ void signal_kernel(uint64_t* flag, uint64_t value) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(value) : "memory");
}

__global__ void wait_kernel(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, uint32_t* status) {
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        uint64_t v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
        if (v >= value) return;
        if (global_timer_ns() - t0 > timeout_ns) {
            atomicOr(status, SKV_STATUS_WAIT_TIMEOUT);
            return;
        }
        __nanosleep(256);
    }
}

}  // namespace

size_t tma_smem_bytes(int stages, uint32_t tile) {
    return (size_t) stages * tile + sizeof(StageStash) * (size_t) stages + 8 * (size_t) stages;
}

int launch_copy(const CopyPlan& plan, uint64_t total_tiles, int engine, DeviceCtx& ctx, cudaStream_t stream) {
    if (total_tiles == 0) return SKV_OK;
    const Tuning tu = tuning();
    if (engine == SKV_COPY_TMA) {
        const size_t smem = tma_smem_bytes(plan.tma_stages, plan.tma_tile);
        if (ctx.tma_smem_configured < smem) {
            const cudaError_t e = cudaFuncSetAttribute(copy_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(copy_tma_kernel)");
            ctx.tma_smem_configured = smem;
        }
        const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms * tu.tma_ctas_per_sm);
        copy_tma_kernel<<<grid, 32, smem, stream>>>(plan, total_tiles);
    } else {
        const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms * tu.vec_ctas_per_sm);
        copy_vec_kernel<<<grid, kVecThreads, 0, stream>>>(plan, total_tiles);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "copy kernel launch");
}

int launch_copy_gated(const CopyPlan& plan, uint64_t total_tiles, const GateArgs& gate, DeviceCtx& ctx,
                      cudaStream_t stream) {
    if (total_tiles == 0) return fail(SKV_EINVAL, "skv_copy_gated: nothing to move");
    const Tuning tu = tuning();
    const size_t smem = tma_smem_bytes(plan.tma_stages, plan.tma_tile);
    if (ctx.tma_gated_smem_configured < smem) {
        const cudaError_t e =
            cudaFuncSetAttribute(copy_tma_gated_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(copy_tma_gated_kernel)");
        ctx.tma_gated_smem_configured = smem;
    }
    const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms * tu.tma_ctas_per_sm);
    copy_tma_gated_kernel<<<grid, 32, smem, stream>>>(plan, total_tiles, gate);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "gated copy kernel launch");
}

int launch_copy_chained(const CopyPlan& plan, uint64_t total_tiles, const ChainArgs& chain, DeviceCtx& ctx,
                        cudaStream_t stream) {
    if (total_tiles == 0) return SKV_OK;
    const Tuning tu = tuning();
    const size_t smem = tma_smem_bytes(plan.tma_stages, plan.tma_tile) + 8 * (size_t) plan.tma_stages;   // + held[]
    if (ctx.tma_chain_smem_configured < smem) {
        const cudaError_t e =
            cudaFuncSetAttribute(copy_tma_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(copy_tma_chain_kernel)");
        ctx.tma_chain_smem_configured = smem;
    }
    cudaError_t e = cudaMemsetAsync(chain.landed, 0, kChainScratchBytes, stream);   // landed[] and next_tile
    if (e != cudaSuccess) return cuda_fail(e, "chained copy: counter reset");
    const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms * tu.tma_ctas_per_sm);
    copy_tma_chain_kernel<<<grid, 32, smem, stream>>>(plan, total_tiles, chain);
    e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "chained copy kernel launch");
}

namespace {
constexpr int kRangeBatch = 128;
struct RangeBatch {
    int n;
    uint32_t len[kRangeBatch];
    uint8_t* dst[kRangeBatch];
    const uint8_t* src[kRangeBatch];   // null: zero the range
};
/// One CTA per range (grid-stride over ranges), one byte per thread and step: the payload's alignment pads and its
/// few sub-16-byte or unaligned pieces (the bulk engines move everything else).
__global__ void byte_ranges_kernel(const __grid_constant__ RangeBatch b) {
    for (int r = blockIdx.x; r < b.n; r += gridDim.x) {
        uint8_t* d = b.dst[r];
        const uint8_t* s = b.src[r];
        for (uint32_t i = threadIdx.x; i < b.len[r]; i += blockDim.x) d[i] = s ? s[i] : uint8_t(0);
    }
}
}  // namespace

int byte_ranges(const std::vector<ByteRange>& ranges, cudaStream_t stream) {
    RangeBatch b;
    for (size_t i = 0; i < ranges.size();) {
        b.n = 0;
        for (; i < ranges.size() && b.n < kRangeBatch; ++i) {
            if (ranges[i].bytes == 0) continue;
            if (ranges[i].bytes > kByteRangeMaxBytes)
                return fail(SKV_EINVAL, "byte_ranges: a range above " + std::to_string(kByteRangeMaxBytes) + " bytes");
            b.len[b.n] = (uint32_t) ranges[i].bytes;
            b.dst[b.n] = ranges[i].dst;
            b.src[b.n] = ranges[i].src;
            ++b.n;
        }
        if (!b.n) continue;
        byte_ranges_kernel<<<b.n, 128, 0, stream>>>(b);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "byte_ranges");
    }
    return SKV_OK;
}

int launch_signal(uint64_t* flag, uint64_t value, cudaStream_t stream) {
    signal_kernel<<<1, 1, 0, stream>>>(flag, value);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "signal kernel launch");
}

int launch_wait(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, uint32_t* status, cudaStream_t stream) {
    wait_kernel<<<1, 1, 0, stream>>>(flag, value, timeout_ns, status);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "wait kernel launch");
}

}  // namespace skv

// ================================================================ allocation-free entry point
//
// skv_copy_noalloc: the vector copy engine for callers that must not allocate device memory.  The engine
// that skv_copy launches needs scratch beyond its inputs and outputs (its status word, which skv_copy
// cudaMallocs once per device), and its plan is capped at SKV_COPY_MAX_SEGMENTS by the kernel-parameter
// size.  Here both live in ONE file-scope device array of fixed size: the plan (up to
// SKV_NOALLOC_MAX_SEGMENTS segments) and the status word.  A small writer kernel fills the array in stream
// order from descriptors passed as kernel parameters, then the copy kernel reads it.
//
// Every call shares the array (one instance per device) and it keeps the last call's contents.  Calls
// issued on ONE stream from one host thread at a time are ordered and safe; calls that overlap on the GPU
// (different streams of the same device, or host threads racing on one stream) race on the plan and the status
// word.  The first call on a device performs the set-up (cudaGetSymbolAddress, which may load the module onto
// the device under lazy loading, and the SM count); make that first call at initialisation, before the token
// path and before any stream capture.
namespace skv {
namespace {

struct NoallocPlan {
    uint32_t status;       // SKV_STATUS_* bits of the current call; cleared by the writer of the first chunk
    uint32_t n_segs;
    uint64_t reserved;
    uint64_t tile_end[SKV_NOALLOC_MAX_SEGMENTS];
    SegDev seg[SKV_NOALLOC_MAX_SEGMENTS];
};
constexpr size_t kNoallocScratchBytes = (sizeof(NoallocPlan) + 255) / 256 * 256;

/// The scratch: a fixed-size array every GPU that loads the library holds until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kNoallocChunk = 128;   // descriptors per writer launch (about 10 KB of kernel parameters)

struct NoallocChunk {
    uint32_t first;        // index of chunk[0] in the plan
    uint32_t count;
    uint32_t n_segs;       // the whole plan's segment count
    uint32_t clear_status; // 1 on the first chunk of a call
    uint64_t tile_end[kNoallocChunk];
    SegDev seg[kNoallocChunk];
};

__global__ void noalloc_plan_writer(const __grid_constant__ NoallocChunk c, NoallocPlan* plan) {
    const uint32_t i = threadIdx.x;
    if (i < c.count) {
        plan->seg[c.first + i] = c.seg[i];
        plan->tile_end[c.first + i] = c.tile_end[i];
    }
    if (i == 0) {
        plan->n_segs = c.n_segs;
        if (c.clear_status) plan->status = 0;
    }
}

__device__ __forceinline__ int noalloc_locate(const NoallocPlan* plan, uint64_t t) {
    int lo = 0, hi = (int) plan->n_segs - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (t < plan->tile_end[mid]) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

/// The vector engine (same addressing, checks and status bits as copy_vec_kernel) over the scratch plan.
__global__ void __launch_bounds__(kVecThreads) copy_vec_noalloc_kernel(const NoallocPlan* plan, uint64_t total_tiles) {
    __shared__ int64_t s_src[kVecMaxPages];
    __shared__ int64_t s_dst[kVecMaxPages];
    uint32_t* status = const_cast<uint32_t*>(&plan->status);
    for (uint64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const int s = noalloc_locate(plan, t);
        const SegDev sg = plan->seg[s];
        const uint64_t local = t - (s ? plan->tile_end[s - 1] : 0);
        if (sg.page_bytes == 0) {
            const uint64_t off = local * sg.tile_bytes;
            const uint32_t n16 = (uint32_t) (min(sg.tile_bytes, sg.bytes - off) >> 4);
            for (uint32_t i = threadIdx.x; i < n16; i += kVecThreads * kVecUnroll) {
                uint4 v[kVecUnroll];
#pragma unroll
                for (int u = 0; u < kVecUnroll; ++u) {
                    const uint32_t e = i + (uint32_t) u * kVecThreads;
                    if (e < n16) v[u] = ld_stream(sg.src + off + (uint64_t) e * 16);
                }
#pragma unroll
                for (int u = 0; u < kVecUnroll; ++u) {
                    const uint32_t e = i + (uint32_t) u * kVecThreads;
                    if (e < n16) st_plain(sg.dst + off + (uint64_t) e * 16, v[u]);
                }
            }
            continue;
        }
        const uint32_t pb = sg.page_bytes;
        const uint64_t page0 = local * sg.pages_per_tile;
        const uint32_t np = (uint32_t) min((uint64_t) sg.pages_per_tile, sg.bytes / pb - page0);
        __syncthreads();
        for (uint32_t p = threadIdx.x; p < np; p += kVecThreads) {
            const LanePage lp = lane_page(sg, page0 + p, true, status);
            s_src[p] = lp.good ? lp.s : -1;
            s_dst[p] = lp.good ? lp.d : -1;
        }
        __syncthreads();
        const uint32_t per_page16 = pb >> 4;
        const uint32_t n16 = np * per_page16;
        for (uint32_t i = threadIdx.x; i < n16; i += kVecThreads * kVecUnroll) {
            uint4 v[kVecUnroll];
            int64_t da[kVecUnroll];
#pragma unroll
            for (int u = 0; u < kVecUnroll; ++u) {
                const uint32_t e = i + (uint32_t) u * kVecThreads;
                da[u] = -1;
                if (e < n16) {
                    const uint32_t p = e / per_page16, w = e - p * per_page16;
                    const int64_t src_page = s_src[p];
                    if (src_page >= 0) {
                        v[u] = ld_stream(sg.src + (uint64_t) src_page * pb + (uint64_t) w * 16);
                        da[u] = s_dst[p] * (int64_t) pb + (int64_t) w * 16;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kVecUnroll; ++u)
                if (da[u] >= 0) st_plain(sg.dst + da[u], v[u]);
        }
    }
}

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
NoallocPlan* g_noalloc_ptr[kNoallocMaxDevices] = {};
int g_noalloc_sms[kNoallocMaxDevices] = {};

/// Per-device set-up, once, with that device current: the scratch's device address and the SM count.
int noalloc_setup(int dev, NoallocPlan** plan, int* sms) {
    if (dev < 0 || dev >= kNoallocMaxDevices) return fail(SKV_EINVAL, "skv_copy_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "skv_copy_noalloc: cudaGetSymbolAddress");
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "skv_copy_noalloc: cudaDeviceGetAttribute");
        g_noalloc_sms[dev] = n;
        g_noalloc_ptr[dev] = static_cast<NoallocPlan*>(p);
    }
    *plan = g_noalloc_ptr[dev];
    *sms = g_noalloc_sms[dev];
    return SKV_OK;
}

}  // namespace
}  // namespace skv

extern "C" int skv_copy_noalloc(const skv_segment* segs, int n_segs, uint32_t* status_out, void* stream_ptr) {
    using namespace skv;
    if (n_segs < 0 || (n_segs && !segs)) return fail(SKV_EINVAL, "skv_copy_noalloc: bad segment list");
    if (n_segs > SKV_NOALLOC_MAX_SEGMENTS)
        return fail(SKV_ERANGE, "skv_copy_noalloc: " + std::to_string(n_segs) + " segments exceed the static plan's " +
                                    std::to_string(SKV_NOALLOC_MAX_SEGMENTS) + "-segment maximum");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "skv_copy_noalloc: cudaGetDevice");
    NoallocPlan* plan = nullptr;
    int sms = 0;
    if (const int rc = noalloc_setup(dev, &plan, &sms)) return rc;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

    // validate everything before enqueuing anything (the same rules as the vector engine of skv_copy)
    NoallocChunk chunk{};
    uint64_t total_tiles = 0;
    uint32_t kept = 0;
    int launched_chunks = 0;
    auto flush = [&](bool last) -> int {
        if (chunk.count == 0 && !(last && launched_chunks == 0)) return SKV_OK;
        chunk.clear_status = launched_chunks == 0 ? 1u : 0u;
        noalloc_plan_writer<<<1, kNoallocChunk, 0, stream>>>(chunk, plan);
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) return cuda_fail(le, "skv_copy_noalloc: plan writer launch");
        ++launched_chunks;
        chunk.first += chunk.count;
        chunk.count = 0;
        return SKV_OK;
    };
    // first pass: validation only
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& s = segs[i];
        if (s.bytes == 0) continue;
        const std::string where = "skv_copy_noalloc: segment " + std::to_string(i) + ": ";
        if (!s.src || !s.dst) return fail(SKV_EINVAL, where + "missing buffer");
        if ((reinterpret_cast<uintptr_t>(s.src) & 15u) || (reinterpret_cast<uintptr_t>(s.dst) & 15u) || s.bytes % 16)
            return fail(SKV_EINVAL, where + "buffers must be 16-byte aligned and bytes a multiple of 16");
        if (s.src_pages || s.dst_pages) {
            if (s.page_bytes == 0 || s.page_bytes % 16 || s.bytes % s.page_bytes)
                return fail(SKV_EINVAL, where + "a paged side needs page_bytes a multiple of 16 dividing bytes");
            if ((s.src_pages && s.src_page_limit <= 0) || (s.dst_pages && s.dst_page_limit <= 0))
                return fail(SKV_EINVAL, where + "a paged side needs a positive page limit");
        }
    }
    // second pass: the plan, written into the scratch by the writer kernel in chunks
    chunk.first = 0;
    chunk.count = 0;
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& s = segs[i];
        if (s.bytes == 0) continue;
        ++kept;
    }
    chunk.n_segs = kept;
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& s = segs[i];
        if (s.bytes == 0) continue;
        SegDev d{};
        d.src = static_cast<const uint8_t*>(s.src);
        d.dst = static_cast<uint8_t*>(s.dst);
        d.src_pages = s.src_pages;
        d.dst_pages = s.dst_pages;
        d.bytes = s.bytes;
        d.src_page_limit = s.src_page_limit;
        d.dst_page_limit = s.dst_page_limit;
        if (s.src_pages || s.dst_pages) {
            d.page_bytes = s.page_bytes;
            d.pages_per_tile = std::max<uint32_t>(1u, std::min<uint32_t>(512u, kVecTileBytes / s.page_bytes));
            d.tile_bytes = (uint64_t) d.pages_per_tile * s.page_bytes;
        } else {
            d.tile_bytes = kVecTileBytes;
        }
        total_tiles += (d.bytes + d.tile_bytes - 1) / d.tile_bytes;
        chunk.seg[chunk.count] = d;
        chunk.tile_end[chunk.count] = total_tiles;
        if (++chunk.count == (uint32_t) kNoallocChunk)
            if (const int rc = flush(false)) return rc;
    }
    if (const int rc = flush(true)) return rc;   // also clears the status word when every segment was empty
    if (total_tiles) {
        const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) sms * tuning().vec_ctas_per_sm);
        copy_vec_noalloc_kernel<<<grid, kVecThreads, 0, stream>>>(plan, total_tiles);
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) return cuda_fail(le, "skv_copy_noalloc: copy kernel launch");
    }
    if (status_out) {
        e = cudaMemcpyAsync(status_out, &plan->status, sizeof(uint32_t), cudaMemcpyDefault, stream);
        if (e != cudaSuccess) return cuda_fail(e, "skv_copy_noalloc: status copy");
    }
    return SKV_OK;
}
