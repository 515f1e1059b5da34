// skv_copy.cu - the sm_100a kernels of the KV handoff path.
//
// Every byte the path moves goes through ONE of two copy engines, driven by the same segment/tile plan:
//
//   copy_tma_kernel  a ring of kTmaStages shared-memory tiles per CTA (one CTA per SM).  One warp issues
//                    cp.async.bulk global->shared loads tracked by an mbarrier per stage, then
//                    cp.async.bulk shared->global stores tracked by bulk groups.  Table lookups are done
//                    32 pages at a time by the warp's lanes, and consecutive pages (the 64 pages of one
//                    256-token block are consecutive in a pool slot) merge into ONE bulk operation, so a
//                    32 KiB tile of K is one load and one store however the block table is permuted.
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

#include <cstdio>

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

__global__ void __launch_bounds__(32, 1) copy_tma_kernel(const __grid_constant__ CopyPlan plan, uint64_t total_tiles) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    StageStash* stash = reinterpret_cast<StageStash*>(smem + (size_t) kTmaStages * kTmaTileBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stash + kTmaStages);
    const int lane = (int) threadIdx.x;

    if (lane == 0)
        for (int s = 0; s < kTmaStages; ++s) mbar_init(&bars[s], 1);
    fence_proxy_async_smem();
    __syncwarp();

    const uint64_t first = blockIdx.x, step = gridDim.x;
    const uint64_t mine = first < total_tiles ? (total_tiles - first + step - 1) / step : 0;
    uint64_t issued = 0;
    for (; issued < mine && issued < (uint64_t) kTmaStages; ++issued)
        tma_issue_load(plan, first + issued * step, ring + (issued % kTmaStages) * kTmaTileBytes,
                       &bars[issued % kTmaStages], stash[issued % kTmaStages], lane);

    uint64_t k = 0;
    bool timed_out = false;
    for (; k < mine; ++k) {
        const int st = (int) (k % kTmaStages);
        const uint32_t phase = (uint32_t) ((k / kTmaStages) & 1u);
        if (!mbar_wait_bounded(&bars[st], phase)) {
            timed_out = true;
            break;
        }
        fence_proxy_async_smem();
        const uint32_t len = stash[st].store_len[lane];
        if (len) bulk_store(stash[st].store_addr[lane], ring + (size_t) st * kTmaTileBytes + stash[st].smem_off[lane], len);
        bulk_commit();
        // refill the stage of tile k-1 once its store has finished reading shared memory
        if (k >= 1 && issued < mine) {
            bulk_wait_read_1();
            __syncwarp();
            const int rs = (int) ((k - 1) % kTmaStages);
            tma_issue_load(plan, first + issued * step, ring + (size_t) rs * kTmaTileBytes, &bars[rs], stash[rs], lane);
            ++issued;
        }
    }
    if (timed_out) {
        if (lane == 0) atomicOr(plan.status, SKV_STATUS_WAIT_TIMEOUT);
        // drain the loads still in flight into this CTA's shared memory, each wait bounded again
        for (uint64_t j = k; j < issued; ++j)
            (void) mbar_wait_bounded(&bars[j % kTmaStages], (uint32_t) ((j / kTmaStages) & 1u));
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

int launch_copy(const CopyPlan& plan, uint64_t total_tiles, int engine, const DeviceCtx& ctx, cudaStream_t stream) {
    if (total_tiles == 0) return SKV_OK;
    if (engine == SKV_COPY_TMA) {
        const size_t smem = (size_t) kTmaStages * kTmaTileBytes + sizeof(StageStash) * kTmaStages + 8 * kTmaStages;
        static thread_local int configured_device = -1;
        if (configured_device != ctx.device) {
            const cudaError_t e = cudaFuncSetAttribute(copy_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(copy_tma_kernel)");
            configured_device = ctx.device;
        }
        const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms);
        copy_tma_kernel<<<grid, 32, smem, stream>>>(plan, total_tiles);
    } else {
        const unsigned grid = (unsigned) std::min<uint64_t>(total_tiles, (uint64_t) ctx.sms * 4);
        copy_vec_kernel<<<grid, kVecThreads, 0, stream>>>(plan, total_tiles);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "copy kernel launch");
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
