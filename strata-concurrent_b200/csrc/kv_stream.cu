// kv_stream.cu - the block movers of streamed (kv_mode 1) and ring (kv_mode 2) QSA layers on sm_100a
// (include/strata_kv/kv_stream.hpp; the reference's interface is include/strata/kernels/kv_stream.hpp:62-96).
//
//   reset_kernel     evict every block: page table -1, slots free, control words zero (grid-stride)
//   ring_kernel      the static ring table block -> block % n_slots
//   resolve_kernel   one CTA of 1,024 threads: (1) every selected block is looked up once per query - a resident
//                    block takes the call's epoch and its reference bit, a missing one is claimed (-1 -> -2) and
//                    appended to the miss list in (query, position) order by a CTA-wide scan; (2) warp 0 sweeps the
//                    CLOCK hand 32 slots at a time with ballots: a slot this call uses is never taken, a free or
//                    unreferenced one is taken for the next miss, a referenced one loses its bit as the hand passes
//                    (second chance), and the hand stops just past the last slot taken; (3) the table is re-pointed
//   fill_kernel      one CTA per missed block copies its runs from the host copy (zero-copy over PCIe) into its slot
//
// The ring restore and the stage-from-host are DMA copies of whole block runs (the copy engine moves pinned host
// memory at the link's rate); they are not capturable, exactly as in the reference.
#include "kv_stream_detail.h"
#include "skv_internal.h"

#include <algorithm>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace skv {
namespace {

using strata::kernels::KvHostPools;
using strata::kernels::KvStreamMap;
using strata::kernels::QsaAttnPools;
using strata::kernels::QsaShapes;

constexpr int kResolveThreads = 1024;

/// The byte runs of one block in each array a format keeps (K and V; for int8 also both scale arrays): block b of
/// array a is bytes [b * len[a], (b + 1) * len[a]) of the host copy and of the slot pool alike.
struct BlockRuns {
    const uint8_t* host[4];
    uint8_t* slot[4];
    uint32_t len[4];
    int n;
};

BlockRuns block_runs(const QsaAttnPools& slots, const KvHostPools& host, int fmt, const QsaShapes& s) {
    const uint64_t rows = (uint64_t) (s.n_head_kv * s.page_size);
    BlockRuns r{};
    auto add = [&r](const void* h, const void* d, uint64_t len) {
        r.host[r.n] = static_cast<const uint8_t*>(h);
        r.slot[r.n] = const_cast<uint8_t*>(static_cast<const uint8_t*>(d));
        r.len[r.n] = (uint32_t) len;
        ++r.n;
    };
    if (fmt == strata::kernels::kKvQ4) {
        const uint64_t len = rows * strata::kernels::kv_q4_bytes_per_head((int) s.head_dim);
        add(host.k_q4, slots.k_q4, len);
        add(host.v_q4, slots.v_q4, len);
    } else if (fmt == strata::kernels::kKvInt8) {
        const uint64_t codes = rows * (uint64_t) s.head_dim;
        const uint64_t scales = rows * (uint64_t) (s.head_dim / strata::kernels::KV_Q8_GROUP) * 2;
        add(host.k_q, slots.k_q, codes);
        add(host.v_q, slots.v_q, codes);
        add(host.k_scale, slots.k_scale, scales);
        add(host.v_scale, slots.v_scale, scales);
    } else {
        const uint64_t len = rows * (uint64_t) s.head_dim * 2;
        add(host.k_pool, slots.k_pool, len);
        add(host.v_pool, slots.v_pool, len);
    }
    return r;
}

__global__ void reset_kernel(KvStreamMap m) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t i = i0; i < m.n_blocks; i += stride) m.page_table[i] = -1;
    for (int64_t i = i0; i < m.n_slots; i += stride) {
        m.slot_block[i] = -1;
        m.slot_stamp[i] = -1;
        m.slot_ref[i] = 0;
    }
    if (i0 < strata::kernels::kKvCtlInts) m.ctl[i0] = 0;
}

__global__ void ring_kernel(int32_t* table, int64_t n_blocks, int64_t n_slots) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n_blocks; i += stride)
        table[i] = (int32_t) (i % n_slots);
}

/// CTA-wide exclusive prefix sum of one int per thread; `total` gets the CTA's sum.  Every thread must call it.
__device__ int cta_exclusive_sum(int v, int* warp_totals, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    int incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int up = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += up;
    }
    if (lane == 31) warp_totals[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int t = lane < warps ? warp_totals[lane] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int up = __shfl_up_sync(0xffffffffu, t, d);
            if (lane >= d) t += up;
        }
        warp_totals[lane] = t;   // inclusive prefix over warps
    }
    __syncthreads();
    total = warp_totals[warps - 1];
    const int before = warp ? warp_totals[warp - 1] : 0;
    __syncthreads();   // warp_totals may be reused by the next call
    return before + incl - v;
}

__global__ void __launch_bounds__(kResolveThreads) resolve_kernel(KvStreamMap m, const int32_t* __restrict__ ids,
                                                                  const int32_t* __restrict__ steps, int n_q, int cap,
                                                                  int page_size) {
    __shared__ int warp_totals[32];
    __shared__ int s_lookups, s_hand, s_got, s_overflow;
    const int tid = threadIdx.x, lane = tid & 31;
    const int epoch = m.ctl[0] + 1;
    const int n = (int) m.n_slots;
    if (tid == 0) {
        s_lookups = 0;
        s_overflow = 0;
    }
    __syncthreads();

    // 1. lookups and claims, the miss list in (query, position) order
    int n_miss = 0, lookups = 0;
    for (int q = 0; q < n_q; ++q) {
        const int width = min(steps[q * strata::kernels::kStepCount + strata::kernels::kStepWidth], cap);
        const int32_t* qi = ids + (int64_t) q * cap;
        for (int base = 0; base < width; base += kResolveThreads) {
            const int i = base + tid;
            int miss = 0, b = -1;
            if (i < width) {
                b = qi[i] / page_size;
                if ((i == 0 || qi[i - 1] / page_size != b) && b >= 0 && b < m.n_blocks) {   // one lookup per block
                    ++lookups;
                    const int sl = m.page_table[b];
                    if (sl >= 0) {
                        if (sl < n) {   // a table entry past the slots is never followed
                            m.slot_stamp[sl] = epoch;
                            m.slot_ref[sl] = 1;
                        }
                    } else if (sl == -1 && atomicCAS(&m.page_table[b], -1, -2) == -1) {
                        miss = 1;
                    }
                }
            }
            int total = 0;
            const int at = n_miss + cta_exclusive_sum(miss, warp_totals, total);
            if (miss) {
                if (at < n) {
                    m.miss_block[at] = b;
                } else {   // more distinct misses than slots: the block stays evicted
                    m.page_table[b] = -1;
                    s_overflow = 1;
                }
            }
            n_miss += total;
            __syncthreads();   // this chunk's claims are visible to the next
        }
    }
    atomicAdd(&s_lookups, lookups);
    const int need = min(n_miss, n);

    // 2. victims: the CLOCK hand, 32 slots per step, by warp 0
    if (tid < 32) {
        int hand = m.ctl[1], got = 0;
        for (int scanned = 0; got < need && scanned < 3 * n;) {
            const int w = min(min(32, n), 3 * n - scanned);   // the hand walks at most three laps
            scanned += w;
            const bool on = lane < w;
            const int j = on ? (int) (((int64_t) hand + lane) % n) : 0;
            const bool mine = on && m.slot_stamp[j] == epoch;
            const bool cand = on && !mine && (m.slot_block[j] < 0 || m.slot_ref[j] == 0);
            const unsigned cmask = __ballot_sync(0xffffffffu, cand);
            const int want = need - got, avail = __popc(cmask);
            int cut = w;
            if (avail >= want) {   // the hand stops just past the want-th candidate
                unsigned rest = cmask;
                for (int k = 1; k < want; ++k) rest &= rest - 1;
                cut = __ffs(rest);
            }
            const int rank = __popc(cmask & ((1u << lane) - 1u));
            if (cand && rank < want) {
                m.miss_slot[got + rank] = j;
                m.slot_stamp[j] = epoch;   // taken: a sweep that laps must not take it again
            } else if (on && lane < cut && !mine) {
                m.slot_ref[j] = 0;         // passed: second chance spent
            }
            got += min(avail, want);
            hand = (int) (((int64_t) hand + cut) % n);
            __syncwarp();
        }
        if (lane == 0) {
            s_hand = hand;
            s_got = got;
        }
    }
    __syncthreads();

    // 3. re-point the table (the fill kernel copies the bytes)
    const int placed = min(s_got, need);
    for (int k = tid; k < n_miss && k < n; k += kResolveThreads) {
        const int b = m.miss_block[k];
        if (k >= placed) {
            m.page_table[b] = -1;
            continue;
        }
        const int sl = m.miss_slot[k];
        const int old = m.slot_block[sl];
        if (old >= 0 && old < m.n_blocks) m.page_table[old] = -1;
        m.slot_block[sl] = b;
        m.slot_stamp[sl] = epoch;
        m.slot_ref[sl] = 1;
        m.page_table[b] = sl;
    }
    __syncthreads();
    if (tid == 0) {
        m.ctl[0] = epoch;
        m.ctl[1] = s_hand;
        m.ctl[2] = placed;
        if (placed < n_miss || s_overflow) m.ctl[3] = 1;
        unsigned long long* c = reinterpret_cast<unsigned long long*>(m.ctl + 4);
        c[0] += (unsigned long long) placed;
        c[1] += (unsigned long long) s_lookups;
        c[2] += 1ull;
    }
}

/// One CTA per placed miss (grid-stride): the block's runs from the host copy into its slot, 16 bytes per thread.
__global__ void fill_kernel(KvStreamMap m, BlockRuns r) {
    const int placed = m.ctl[2];
    for (int k = blockIdx.x; k < placed; k += gridDim.x) {
        const int64_t b = m.miss_block[k], sl = m.miss_slot[k];
        for (int a = 0; a < r.n; ++a) {
            const uint4* src = reinterpret_cast<const uint4*>(r.host[a] + b * r.len[a]);
            uint4* dst = reinterpret_cast<uint4*>(r.slot[a] + sl * r.len[a]);
            for (uint32_t i = threadIdx.x; i < r.len[a] / 16; i += blockDim.x) dst[i] = src[i];
        }
    }
}

int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, what);
}

/// The reference's wrappers end the process on a CUDA failure (src/kernels/cuda/kv_stream.cu:15-21); these public
/// functions keep that contract.  The snapshot layer calls the status-returning forms instead.
void or_exit(int rc) {
    if (rc == SKV_OK) return;
    std::fprintf(stderr, "kv_stream: %s\n", skv_last_error());
    std::exit(1);
}

}  // namespace

int stream_reset(const KvStreamMap& m, cudaStream_t stream) {
    if (!m.page_table || !m.slot_block || !m.slot_stamp || !m.slot_ref || !m.ctl)
        return fail(SKV_EINVAL, "kv_stream_reset: incomplete streaming map");
    reset_kernel<<<128, 256, 0, stream>>>(m);
    return launched("kv_stream_reset");
}

int ring_table(int32_t* table, int64_t n_blocks, int64_t n_slots, cudaStream_t stream) {
    if (n_blocks <= 0) return SKV_OK;
    if (!table || n_slots <= 0) return fail(SKV_EINVAL, "kv_ring_table: no table or no slots");
    ring_kernel<<<64, 256, 0, stream>>>(table, n_blocks, n_slots);
    return launched("kv_ring_table");
}

int ring_restore(const QsaAttnPools& slots, const KvHostPools& host, int fmt, int64_t b0, int64_t b1, int64_t n_slots,
                 const QsaShapes& s, cudaStream_t stream) {
    if (b1 <= b0) return SKV_OK;
    if (b0 < 0 || n_slots <= 0) return fail(SKV_EINVAL, "kv_ring_restore: bad block range or ring");
    const BlockRuns r = block_runs(slots, host, fmt, s);
    for (int a = 0; a < r.n; ++a)
        if (!r.host[a] || !r.slot[a]) return fail(SKV_EINVAL, "kv_ring_restore: missing pool");
    for (int64_t b = b0; b < b1;) {
        const int64_t sl = b % n_slots, run = std::min<int64_t>(b1 - b, n_slots - sl);   // up to the ring's end
        for (int a = 0; a < r.n; ++a) {
            const cudaError_t e = cudaMemcpyAsync(r.slot[a] + sl * r.len[a], r.host[a] + b * r.len[a],
                                                  (size_t) (run * r.len[a]), cudaMemcpyDefault, stream);
            if (e != cudaSuccess) return cuda_fail(e, "kv_ring_restore");
        }
        b += run;
    }
    return SKV_OK;
}

int stage_from_host(const QsaAttnPools& stage, const KvHostPools& host, int fmt, int64_t n_blocks, const QsaShapes& s,
                    cudaStream_t stream) {
    if (n_blocks <= 0) return SKV_OK;
    const BlockRuns r = block_runs(stage, host, fmt, s);
    for (int a = 0; a < r.n; ++a) {
        if (!r.host[a] || !r.slot[a]) return fail(SKV_EINVAL, "kv_stage_from_host: missing pool");
        const cudaError_t e =
            cudaMemcpyAsync(r.slot[a], r.host[a], (size_t) (n_blocks * r.len[a]), cudaMemcpyDefault, stream);
        if (e != cudaSuccess) return cuda_fail(e, "kv_stage_from_host");
    }
    return SKV_OK;
}

int stream_resolve(const KvStreamMap& m, const QsaAttnPools& slots, const KvHostPools& host, int fmt,
                   const int32_t* ids, const int32_t* steps, int64_t n_q, int64_t cap, const QsaShapes& s,
                   cudaStream_t stream) {
    if (n_q <= 0) return SKV_OK;
    if (!m.page_table || !m.slot_block || !m.slot_stamp || !m.slot_ref || !m.ctl || !m.miss_block || !m.miss_slot ||
        m.n_slots <= 0 || m.n_slots > INT32_MAX / 4 || !ids || !steps || cap <= 0 || s.page_size <= 0)
        return fail(SKV_EINVAL, "kv_stream_resolve: incomplete map or selection");
    const BlockRuns r = block_runs(slots, host, fmt, s);
    for (int a = 0; a < r.n; ++a)
        if (r.len[a] % 16 || !r.host[a] || !r.slot[a])
            return fail(SKV_EINVAL, "kv_stream_resolve: every block run must be present and a multiple of 16 bytes");
    resolve_kernel<<<1, kResolveThreads, 0, stream>>>(m, ids, steps, (int) n_q, (int) cap, (int) s.page_size);
    if (const int rc = launched("kv_stream_resolve")) return rc;
    fill_kernel<<<96, 128, 0, stream>>>(m, r);
    return launched("kv_stream_resolve fill");
}

}  // namespace skv

namespace strata::kernels {

void kv_stream_reset(const KvStreamMap& m, void* stream) {
    skv::or_exit(skv::stream_reset(m, static_cast<cudaStream_t>(stream)));
}

void kv_stream_resolve(const KvStreamMap& m, const QsaAttnPools& slots, const KvHostPools& host, int fmt,
                       const int32_t* ids, const int32_t* steps, int64_t n_q, int64_t cap, const QsaShapes& s,
                       void* stream) {
    skv::or_exit(skv::stream_resolve(m, slots, host, fmt, ids, steps, n_q, cap, s, static_cast<cudaStream_t>(stream)));
}

void kv_ring_table(int32_t* page_table, int64_t n_blocks, int64_t n_slots, void* stream) {
    skv::or_exit(skv::ring_table(page_table, n_blocks, n_slots, static_cast<cudaStream_t>(stream)));
}

void kv_ring_restore(const QsaAttnPools& slots, const KvHostPools& host, int fmt, int64_t b0, int64_t b1,
                     int64_t n_slots, const QsaShapes& s, void* stream) {
    skv::or_exit(skv::ring_restore(slots, host, fmt, b0, b1, n_slots, s, static_cast<cudaStream_t>(stream)));
}

void kv_stage_from_host(const QsaAttnPools& stage, const KvHostPools& host, int fmt, int64_t n_blocks,
                        const QsaShapes& s, void* stream) {
    skv::or_exit(skv::stage_from_host(stage, host, fmt, n_blocks, s, static_cast<cudaStream_t>(stream)));
}

KvStreamCounters kv_stream_counters(const KvStreamMap& m) {
    int32_t c[kKvCtlInts] = {};
    KvStreamCounters r;
    if (!m.ctl || cudaMemcpy(c, m.ctl, sizeof c, cudaMemcpyDeviceToHost) != cudaSuccess) {
        (void) cudaGetLastError();
        return r;
    }
    uint64_t u[3];
    static_assert(sizeof u == 6 * sizeof(int32_t));
    std::memcpy(u, c + 4, sizeof u);
    r.misses = u[0];
    r.lookups = u[1];
    r.calls = u[2];
    r.overflow = c[3] != 0;
    return r;
}

uint64_t kv_block_bytes(const QsaShapes& s, int fmt) {
    const uint64_t rows = (uint64_t) (s.n_head_kv * s.page_size);
    if (fmt == kKvQ4) return 2 * rows * kv_q4_bytes_per_head((int) s.head_dim);
    if (fmt == kKvInt8) return 2 * rows * (uint64_t) s.head_dim + 2 * rows * (uint64_t) (s.head_dim / KV_Q8_GROUP) * 2;
    return 2 * rows * (uint64_t) s.head_dim * 2;
}

}  // namespace strata::kernels
