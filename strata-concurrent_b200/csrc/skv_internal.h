// skv_internal.h - shared declarations between the kernel file and the C-ABI glue of libstrata_kv.so.
#pragma once

#include "strata_kv.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace skv {

/// One segment as the kernels see it: the public skv_segment plus its tiling.
struct SegDev {
    const uint8_t* src;
    uint8_t* dst;
    const int32_t* src_pages;
    const int32_t* dst_pages;
    uint64_t bytes;
    uint64_t tile_bytes;      // bytes per tile (whole pages when either side is paged)
    uint32_t page_bytes;      // 0 when both sides are contiguous
    uint32_t pages_per_tile;  // 0 when both sides are contiguous
    int64_t src_page_limit;
    int64_t dst_page_limit;
};

/// The whole launch: passed by value as a __grid_constant__ kernel parameter (no device allocation, no
/// H2D copy, capturable in a CUDA graph).
struct CopyPlan {
    int n_segs;
    int tma_stages;                             // TMA engine: ring stages per CTA
    uint32_t* status;                           // the device status word (SKV_STATUS_* bits)
    uint32_t tma_tile;                          // TMA engine: bytes per ring stage
    uint32_t pad;
    uint64_t tile_end[SKV_COPY_MAX_SEGMENTS];   // inclusive prefix sum of tiles per segment
    SegDev seg[SKV_COPY_MAX_SEGMENTS];
};

/// TMA engine geometry: a ring of `tma_stages` tiles of `tma_tile` bytes in dynamic shared memory per CTA,
/// `tma_ctas_per_sm` CTAs per SM.  Runtime-tunable (skv_set_copy_tuning); these bound the accepted values.
constexpr uint32_t kTmaMinTileBytes = 4096;
constexpr uint32_t kTmaMaxTileBytes = 65536;
constexpr int kTmaMaxStages = 12;
constexpr uint32_t kSmemPerSm = 228 * 1024;    // B200: 228 KB of shared memory per SM, 227 KB per CTA
constexpr uint32_t kVecTileBytes = 32768;
constexpr int kVecThreads = 512;

/// Defaults measured on B200 (config 2a, 32K pool->pool): 3 CTAs/SM x 4 stages x 16 KiB reaches 98.6 % of the
/// measured copy peak; one CTA per SM is bound by the serial table-load latency of its single issuing warp.
struct Tuning {
    int tma_stages = 4;
    uint32_t tma_tile = 16384;
    int tma_ctas_per_sm = 3;
    int vec_ctas_per_sm = 4;
};
/// The process-wide copy-engine geometry in force.
Tuning tuning();
/// Dynamic shared memory one TMA CTA needs for `stages` x `tile`.
size_t tma_smem_bytes(int stages, uint32_t tile);

/// A copy launch gated by flags (skv_copy_gated).
struct GateArgs {
    const uint64_t* wait_flag = nullptr;   // every CTA waits for *wait_flag >= wait_value before its first load
    uint64_t wait_value = 0;
    uint64_t timeout_ns = 0;
    uint64_t* done_flag = nullptr;         // the last CTA to land stores done_value here (release, system scope)
    uint64_t done_value = 0;
    uint32_t* counters = nullptr;          // [0] CTAs reported, [1] CTAs that moved all their tiles; zero between launches
};

/// Per-device runtime facts the launchers need (SM count, the status word).
struct DeviceCtx {
    int device = -1;
    int sms = 0;
    uint32_t* status = nullptr;
    size_t tma_smem_configured = 0;   // the copy_tma_kernel dynamic-smem limit set on this device so far
    size_t tma_chain_smem_configured = 0;
    size_t tma_gated_smem_configured = 0;
    uint32_t* gate_counters = nullptr;   // skv_copy_gated's two counters (allocated zeroed on first use)
    uint32_t* chain_landed = nullptr; // skv_copy_chained scratch (kChainScratchBytes, allocated on first use)
};

/// skv_copy_chained scratch per device: landed-tile counters of up to SKV_COPY_MAX_SEGMENTS chunks, then the
/// 8-byte tile-claim counter.
constexpr size_t kChainScratchBytes = 4 * SKV_COPY_MAX_SEGMENTS + 8;

/// Chaining of one TMA launch (skv_copy_chained): segment c of the plan is chunk c.
struct ChainArgs {
    const uint64_t* wait_flags;   // chunk c is loaded only once wait_flags[c] >= value (null: no waits)
    uint64_t* signal_flags;       // chunk c landed: release store of value to signal_flags[c] (null: none)
    uint32_t* landed;             // per-chunk landed-tile counters, zeroed in stream order before the launch
    unsigned long long* next_tile;   // the tile-claim counter, zeroed with them
    uint64_t value;
    uint64_t timeout_ns;
};
/// Returns the context of the CURRENT device, creating it on first use.  Null on failure (error set).
DeviceCtx* current_ctx();

/// True when `address` lies inside a live block pool (skv_pool_create / skv_pool_wrap): such a resident layer is
/// addressed through its page table; any other resident layer is identity-addressed.
bool in_block_pool(const void* address);

/// Thread-local error message used by skv_last_error().
void set_error(const std::string& message);
int fail(int code, const std::string& message);
int cuda_fail(cudaError_t e, const char* what);

/// Launch one copy kernel for a prepared plan.  `engine` is SKV_COPY_TMA or SKV_COPY_VEC.
int launch_copy(const CopyPlan& plan, uint64_t total_tiles, int engine, DeviceCtx& ctx, cudaStream_t stream);
/// Launch the gated TMA kernel (skv_copy_gated).
int launch_copy_gated(const CopyPlan& plan, uint64_t total_tiles, const GateArgs& gate, DeviceCtx& ctx,
                      cudaStream_t stream);
/// Launch the chained TMA kernel (the counters are reset on `stream` first).
int launch_copy_chained(const CopyPlan& plan, uint64_t total_tiles, const ChainArgs& chain, DeviceCtx& ctx,
                        cudaStream_t stream);
/// A short byte range to write on the device: `bytes` from `src`, or zeros when `src` is null.  Both sides
/// device-addressable (this GPU's memory, a peer's through P2P or CUDA IPC, or mapped pinned host memory).
struct ByteRange {
    uint8_t* dst;
    const uint8_t* src;
    uint64_t bytes;
};
/// The largest range byte_ranges takes: it is for pads and small unaligned pieces, not bulk data.
constexpr uint64_t kByteRangeMaxBytes = 1u << 20;
/// Write every range on `stream` in one launch per 128 ranges (byte loads and stores): a payload's alignment pads
/// and the pieces too small or too unaligned for the bulk engines, instead of one copy-engine call each.
int byte_ranges(const std::vector<ByteRange>& ranges, cudaStream_t stream);
/// Enqueue the flag kernels.
int launch_signal(uint64_t* flag, uint64_t value, cudaStream_t stream);
int launch_wait(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, uint32_t* status, cudaStream_t stream);

}  // namespace skv
