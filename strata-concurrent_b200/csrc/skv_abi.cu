// skv_abi.cu - the extern "C" surface of libstrata_kv.so (declared in include/strata_kv.h).
//
// Host-side glue only: argument checks (refusals happen here, before anything is enqueued, the way the
// reference validates before its first write - include/strata/core/conversation_snapshot.hpp:103-108),
// the block pool and its allocator, plan building for the copy kernels in skv_copy.cu, pinned host
// memory, peer access / CUDA IPC and the completion flags.
#include "skv_internal.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

namespace skv {

namespace {
thread_local std::string t_error;
std::mutex g_tuning_mu;
Tuning g_tuning;
std::mutex g_ctx_mu;
std::vector<std::unique_ptr<DeviceCtx>> g_ctx;   // indexed by device ordinal

uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

/// Makes `device` the calling thread's current device for a scope and gives the caller's device back after it.
/// `error` is the failure of the switch (an ordinal that does not exist), with nothing switched.
struct DeviceScope {
    int prev = -1;
    cudaError_t error = cudaSuccess;
    explicit DeviceScope(int device) {
        error = cudaGetDevice(&prev);
        if (error != cudaSuccess) prev = -1;
        else if (prev != device) error = cudaSetDevice(device);
        if (error != cudaSuccess) (void) cudaGetLastError();
    }
    ~DeviceScope() {
        if (prev >= 0) (void) cudaSetDevice(prev);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
};

void set_error(const std::string& message) { t_error = message; }

Tuning tuning() {
    std::lock_guard<std::mutex> lock(g_tuning_mu);
    return g_tuning;
}

int fail(int code, const std::string& message) {
    t_error = message;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    t_error = std::string(what) + ": " + cudaGetErrorString(e);
    return SKV_ECUDA;
}

DeviceCtx* current_ctx() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cuda_fail(e, "cudaGetDevice");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    if ((size_t) dev >= g_ctx.size()) g_ctx.resize((size_t) dev + 1);
    if (g_ctx[(size_t) dev]) return g_ctx[(size_t) dev].get();
    auto ctx = std::make_unique<DeviceCtx>();
    ctx->device = dev;
    e = cudaDeviceGetAttribute(&ctx->sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
        cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
        return nullptr;
    }
    e = cudaMalloc(&ctx->status, 256);
    if (e == cudaSuccess) e = cudaMemset(ctx->status, 0, 256);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cuda_fail(e, "device status word");
        return nullptr;
    }
    g_ctx[(size_t) dev] = std::move(ctx);
    return g_ctx[(size_t) dev].get();
}

/// Validate the public segments and turn them into a kernel plan.  Zero-byte segments are dropped.
static int build_plan(const skv_segment* segs, int n_segs, int engine, CopyPlan& plan, uint64_t& total_tiles) {
    const Tuning tu = tuning();
    if (n_segs < 0 || n_segs > SKV_COPY_MAX_SEGMENTS || (n_segs && !segs))
        return fail(SKV_EINVAL, "skv_copy: segment count must be in [0, SKV_COPY_MAX_SEGMENTS]");
    if (engine != SKV_COPY_TMA && engine != SKV_COPY_VEC) return fail(SKV_EINVAL, "skv_copy: unknown copy engine");
    std::memset(&plan, 0, sizeof plan);
    plan.tma_stages = tu.tma_stages;
    plan.tma_tile = tu.tma_tile;
    total_tiles = 0;
    int k = 0;
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& s = segs[i];
        if (s.bytes == 0) continue;
        char where[96];
        std::snprintf(where, sizeof where, "skv_copy: segment %d: ", i);
        if (!s.src || !s.dst) return fail(SKV_EINVAL, std::string(where) + "missing buffer");
        if (!aligned16(s.src) || !aligned16(s.dst) || s.bytes % 16)
            return fail(SKV_EINVAL, std::string(where) + "buffers must be 16-byte aligned and bytes a multiple of 16");
        const bool paged = s.src_pages || s.dst_pages;
        SegDev d{};
        d.src = static_cast<const uint8_t*>(s.src);
        d.dst = static_cast<uint8_t*>(s.dst);
        d.src_pages = s.src_pages;
        d.dst_pages = s.dst_pages;
        d.bytes = s.bytes;
        d.src_page_limit = s.src_page_limit;
        d.dst_page_limit = s.dst_page_limit;
        if (paged) {
            if (s.page_bytes == 0 || s.page_bytes % 16 || s.bytes % s.page_bytes)
                return fail(SKV_EINVAL, std::string(where) + "a paged side needs page_bytes a multiple of 16 dividing bytes");
            if ((s.src_pages && s.src_page_limit <= 0) || (s.dst_pages && s.dst_page_limit <= 0))
                return fail(SKV_EINVAL, std::string(where) + "a paged side needs a positive page limit");
            d.page_bytes = s.page_bytes;
            if (engine == SKV_COPY_TMA) {
                if (s.page_bytes < 1024 || s.page_bytes > tu.tma_tile)
                    return fail(SKV_EINVAL, std::string(where) + "the TMA engine stages pages of 1 KiB up to its tile size");
                d.pages_per_tile = std::min<uint32_t>(32u, tu.tma_tile / s.page_bytes);
            } else {
                d.pages_per_tile = std::max<uint32_t>(1u, std::min<uint32_t>(512u, kVecTileBytes / s.page_bytes));
            }
            d.tile_bytes = (uint64_t) d.pages_per_tile * s.page_bytes;
        } else {
            d.tile_bytes = engine == SKV_COPY_TMA ? tu.tma_tile : kVecTileBytes;
        }
        total_tiles += (d.bytes + d.tile_bytes - 1) / d.tile_bytes;
        plan.seg[k] = d;
        plan.tile_end[k] = total_tiles;
        ++k;
    }
    plan.n_segs = k;
    return SKV_OK;
}

/// AUTO: the bulk engine when every buffer is this device's own memory and every page granule suits it.
static int pick_engine(const skv_segment* segs, int n_segs, int device) {
    const uint32_t tile = tuning().tma_tile;
    for (int i = 0; i < n_segs; ++i) {
        const skv_segment& s = segs[i];
        if (s.bytes == 0) continue;
        if ((s.src_pages || s.dst_pages) && (s.page_bytes < 1024 || s.page_bytes > tile)) return SKV_COPY_VEC;
        for (const void* p : {s.src, static_cast<const void*>(s.dst)}) {
            cudaPointerAttributes a{};
            if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
                (void) cudaGetLastError();
                return SKV_COPY_VEC;
            }
            if (a.type != cudaMemoryTypeDevice || a.device != device) return SKV_COPY_VEC;
        }
    }
    return SKV_COPY_TMA;
}

}  // namespace skv

using namespace skv;

// ====================================================================== extern "C"

struct skv_pool {
    int device = -1;
    bool owned = true;
    void* base = nullptr;
    uint64_t block_bytes = 0;
    int64_t n_blocks = 0;
    std::vector<int32_t> free_list;   // popped from the back
    std::vector<uint8_t> used;
    std::mutex mu;
};

namespace skv {
namespace {
std::mutex g_pools_mu;
std::vector<const skv_pool*> g_pools;   // every live pool, created or wrapped

void register_pool(const skv_pool* p) {
    std::lock_guard<std::mutex> lock(g_pools_mu);
    g_pools.push_back(p);
}
void unregister_pool(const skv_pool* p) {
    std::lock_guard<std::mutex> lock(g_pools_mu);
    g_pools.erase(std::remove(g_pools.begin(), g_pools.end(), p), g_pools.end());
}
}  // namespace

bool in_block_pool(const void* address) {
    const auto a = reinterpret_cast<uintptr_t>(address);
    std::lock_guard<std::mutex> lock(g_pools_mu);
    for (const skv_pool* p : g_pools) {
        const auto b = reinterpret_cast<uintptr_t>(p->base);
        if (a >= b && a - b < (uint64_t) p->n_blocks * p->block_bytes) return true;
    }
    return false;
}
}  // namespace skv

extern "C" {

const char* skv_last_error(void) { return t_error.c_str(); }

int skv_version(void) { return 1; }

int skv_pool_create(int device, int64_t n_blocks, uint64_t block_bytes, skv_pool** out) {
    if (!out) return fail(SKV_EINVAL, "skv_pool_create: null output");
    *out = nullptr;
    if (n_blocks <= 0 || n_blocks > INT32_MAX || block_bytes == 0 || block_bytes % 1024)
        return fail(SKV_EINVAL, "skv_pool_create: n_blocks in [1, 2^31) and block_bytes a positive multiple of 1 KiB");
    if ((uint64_t) n_blocks > UINT64_MAX / block_bytes) return fail(SKV_ERANGE, "skv_pool_create: pool size overflows");
    auto pool = std::make_unique<skv_pool>();
    pool->device = device;
    pool->block_bytes = block_bytes;
    pool->n_blocks = n_blocks;
    cudaError_t e;
    {
        DeviceScope on(device);
        if (on.error != cudaSuccess) return cuda_fail(on.error, "skv_pool_create: cudaSetDevice");
        e = cudaMalloc(&pool->base, (size_t) n_blocks * block_bytes);
    }
    if (e != cudaSuccess) {
        (void) cudaGetLastError();
        return fail(SKV_ENOMEM, std::string("skv_pool_create: cudaMalloc: ") + cudaGetErrorString(e));
    }
    pool->free_list.resize((size_t) n_blocks);
    for (int64_t i = 0; i < n_blocks; ++i) pool->free_list[(size_t) i] = (int32_t) (n_blocks - 1 - i);
    pool->used.assign((size_t) n_blocks, 0);
    register_pool(pool.get());
    *out = pool.release();
    return SKV_OK;
}

int skv_pool_wrap(int device, void* base, int64_t n_blocks, uint64_t block_bytes, skv_pool** out) {
    if (!out) return fail(SKV_EINVAL, "skv_pool_wrap: null output");
    *out = nullptr;
    if (!base || (reinterpret_cast<uintptr_t>(base) & 255u) || n_blocks <= 0 || n_blocks > INT32_MAX ||
        block_bytes == 0 || block_bytes % 1024)
        return fail(SKV_EINVAL, "skv_pool_wrap: a 256-byte aligned base, n_blocks in [1, 2^31), block_bytes a multiple of 1 KiB");
    auto pool = std::make_unique<skv_pool>();
    pool->device = device;
    pool->owned = false;
    pool->base = base;
    pool->block_bytes = block_bytes;
    pool->n_blocks = n_blocks;
    pool->free_list.resize((size_t) n_blocks);
    for (int64_t i = 0; i < n_blocks; ++i) pool->free_list[(size_t) i] = (int32_t) (n_blocks - 1 - i);
    pool->used.assign((size_t) n_blocks, 0);
    register_pool(pool.get());
    *out = pool.release();
    return SKV_OK;
}

int skv_pool_destroy(skv_pool* pool) {
    if (!pool) return SKV_OK;
    unregister_pool(pool);
    if (!pool->owned) {
        delete pool;
        return SKV_OK;
    }
    cudaError_t e;
    {
        DeviceScope on(pool->device);
        e = on.error != cudaSuccess ? on.error : cudaFree(pool->base);
    }
    delete pool;
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "skv_pool_destroy: cudaFree");
}

void* skv_pool_base(const skv_pool* pool) { return pool ? pool->base : nullptr; }
uint64_t skv_pool_block_bytes(const skv_pool* pool) { return pool ? pool->block_bytes : 0; }
int64_t skv_pool_blocks(const skv_pool* pool) { return pool ? pool->n_blocks : 0; }
int skv_pool_device(const skv_pool* pool) { return pool ? pool->device : -1; }

int skv_alloc_blocks(skv_pool* pool, int64_t n, int32_t* out_ids) {
    if (!pool || n < 0 || (n && !out_ids)) return fail(SKV_EINVAL, "skv_alloc_blocks: bad arguments");
    std::lock_guard<std::mutex> lock(pool->mu);
    if ((uint64_t) n > pool->free_list.size()) return fail(SKV_ENOMEM, "skv_alloc_blocks: the pool has too few free blocks");
    for (int64_t i = 0; i < n; ++i) {
        const int32_t id = pool->free_list.back();
        pool->free_list.pop_back();
        pool->used[(size_t) id] = 1;
        out_ids[i] = id;
    }
    return SKV_OK;
}

int skv_free_blocks(skv_pool* pool, const int32_t* ids, int64_t n) {
    if (!pool || n < 0 || (n && !ids)) return fail(SKV_EINVAL, "skv_free_blocks: bad arguments");
    std::lock_guard<std::mutex> lock(pool->mu);
    // validate all first: a double free or a foreign id frees nothing
    std::vector<uint8_t> seen;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t id = ids[i];
        if (id < 0 || id >= pool->n_blocks || !pool->used[(size_t) id])
            return fail(SKV_EINVAL, "skv_free_blocks: block " + std::to_string(id) + " is not allocated");
        if (seen.empty()) seen.assign((size_t) pool->n_blocks, 0);
        if (seen[(size_t) id]++) return fail(SKV_EINVAL, "skv_free_blocks: block " + std::to_string(id) + " listed twice");
    }
    for (int64_t i = 0; i < n; ++i) {
        pool->used[(size_t) ids[i]] = 0;
        pool->free_list.push_back(ids[i]);
    }
    return SKV_OK;
}

int64_t skv_pool_free_count(const skv_pool* pool) {
    if (!pool) return -1;
    std::lock_guard<std::mutex> lock(const_cast<skv_pool*>(pool)->mu);
    return (int64_t) pool->free_list.size();
}

int skv_pool_scramble(skv_pool* pool, uint64_t seed) {
    if (!pool) return fail(SKV_EINVAL, "skv_pool_scramble: null pool");
    std::lock_guard<std::mutex> lock(pool->mu);
    uint64_t state = splitmix64(seed ^ 0xBB67AE8584CAA73Bull);
    auto& f = pool->free_list;
    for (size_t i = f.size(); i > 1; --i) {
        state = splitmix64(state);
        std::swap(f[i - 1], f[(size_t) (state % i)]);
    }
    return SKV_OK;
}

int skv_expand_block_table(const int32_t* block_table, int64_t n_blocks, int64_t pages_per_block, int64_t slot_pages,
                           int64_t page_offset, int32_t* page_table) {
    if (n_blocks < 0 || pages_per_block <= 0 || slot_pages < pages_per_block || page_offset < 0 ||
        page_offset + pages_per_block > slot_pages || (n_blocks && (!block_table || !page_table)))
        return fail(SKV_EINVAL, "skv_expand_block_table: bad arguments");
    for (int64_t b = 0; b < n_blocks; ++b) {
        const int64_t base = (int64_t) block_table[b] * slot_pages + page_offset;
        if (block_table[b] < 0 || base + pages_per_block - 1 > INT32_MAX)
            return fail(SKV_ERANGE, "skv_expand_block_table: page index outside int32");
        for (int64_t j = 0; j < pages_per_block; ++j) page_table[b * pages_per_block + j] = (int32_t) (base + j);
    }
    return SKV_OK;
}

int skv_copy(const skv_segment* segs, int n_segs, int engine, void* stream) {
    DeviceCtx* ctx = current_ctx();
    if (!ctx) return SKV_ECUDA;
    if (engine == SKV_COPY_AUTO) engine = pick_engine(segs, n_segs, ctx->device);
    CopyPlan plan;
    uint64_t tiles = 0;
    if (const int rc = build_plan(segs, n_segs, engine, plan, tiles)) return rc;
    plan.status = ctx->status;
    return launch_copy(plan, tiles, engine, *ctx, static_cast<cudaStream_t>(stream));
}

int skv_copy_gated(const skv_segment* segs, int n_segs, const uint64_t* wait_flag, uint64_t wait_value,
                   uint64_t timeout_ns, uint64_t* done_flag, uint64_t done_value, void* stream) {
    if ((reinterpret_cast<uintptr_t>(wait_flag) | reinterpret_cast<uintptr_t>(done_flag)) & 7u)
        return fail(SKV_EINVAL, "skv_copy_gated: flags must be 8-byte aligned");
    if (timeout_ns > 60ull * 1000000000ull) return fail(SKV_EINVAL, "skv_copy_gated: timeout must be at most 60 s");
    DeviceCtx* ctx = current_ctx();
    if (!ctx) return SKV_ECUDA;
    CopyPlan plan;
    uint64_t tiles = 0;
    if (const int rc = build_plan(segs, n_segs, SKV_COPY_TMA, plan, tiles)) return rc;
    if (tiles == 0) return fail(SKV_EINVAL, "skv_copy_gated: nothing to move (use skv_wait_flag / skv_signal)");
    if (!ctx->gate_counters) {
        cudaError_t e = cudaMalloc(&ctx->gate_counters, 256);
        if (e == cudaSuccess) e = cudaMemset(ctx->gate_counters, 0, 256);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "skv_copy_gated: counters");
    }
    plan.status = ctx->status;
    GateArgs gate;
    gate.wait_flag = wait_flag;
    gate.wait_value = wait_value;
    gate.timeout_ns = timeout_ns ? timeout_ns : 2000000000ull;
    gate.done_flag = done_flag;
    gate.done_value = done_value;
    gate.counters = ctx->gate_counters;
    return launch_copy_gated(plan, tiles, gate, *ctx, static_cast<cudaStream_t>(stream));
}

int skv_copy_chained(const skv_segment* segs, int n_segs, const uint64_t* wait_flags, uint64_t* signal_flags,
                     uint64_t value, uint64_t timeout_ns, void* stream) {
    DeviceCtx* ctx = current_ctx();
    if (!ctx) return SKV_ECUDA;
    if (n_segs < 1 || n_segs > SKV_COPY_MAX_SEGMENTS || !segs)
        return fail(SKV_EINVAL, "skv_copy_chained: chunk count must be in [1, SKV_COPY_MAX_SEGMENTS]");
    for (int i = 0; i < n_segs; ++i)
        if (segs[i].bytes == 0) return fail(SKV_EINVAL, "skv_copy_chained: every chunk must move at least one byte");
    if ((reinterpret_cast<uintptr_t>(wait_flags) | reinterpret_cast<uintptr_t>(signal_flags)) & 7u)
        return fail(SKV_EINVAL, "skv_copy_chained: flags must be 8-byte aligned");
    if (timeout_ns > 60ull * 1000000000ull) return fail(SKV_EINVAL, "skv_copy_chained: timeout must be at most 60 s");
    CopyPlan plan;
    uint64_t tiles = 0;
    if (const int rc = build_plan(segs, n_segs, SKV_COPY_TMA, plan, tiles)) return rc;
    if (!ctx->chain_landed) {
        const cudaError_t e = cudaMalloc(&ctx->chain_landed, kChainScratchBytes);
        if (e != cudaSuccess) return cuda_fail(e, "skv_copy_chained: counters");
    }
    plan.status = ctx->status;
    auto* next_tile = reinterpret_cast<unsigned long long*>(ctx->chain_landed + SKV_COPY_MAX_SEGMENTS);
    ChainArgs chain{wait_flags, signal_flags, ctx->chain_landed, next_tile, value, timeout_ns ? timeout_ns : 2000000000ull};
    return launch_copy_chained(plan, tiles, chain, *ctx, static_cast<cudaStream_t>(stream));
}

int skv_set_copy_tuning(int tma_stages, uint32_t tma_tile_bytes, int tma_ctas_per_sm, int vec_ctas_per_sm) {
    if (tma_stages < 2 || tma_stages > kTmaMaxStages || tma_tile_bytes < kTmaMinTileBytes ||
        tma_tile_bytes > kTmaMaxTileBytes || tma_tile_bytes % 1024 || tma_ctas_per_sm < 1 || tma_ctas_per_sm > 8 ||
        vec_ctas_per_sm < 1 || vec_ctas_per_sm > 8)
        return fail(SKV_EINVAL, "skv_set_copy_tuning: stages in [2, 12], tile a multiple of 1 KiB in [4, 64] KiB, "
                                "CTAs per SM in [1, 8]");
    const size_t per_cta = tma_smem_bytes(tma_stages, tma_tile_bytes) + 1024;   // + the per-CTA reservation
    if (per_cta > 227 * 1024 || per_cta * (size_t) tma_ctas_per_sm > kSmemPerSm)
        return fail(SKV_ERANGE, "skv_set_copy_tuning: the TMA rings do not fit the SM's shared memory");
    std::lock_guard<std::mutex> lock(g_tuning_mu);
    g_tuning.tma_stages = tma_stages;
    g_tuning.tma_tile = tma_tile_bytes;
    g_tuning.tma_ctas_per_sm = tma_ctas_per_sm;
    g_tuning.vec_ctas_per_sm = vec_ctas_per_sm;
    return SKV_OK;
}

int skv_get_copy_tuning(int* tma_stages, uint32_t* tma_tile_bytes, int* tma_ctas_per_sm, int* vec_ctas_per_sm) {
    const Tuning t = tuning();
    if (tma_stages) *tma_stages = t.tma_stages;
    if (tma_tile_bytes) *tma_tile_bytes = t.tma_tile;
    if (tma_ctas_per_sm) *tma_ctas_per_sm = t.tma_ctas_per_sm;
    if (vec_ctas_per_sm) *vec_ctas_per_sm = t.vec_ctas_per_sm;
    return SKV_OK;
}

int skv_device_initialized(int device) {
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    return device >= 0 && (size_t) device < g_ctx.size() && g_ctx[(size_t) device] ? 1 : 0;
}

int skv_query_status(int device, void* stream, uint32_t* out_status) {
    if (!out_status) return fail(SKV_EINVAL, "skv_query_status: null output");
    DeviceScope on(device);
    if (on.error != cudaSuccess) return cuda_fail(on.error, "skv_query_status: cudaSetDevice");
    DeviceCtx* ctx = current_ctx();
    int rc = SKV_OK;
    if (!ctx) rc = SKV_ECUDA;
    else {
        cudaError_t e = cudaMemcpyAsync(out_status, ctx->status, 4, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
        if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) rc = cuda_fail(e, "skv_query_status");
    }
    return rc;
}

int skv_clear_status(int device, void* stream) {
    DeviceScope on(device);
    if (on.error != cudaSuccess) return cuda_fail(on.error, "skv_clear_status: cudaSetDevice");
    DeviceCtx* ctx = current_ctx();
    int rc = SKV_OK;
    if (!ctx) rc = SKV_ECUDA;
    else {
        const cudaError_t e = cudaMemsetAsync(ctx->status, 0, 4, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) rc = cuda_fail(e, "skv_clear_status");
    }
    return rc;
}

int skv_host_alloc(uint64_t bytes, void** out) {
    if (!out) return fail(SKV_EINVAL, "skv_host_alloc: null output");
    *out = nullptr;
    if (bytes == 0) return SKV_OK;
    const cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocPortable | cudaHostAllocMapped);
    if (e != cudaSuccess) {
        (void) cudaGetLastError();
        return fail(SKV_ENOMEM, std::string("skv_host_alloc: ") + cudaGetErrorString(e));
    }
    return SKV_OK;
}

int skv_host_free(void* p) {
    if (!p) return SKV_OK;
    const cudaError_t e = cudaFreeHost(p);
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "skv_host_free");
}

int skv_host_register(void* p, uint64_t bytes) {
    if (!p || !bytes) return fail(SKV_EINVAL, "skv_host_register: bad arguments");
    cudaError_t e = cudaHostRegister(p, (size_t) bytes, cudaHostRegisterPortable | cudaHostRegisterMapped);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostRegister");
    // kernels (flags, direct copies) use the host address itself: the device must map it at the same address
    void* dev = nullptr;
    e = cudaHostGetDevicePointer(&dev, p, 0);
    if (e != cudaSuccess || dev != p) {
        (void) cudaGetLastError();
        cudaHostUnregister(p);
        return fail(SKV_EINVAL, "skv_host_register: this device does not map registered memory at its host address");
    }
    return SKV_OK;
}

int skv_host_unregister(void* p) {
    if (!p) return SKV_OK;
    const cudaError_t e = cudaHostUnregister(p);
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "cudaHostUnregister");
}

/// STAGED transfers: the staging layout is the segments' bytes back to back, each 256-byte aligned.
static int staged_offsets(const skv_segment* segs, int n, uint64_t staging_bytes, std::vector<uint64_t>& off) {
    off.assign((size_t) n, 0);
    uint64_t at = 0;
    for (int i = 0; i < n; ++i) {
        off[(size_t) i] = at;
        at += (segs[i].bytes + 255) & ~255ull;
    }
    if (at > staging_bytes) return fail(SKV_ERANGE, "skv_park/resume: staging buffer smaller than the segments");
    return SKV_OK;
}

int skv_park(const skv_segment* segs, int n_segs, int mode, void* staging, uint64_t staging_bytes, void* stream) {
    if (mode == SKV_PARK_DIRECT) return skv_copy(segs, n_segs, SKV_COPY_VEC, stream);
    if (mode != SKV_PARK_STAGED) return fail(SKV_EINVAL, "skv_park: unknown mode");
    if (n_segs < 0 || n_segs > SKV_COPY_MAX_SEGMENTS || (n_segs && !segs) || !staging)
        return fail(SKV_EINVAL, "skv_park: bad arguments");
    std::vector<uint64_t> off;
    if (const int rc = staged_offsets(segs, n_segs, staging_bytes, off)) return rc;
    std::vector<skv_segment> gather(segs, segs + n_segs);
    for (int i = 0; i < n_segs; ++i) {
        if (segs[i].dst_pages) return fail(SKV_EINVAL, "skv_park: a staged park needs contiguous host destinations");
        gather[(size_t) i].dst = static_cast<uint8_t*>(staging) + off[(size_t) i];
        gather[(size_t) i].dst_pages = nullptr;
    }
    if (const int rc = skv_copy(gather.data(), n_segs, SKV_COPY_AUTO, stream)) return rc;
    for (int i = 0; i < n_segs; ++i) {
        if (!segs[i].bytes) continue;
        const cudaError_t e = cudaMemcpyAsync(segs[i].dst, static_cast<uint8_t*>(staging) + off[(size_t) i], segs[i].bytes,
                                              cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "skv_park: cudaMemcpyAsync");
    }
    return SKV_OK;
}

int skv_resume(const skv_segment* segs, int n_segs, int mode, void* staging, uint64_t staging_bytes, void* stream) {
    if (mode == SKV_PARK_DIRECT) return skv_copy(segs, n_segs, SKV_COPY_VEC, stream);
    if (mode != SKV_PARK_STAGED) return fail(SKV_EINVAL, "skv_resume: unknown mode");
    if (n_segs < 0 || n_segs > SKV_COPY_MAX_SEGMENTS || (n_segs && !segs) || !staging)
        return fail(SKV_EINVAL, "skv_resume: bad arguments");
    std::vector<uint64_t> off;
    if (const int rc = staged_offsets(segs, n_segs, staging_bytes, off)) return rc;
    std::vector<skv_segment> scatter(segs, segs + n_segs);
    for (int i = 0; i < n_segs; ++i) {
        if (segs[i].src_pages) return fail(SKV_EINVAL, "skv_resume: a staged resume needs contiguous host sources");
        if (!segs[i].bytes) continue;
        const cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(staging) + off[(size_t) i], segs[i].src, segs[i].bytes,
                                              cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "skv_resume: cudaMemcpyAsync");
        scatter[(size_t) i].src = static_cast<uint8_t*>(staging) + off[(size_t) i];
    }
    return skv_copy(scatter.data(), n_segs, SKV_COPY_AUTO, stream);
}

int skv_enable_peer(int device, int peer) {
    if (device == peer) return SKV_OK;
    int can = 0;
    cudaError_t e = cudaDeviceCanAccessPeer(&can, device, peer);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
    if (!can) return fail(SKV_EINVAL, "skv_enable_peer: the devices cannot access each other");
    {
        DeviceScope on(device);
        e = on.error != cudaSuccess ? on.error : cudaDeviceEnablePeerAccess(peer, 0);
    }
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        (void) cudaGetLastError();
        return SKV_OK;
    }
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "cudaDeviceEnablePeerAccess");
}

int skv_ipc_export(void* dev_ptr, uint8_t handle[64]) {
    if (!dev_ptr || !handle) return fail(SKV_EINVAL, "skv_ipc_export: bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle, &h, 64);
    return SKV_OK;
}

int skv_ipc_import(int device, const uint8_t handle[64], void** out_ptr) {
    if (!handle || !out_ptr) return fail(SKV_EINVAL, "skv_ipc_import: bad arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, 64);
    *out_ptr = nullptr;
    DeviceScope on(device);
    if (on.error != cudaSuccess) return cuda_fail(on.error, "skv_ipc_import: cudaSetDevice");
    const cudaError_t e = cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int skv_ipc_close(void* ptr) {
    if (!ptr) return SKV_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? SKV_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int skv_signal(uint64_t* flag, uint64_t value, void* stream) {
    if (!flag || (reinterpret_cast<uintptr_t>(flag) & 7u))
        return fail(SKV_EINVAL, "skv_signal: the flag must be an 8-byte aligned device address");
    return launch_signal(flag, value, static_cast<cudaStream_t>(stream));
}

int skv_wait_flag(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, void* stream) {
    if (!flag || (reinterpret_cast<uintptr_t>(flag) & 7u))
        return fail(SKV_EINVAL, "skv_wait_flag: the flag must be an 8-byte aligned device address");
    if (timeout_ns == 0 || timeout_ns > 60ull * 1000000000ull)
        return fail(SKV_EINVAL, "skv_wait_flag: timeout must be in (0, 60 s]");
    DeviceCtx* ctx = current_ctx();
    if (!ctx) return SKV_ECUDA;
    return launch_wait(flag, value, timeout_ns, ctx->status, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
