/* include/strata_kv.h - the C ABI of the B200 KV handoff / park-resume path.
 *
 * Plain pointers, sizes and integer status codes; no exceptions, no torch types.  Everything the
 * reference's path does with cudaMemcpy (src/core/conversation_snapshot.cpp:105-113, 139-219;
 * src/core/conversation_state.cpp:33-40, 228-267) and with its block movers
 * (src/kernels/cuda/kv_stream.cu:160-252) goes through the entry points below.  The C++ drop-in layer
 * (the headers under include/strata_kv/, same names and signatures as the reference's conversation_* API) is built on
 * them, and so are the Python bindings used by the tests and bench.py.
 *
 * Conventions
 *   - Every function returns SKV_OK (0) or a positive SKV_E* code; skv_last_error() gives the message of
 *     the most recent failure on the calling thread.
 *   - Device pointers are plain CUDA device (or peer, or mapped-pinned-host) addresses.  `stream` is a
 *     cudaStream_t passed as void* (NULL = the legacy default stream).
 *   - Asynchronous entry points only enqueue work; a device-side problem (a table entry outside its pool,
 *     a bounded wait that ran out) is recorded in the device's status word and read by skv_query_status().
 */
#ifndef STRATA_KV_H
#define STRATA_KV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SKV_API __attribute__((visibility("default")))
#else
#define SKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
#define SKV_OK 0
#define SKV_EINVAL 1     /* an argument the reference would also refuse (bad extent, null buffer, ...) */
#define SKV_ECUDA 2      /* a CUDA runtime call failed */
#define SKV_ENOMEM 3     /* the pool (or host arena) has no room */
#define SKV_ETIMEOUT 4   /* a bounded device-side wait ran out */
#define SKV_EDEVICE 5    /* the device status word reports a refused access */
#define SKV_ERANGE 6     /* a size beyond a documented maximum */

/* device status word bits (skv_query_status) */
#define SKV_STATUS_BAD_SRC_PAGE 0x1u   /* a source table entry was outside [0, src_page_limit): page skipped */
#define SKV_STATUS_BAD_DST_PAGE 0x2u   /* a destination table entry was outside [0, dst_page_limit): page skipped */
#define SKV_STATUS_WAIT_TIMEOUT 0x4u   /* a bounded wait (mbarrier or peer flag) gave up */

/* Message of the calling thread's most recent failure ("" if none).  Reference: the named
 * `std::string& error` every conversation_* function fills (include/strata/core/conversation_snapshot.hpp:13-48). */
SKV_API const char* skv_last_error(void);
/* Library version, for the binding's load check. */
SKV_API int skv_version(void);

/* ------------------------------------------------------------------ the KV block pool and its allocator
 * A pool is one device allocation of n_blocks fixed-size slots.  One slot holds one 256-token block of ONE
 * layer: its K pages followed by its V pages, each page in the reference layout
 * [kv_head][page_size=4][head_dim] (include/strata/kernels/qsa.hpp:178).  The reference has no block
 * allocator: its QsaState pools are carved once by qsa_state_init (src/core/layer.cpp:547-678) with an
 * identity page_table (layer.cpp:666-671); this allocator is what makes the table non-identity. */
typedef struct skv_pool skv_pool;

SKV_API int skv_pool_create(int device, int64_t n_blocks, uint64_t block_bytes, skv_pool** out);
/* The same allocator over caller-owned device memory (base 256-byte aligned, n_blocks*block_bytes long);
 * destroying such a pool frees only the bookkeeping. */
SKV_API int skv_pool_wrap(int device, void* base, int64_t n_blocks, uint64_t block_bytes, skv_pool** out);
SKV_API int skv_pool_destroy(skv_pool* pool);
/* Device base address, slot size, slot count, device ordinal. */
SKV_API void* skv_pool_base(const skv_pool* pool);
SKV_API uint64_t skv_pool_block_bytes(const skv_pool* pool);
SKV_API int64_t skv_pool_blocks(const skv_pool* pool);
SKV_API int skv_pool_device(const skv_pool* pool);
/* All-or-nothing: n distinct free slots, or SKV_ENOMEM and nothing taken.  Slots come out in a
 * seed-dependent order when the pool was scrambled by skv_pool_scramble (tests and bench use this to get
 * the seed-random placements the configs name); otherwise lowest-first. */
SKV_API int skv_alloc_blocks(skv_pool* pool, int64_t n, int32_t* out_ids);
/* Returns slots to the pool.  A slot that is not currently allocated is refused (SKV_EINVAL) and nothing
 * is freed. */
SKV_API int skv_free_blocks(skv_pool* pool, const int32_t* ids, int64_t n);
SKV_API int64_t skv_pool_free_count(const skv_pool* pool);
/* Reorder the free list by a seed-random permutation (splitmix64-driven Fisher-Yates). */
SKV_API int skv_pool_scramble(skv_pool* pool, uint64_t seed);

/* Expand a block table into the reference's per-page table format (QsaState::page_table,
 * include/strata/core/layer.hpp:220): page_table[b*pages_per_block + j] = block_table[b]*slot_pages +
 * page_offset + j.  With K and V in one slot, K uses page_offset 0 and V uses pages_per_block.  Host only. */
SKV_API int skv_expand_block_table(const int32_t* block_table, int64_t n_blocks, int64_t pages_per_block,
                           int64_t slot_pages, int64_t page_offset, int32_t* page_table);

/* ------------------------------------------------------------------ copy plans: gather / scatter / pool->pool
 * One segment moves `bytes` logical bytes.  Each side is either contiguous (its page table is NULL) or
 * paged: logical page p lives at base + pages[p]*page_bytes, the address rule of the reference's readers
 * and writers (kv_gather/kv_append, src/kernels/cuda/qsa.cu:121-142, 405-423).  Page tables are device
 * int32 arrays.  A table entry outside [0, *_page_limit) is not dereferenced: that page is skipped and
 * SKV_STATUS_BAD_*_PAGE is set.
 *
 * Alignment: base addresses 16-byte aligned; page_bytes and bytes multiples of 16; a paged side needs
 * bytes to be a multiple of page_bytes. */
typedef struct skv_segment {
    const void* src;
    void* dst;
    const int32_t* src_pages;   /* NULL: contiguous source */
    const int32_t* dst_pages;   /* NULL: contiguous destination */
    uint64_t bytes;
    uint32_t page_bytes;        /* granule of both tables; ignored when both sides are contiguous */
    uint32_t reserved;
    int64_t src_page_limit;     /* pages addressable from src (paged side only) */
    int64_t dst_page_limit;     /* pages addressable from dst (paged side only) */
} skv_segment;

/* copy engines */
#define SKV_COPY_AUTO 0   /* TMA bulk staging for device-local destinations, vector stores otherwise */
#define SKV_COPY_TMA 1    /* cp.async.bulk global->shared->global, mbarrier-tracked ring, 1 CTA per SM */
#define SKV_COPY_VEC 2    /* 16-byte vector loads and stores, many in flight per thread */
#define SKV_COPY_MAX_SEGMENTS 64

/* Enqueue ONE kernel launch that performs every segment.  The gather/pack of conversation_kv_save
 * (conversation_snapshot.cpp:139-173), the scatter/unpack of conversation_kv_restore (:196-219), the
 * running-state rows of conversation_checkpoint_save/restore (conversation_state.cpp:228-267) and the
 * block copy of kv_stream.cu's copy kernel (kv_stream.cu:160-171) are all instances.  Destinations may be
 * device, peer (P2P over NVLink) or mapped pinned host memory.  n_segs <= SKV_COPY_MAX_SEGMENTS. */
SKV_API int skv_copy(const skv_segment* segs, int n_segs, int engine, void* stream);

/* skv_copy_gated - skv_copy on the TMA engine with a hand-off's two flags inside the one launch: every CTA
 * waits until *wait_flag >= wait_value (acquire at system scope, bounded by timeout_ns of device time, 0 = 2 s)
 * before its first load, and once every CTA has landed all of its tiles the last one stores done_value to
 * *done_flag with release semantics at system scope, so a GPU or host thread that acquires done_flag reads every
 * byte.  A wait that runs out sets SKV_STATUS_WAIT_TIMEOUT, that CTA moves nothing and done_flag is not raised.
 * Either flag may be null; flags are 8-byte aligned device or mapped host words; at least one byte must move.
 * Replaces skv_wait_flag + skv_copy + skv_signal of a P2P pull (two launches and a flag round trip fewer).  The
 * gated copies of one device share two counters: issue them from one stream, one after another.  No counterpart in
 * the reference (it has no P2P path). */
SKV_API int skv_copy_gated(const skv_segment* segs, int n_segs, const uint64_t* wait_flag, uint64_t wait_value,
                           uint64_t timeout_ns, uint64_t* done_flag, uint64_t done_value, void* stream);

/* skv_copy_noalloc - the same copy for callers that cannot allocate device memory.
 * No counterpart in the reference (its park path only has synchronous cudaMemcpy calls).
 *
 * Who needs it: an engine whose token path must not allocate (the reference's session requires zero
 * token-path allocations, and a park or mount happens between tokens of a running server), a caller
 * that has given every free byte of HBM to its block pool, and any caller that cannot afford the implicit
 * device-wide synchronisation a first cudaMalloc can cause while other streams are decoding.  skv_copy
 * allocates a small status word on a device's first use; this entry point never calls an allocator and never
 * creates that per-device state (skv_device_initialized stays 0 if nothing else ran).
 *
 * It moves the segments with the vector engine in one copy launch (the vec_ctas_per_sm of
 * skv_set_copy_tuning), up to SKV_NOALLOC_MAX_SEGMENTS segments per call (skv_copy takes 64).  Its plan and
 * status word live in one fixed-size device array of the library (about 41 KB per GPU, held until the process
 * exits).  More segments than the maximum is refused with SKV_ERANGE before anything is enqueued.
 *   status_out  optional; receives the call's SKV_STATUS_* bits (device or mapped pinned host memory),
 *               written in stream order after the copy.
 * The first call on a device does a one-time set-up: it looks up the array's device address and the SM count.
 * Under CUDA's lazy module loading that lookup may load the library's module onto the device (its code and the
 * array) and can synchronise the device.  So make one warm-up call per device at initialisation, before the
 * token path starts and before any stream capture.
 * Calls share the array.  Calls on one stream from ONE host thread at a time are ordered and safe.  Two host
 * threads issuing calls on the same stream can interleave their plan-writer and copy launches (call A's copy
 * may then run on call B's plan), and calls that overlap on the GPU (other streams of the same device) race on
 * the plan and the status word. */
#define SKV_NOALLOC_MAX_SEGMENTS 512
SKV_API int skv_copy_noalloc(const skv_segment* segs, int n_segs, uint32_t* status_out, void* stream);

/* Copy-engine geometry, process-wide.  The TMA engine runs tma_ctas_per_sm CTAs per SM, each with a ring of
 * tma_stages x tma_tile_bytes of shared memory (the rings must fit the SM's 228 KB together); the vector
 * engine runs vec_ctas_per_sm CTAs of 512 threads per SM.  Defaults are the values measured best on B200. */
SKV_API int skv_set_copy_tuning(int tma_stages, uint32_t tma_tile_bytes, int tma_ctas_per_sm, int vec_ctas_per_sm);
SKV_API int skv_get_copy_tuning(int* tma_stages, uint32_t* tma_tile_bytes, int* tma_ctas_per_sm, int* vec_ctas_per_sm);

/* The device status word of `device` (OR of SKV_STATUS_* since the last clear); synchronises `stream`. */
SKV_API int skv_query_status(int device, void* stream, uint32_t* out_status);
/* 1 when the library has set up its per-device state on `device` (the SM count and the status word that
 * skv_copy, skv_query_status and the park / resume calls create on a device's first use), else 0.  A read only:
 * it sets nothing up.  No counterpart in the reference. */
SKV_API int skv_device_initialized(int device);
SKV_API int skv_clear_status(int device, void* stream);

/* ------------------------------------------------------------------ pinned host arena (park / resume)
 * Page-locked, device-mapped, portable host memory.  The reference parks into pageable std::vector
 * segments (include/strata/core/conversation_buffer.hpp:16-152); a pinned image is what lets the copy
 * run asynchronously on a side stream at PCIe speed. */
SKV_API int skv_host_alloc(uint64_t bytes, void** out);
SKV_API int skv_host_free(void* p);
/* Page-lock and device-map memory the caller already owns (no reference counterpart): e.g. a shared-memory
 * mapping two processes on one node both register, so one GPU parks into it and another resumes from it. */
SKV_API int skv_host_register(void* p, uint64_t bytes);
SKV_API int skv_host_unregister(void* p);

/* Park: move the segments (paged device sources) into pinned host memory.  mode SKV_PARK_DIRECT writes
 * the host image from the kernel through the mapping; SKV_PARK_STAGED gathers into `staging` (device, at
 * least the sum of segment bytes) and then issues one cudaMemcpyAsync per segment on `stream`.
 * Resume is the same call with host sources and paged device destinations (staged: H2D copies into
 * `staging`, then the scatter kernel). */
#define SKV_PARK_DIRECT 1
#define SKV_PARK_STAGED 2
SKV_API int skv_park(const skv_segment* segs, int n_segs, int mode, void* staging, uint64_t staging_bytes, void* stream);
SKV_API int skv_resume(const skv_segment* segs, int n_segs, int mode, void* staging, uint64_t staging_bytes, void* stream);

/* Chained copy (no reference counterpart: the pipelined relay of a one-to-many handoff).  Like skv_copy with
 * the TMA engine, but segment c is chunk c of a pipeline: no byte of chunk c is read before
 * wait_flags[c] >= value (this device's memory; bounded by timeout_ns of device time, 0 = 2 s, at most 60 s),
 * and once every byte of chunk c has landed, value is stored to signal_flags[c] (any device's memory, e.g. the
 * next GPU's flags through CUDA IPC) with system-scope release semantics - while later chunks are still
 * moving.  A destination may be a peer's memory too (the pushed form of a chain).  Either
 * flag array may be NULL.  Every chunk must be non-empty.  A wait that runs out sets SKV_STATUS_WAIT_TIMEOUT,
 * stops new reads, and leaves the unfinished chunks unsignalled.  One chained copy in flight per device (the
 * per-chunk counters are per device). */
SKV_API int skv_copy_chained(const skv_segment* segs, int n_segs, const uint64_t* wait_flags, uint64_t* signal_flags,
                             uint64_t value, uint64_t timeout_ns, void* stream);

/* ------------------------------------------------------------------ peer-to-peer handoff
 * The reference has no P2P path at all (its multi-GPU split stages through pinned RAM, docs/MULTI_GPU.md:9-12).
 * skv_copy with destinations in a peer's pool is the P2P scatter; these make the peer reachable and give
 * the handoff a completion signal. */
/* Enable peer access from the current device to `peer` (idempotent). */
SKV_API int skv_enable_peer(int device, int peer);
/* Export / import a device allocation across processes (CUDA IPC).  handle is 64 bytes. */
SKV_API int skv_ipc_export(void* dev_ptr, uint8_t handle[64]);
SKV_API int skv_ipc_import(int device, const uint8_t handle[64], void** out_ptr);
SKV_API int skv_ipc_close(void* ptr);
/* After the copies already on `stream`: a system-scope release store of `value` to the 8-byte flag
 * (peer or local device memory). */
SKV_API int skv_signal(uint64_t* flag, uint64_t value, void* stream);
/* On `stream`: wait until the local 8-byte flag is >= value, for at most timeout_ns of device time.  On
 * timeout the wait ends and SKV_STATUS_WAIT_TIMEOUT is set (never a trap, never an endless loop). */
SKV_API int skv_wait_flag(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, void* stream);

/* ------------------------------------------------------------------ many-to-many hand-off order
 * No reference counterpart (its split roles move one conversation at a time through pinned RAM).  When several
 * destination GPUs pull from several source GPUs at once, two destinations reading one source split its NVLink
 * egress while another port idles.  skv_schedule_phases orders such a batch in port-exclusive phases: in each
 * phase every source feeds at most one destination, and with equal port rates the batch ends when the busiest
 * port (a row or column sum of `demand`) has carried its bytes - the bound for any order.
 *
 * demand: n_src x n_dst bytes, row-major (source s, destination d); 1 <= n_src, n_dst <= 64.  Destination d's
 * runs are written at runs + d * max_runs, in the order to issue them, and their count to n_runs[d]; a
 * destination's flag index is its run index.  max_runs >= n * n with n = max(n_src, n_dst) always suffices;
 * fewer is refused with SKV_ERANGE if a destination needs more.  *bound_bytes = the busiest port's bytes,
 * *n_phases = the number of phases.  Host-only: no device is touched. */
typedef struct skv_sched_run {
    int32_t phase;       /* phase index */
    int32_t src;         /* the source it reads (row of demand) */
    uint64_t lo, hi;     /* bytes [lo, hi) of the flow src -> this destination */
    int32_t wait;        /* before the run: wait for this destination's flag `wait` (-1: none) */
    int32_t signal_dst;  /* after the run: release flag signal_idx of destination signal_dst (-1: none) */
    int32_t signal_idx;
    int32_t reserved;
} skv_sched_run;
SKV_API int skv_schedule_phases(const uint64_t* demand, int n_src, int n_dst, skv_sched_run* runs, int max_runs,
                                int* n_runs, uint64_t* bound_bytes, int* n_phases);
/* Bytes [lo, hi) of a segment list taken as one stream, as segments (a run's share of its flow).  A cut inside a
 * segment falls on that segment's granule, rounded down: a whole page when a side is paged, 16 bytes otherwise.
 * So adjacent ranges [a, b) and [b, c) tile the stream exactly.  Writes at most out_cap segments to `out` and their
 * count to *n_out; SKV_ERANGE if more are needed.  Host-only. */
SKV_API int skv_slice_segments(const skv_segment* segs, int n_segs, uint64_t lo, uint64_t hi, skv_segment* out,
                               int out_cap, int* n_out);

#ifdef __cplusplus
}
#endif
#endif
