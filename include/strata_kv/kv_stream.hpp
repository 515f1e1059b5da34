// include/strata_kv/kv_stream.hpp - the block movers of streamed and ring-buffered QSA layers.
//
// The same functions, names and contracts as the reference's include/strata/kernels/kv_stream.hpp:62-96, written
// for sm_100a.  A streamed layer (kv_mode 1) keeps its AUTHORITATIVE K/V in pinned, device-mapped host memory in
// the identity layout, and VRAM holds `n_slots` pages of it; `page_table` is then a residency map (block -> slot,
// or -1).  A ring layer (kv_mode 2, the drafter) maps block b to slot b % n_slots statically.  A park saves the
// host copy; a mount writes the host copy back and then either evicts every block (mode 1: kv_stream_reset) or
// refills the ring from it (mode 2: kv_ring_restore).
//
// kv_stream_resolve (the decode-time CLOCK residency resolve) follows the reference's policy: hits take the call's
// epoch and their reference bit, every missing block is claimed once, victims come from a second-chance sweep from
// the hand that never takes a slot this call uses.  This build's miss list is in a deterministic order (query by
// query, ascending block), so a resolve is reproducible and checked against a sequential restatement.
#pragma once

#include "strata_kv/types.hpp"

#include <cstdint>

/// These are compiled into libstrata_kv.so with the CUDA sources (hidden by default there): export them.
#define STRATA_KV_STREAM_API __attribute__((visibility("default")))

namespace strata::kernels {

/// Every block evicted: page table all -1, slots free (block -1, stamp -1, reference bit 0), control words zero.
STRATA_KV_STREAM_API void kv_stream_reset(const KvStreamMap& m, void* stream);

/// Make every block named by the selections of `n_q` queries resident (ids [n_q][cap], ascending per query, width
/// from steps[q * kStepCount + kStepWidth]).  Capturable.  A call that cannot place every miss sets ctl[3].
STRATA_KV_STREAM_API void kv_stream_resolve(const KvStreamMap& m, const QsaAttnPools& slots, const KvHostPools& host, int fmt,
                       const int32_t* ids, const int32_t* steps, int64_t n_q, int64_t cap, const QsaShapes& s,
                       void* stream);

/// The static ring table `block -> block % n_slots`.
STRATA_KV_STREAM_API void kv_ring_table(int32_t* page_table, int64_t n_blocks, int64_t n_slots, void* stream);

/// Copy blocks [b0, b1) of the host copy into the ring slots b % n_slots.  Not capturable.
STRATA_KV_STREAM_API void kv_ring_restore(const QsaAttnPools& slots, const KvHostPools& host, int fmt, int64_t b0, int64_t b1,
                     int64_t n_slots, const QsaShapes& s, void* stream);

/// Copy the first `n_blocks` blocks of the host copy into an identity-layout resident pool.  Not capturable.
STRATA_KV_STREAM_API void kv_stage_from_host(const QsaAttnPools& stage, const KvHostPools& host, int fmt, int64_t n_blocks,
                        const QsaShapes& s, void* stream);

struct KvStreamCounters {
    uint64_t misses = 0, lookups = 0, calls = 0;
    bool overflow = false;
};
/// Synchronous read of the counters.
STRATA_KV_STREAM_API KvStreamCounters kv_stream_counters(const KvStreamMap& m);

/// Bytes of one block (page) of K and V together.
STRATA_KV_STREAM_API uint64_t kv_block_bytes(const QsaShapes& s, int fmt);

}  // namespace strata::kernels
