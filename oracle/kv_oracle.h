/* oracle/kv_oracle.h - TEST INFRASTRUCTURE: the CPU restatement of the reference's KV handoff / park path.
 *
 * This is the checker the CUDA path is compared against.  It is never the product: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load liboracle.so.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the reference's own code
 * (oracle/_ref/libstrata_ref.so, built from the reference sources by oracle/Makefile) and against the
 * golden fixtures in tests/golden/ that the reference produced.
 */
#ifndef STRATA_KV_ORACLE_H
#define STRATA_KV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (counter-based, so any element can be regenerated independently) ---- */
/* out[i] = fp16(N(0,1)) for element (offset + i) of stream `seed`: splitmix64 -> two 53-bit uniforms ->
 * Box-Muller (the cosine branch) -> fp32 -> fp16 with round-to-nearest-even. */
void orc_fill_f16_normal(uint16_t* out, uint64_t n, uint64_t seed, uint64_t offset);
/* out[i] = sigma * N(0,1) as fp32, same element rule. */
void orc_fill_f32_normal(float* out, uint64_t n, uint64_t seed, uint64_t offset, float sigma);
/* out[i] uniform in [0, vocab). */
void orc_fill_ids(int32_t* out, uint64_t n, uint64_t seed, int32_t vocab);
/* A seed-random permutation of [0, n) (Fisher-Yates driven by splitmix64). */
void orc_permutation(int32_t* out, int64_t n, uint64_t seed);
/* fp32 -> fp16 bits, round to nearest even (IEEE 754 binary16, subnormals and inf/nan handled). */
uint16_t orc_f32_to_f16(float x);

/* ---- the block table (include/strata/core/layer.hpp:220, src/kernels/cuda/qsa.cu:121-142, 405-423) ----
 * A 256-token block is 64 consecutive reference pages of 4 cells.  A block table entry names a pool slot;
 * the reference's per-page table is page_table[b*pages_per_block + j] = slot*slot_pages + j. */
void orc_expand_block_table(const int32_t* block_table, int64_t n_blocks, int64_t pages_per_block,
                            int64_t slot_pages, int64_t page_offset, int32_t* page_table);
/* out[p*page_bytes ...] = pool[page_table[p]*page_bytes ...] for p < n_pages: the reference's reader rule
 * row = (table[pos/ps]*H + h)*ps + pos%ps applied to whole pages (qsa.hpp:63-70). */
void orc_gather_pages(const uint8_t* pool, const int32_t* page_table, int64_t n_pages, uint64_t page_bytes,
                      uint8_t* out);
/* pool[page_table[p]*page_bytes ...] = in[p*page_bytes ...]: the writer rule (kv_append, qsa.cu:121-142). */
void orc_scatter_pages(const uint8_t* in, const int32_t* page_table, int64_t n_pages, uint64_t page_bytes,
                       uint8_t* pool);

/* ---- snapshot byte extents (src/core/conversation_snapshot.cpp:27-67, conversation_state.cpp:180-205) ---- */
typedef struct OrcKvLayout {
    int32_t format;       /* 0 fp16, 1 int8, 2 q4_0, 3 hybrid K8V4 */
    int64_t cells;        /* upto rounded up to the 4-cell page */
    int64_t pooled_rows;  /* indexer rows incl. the moving spare row; 0 without an indexer */
    uint64_t data, scales, pooled, value_data, value_scales;  /* bytes of k, k_scale, pooled, v, v_scale */
} OrcKvLayout;
/* Returns 0, or -1 for a geometry/extent the reference refuses. */
int orc_kv_layout(int32_t format, int64_t upto, int include_index, int64_t n_head_kv, int64_t head_dim,
                  int64_t idx_key_dim, OrcKvLayout* out);

typedef struct OrcStateSizes {
    uint64_t gdn, ple, tail, dead, block_pos;
} OrcStateSizes;
/* The whole-model running-state sizes: gdn over every GDN layer, the indexer ones per QSA layer. */
int orc_state_sizes(int64_t n_layers, int64_t qsa_interval, int64_t ssm_state_size, int64_t ssm_v_heads,
                    int64_t ssm_d_conv, int64_t ssm_conv_channels, int64_t idx_key_dim, OrcStateSizes* out);

/* ---- FNV-1a 64 (src/core/pinned.cu:594-601; offset basis 1469598103934665603, prime 1099511628211) ---- */
uint64_t orc_fnv1a64(const uint8_t* p, uint64_t n, uint64_t seed);

/* ---- order-independent content check for full-size runs: a checksum of per-page checksums ----
 * page_sums[p] = FNV-1a of page p; the sequence checksum is FNV-1a over the page_sums array. */
uint64_t orc_page_checksum(const uint8_t* p, int64_t n_pages, uint64_t page_bytes);

/* ---- the streaming residency resolve (src/kernels/cuda/kv_stream.cu:82-158; policy: kv_stream.hpp:8-15) ----
 * One call over host copies of the map arrays, sequentially: for each query q and each position i < width(q) that
 * starts a block (ids ascending), a resident block takes `epoch = ctl[0] + 1` and its reference bit; a missing block
 * (table -1) is claimed (-2) and appended to the miss list.  Then the CLOCK hand from ctl[1] walks the slots: a
 * slot stamped this epoch is skipped, a free (block < 0) or unreferenced slot is taken for the next miss (stamped),
 * any other slot it passes loses its reference bit; the hand stops just past the slot that takes the last miss, and
 * walks at most 3 * n_slots slots.  Placed misses re-point the table (an evicted block goes to -1); unplaced ones
 * go back to -1 and set ctl[3].  ctl[0] = epoch, ctl[1] = hand, ctl[2] = placed, u64 counters at ctl[4..9]
 * (misses placed, lookups, calls).  Returns the number placed. */
int64_t orc_stream_resolve(int32_t* table, int32_t* slot_block, int32_t* slot_stamp, int32_t* slot_ref, int32_t* ctl,
                           int32_t* miss_block, int32_t* miss_slot, int64_t n_blocks, int64_t n_slots,
                           const int32_t* ids, const int32_t* steps, int64_t n_q, int64_t cap, int64_t page_size);

#ifdef __cplusplus
}
#endif
#endif
