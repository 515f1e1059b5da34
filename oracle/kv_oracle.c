/* oracle/kv_oracle.c - TEST INFRASTRUCTURE: CPU restatement of the reference's KV handoff / park path.
 * The checker, never the product (see kv_oracle.h).  Plain C, byte-exact by construction. */
#include "kv_oracle.h"

#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------- seeded generators */

static uint64_t splitmix64(uint64_t x) {
    /* Steele, Lea & Flood, "Fast splittable pseudorandom number generators" (OOPSLA 2014). */
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static double unit53(uint64_t r) { return (double) (r >> 11) * (1.0 / 9007199254740992.0); }

/* Element `i` of stream `seed`: two independent uniforms from two counters, Box-Muller cosine branch. */
static double normal_at(uint64_t seed, uint64_t i) {
    const uint64_t base = splitmix64(seed ^ 0xD1B54A32D192ED03ull);
    const double u1 = 1.0 - unit53(splitmix64(base + 2 * i));   /* (0, 1] so log() is finite */
    const double u2 = unit53(splitmix64(base + 2 * i + 1));
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

uint16_t orc_f32_to_f16(float x) {
    /* IEEE 754 binary32 -> binary16, round to nearest, ties to even. */
    uint32_t f;
    memcpy(&f, &x, 4);
    const uint32_t sign = (f >> 16) & 0x8000u;
    const uint32_t exp = (f >> 23) & 0xFFu;
    uint32_t man = f & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t) (sign | 0x7C00u | (man ? 0x200u | (man >> 13) : 0u));
    const int32_t e = (int32_t) exp - 127 + 15;
    if (e >= 31) return (uint16_t) (sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t) sign;
        man |= 0x800000u;
        const uint32_t shift = (uint32_t) (14 - e);
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t) (sign | h);
    }
    uint32_t h = ((uint32_t) e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  /* a carry into the exponent is still correct */
    return (uint16_t) (sign | h);
}

void orc_fill_f16_normal(uint16_t* out, uint64_t n, uint64_t seed, uint64_t offset) {
    for (uint64_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16((float) normal_at(seed, offset + i));
}

void orc_fill_f32_normal(float* out, uint64_t n, uint64_t seed, uint64_t offset, float sigma) {
    for (uint64_t i = 0; i < n; ++i) out[i] = sigma * (float) normal_at(seed, offset + i);
}

void orc_fill_ids(int32_t* out, uint64_t n, uint64_t seed, int32_t vocab) {
    const uint64_t base = splitmix64(seed ^ 0x6A09E667F3BCC909ull);
    for (uint64_t i = 0; i < n; ++i) out[i] = (int32_t) (splitmix64(base + i) % (uint64_t) vocab);
}

void orc_permutation(int32_t* out, int64_t n, uint64_t seed) {
    uint64_t state = splitmix64(seed ^ 0xBB67AE8584CAA73Bull);
    for (int64_t i = 0; i < n; ++i) out[i] = (int32_t) i;
    for (int64_t i = n - 1; i > 0; --i) {
        state = splitmix64(state);
        const int64_t j = (int64_t) (state % (uint64_t) (i + 1));
        const int32_t t = out[i];
        out[i] = out[j];
        out[j] = t;
    }
}

/* ---------------------------------------------------------------- the block table */

void orc_expand_block_table(const int32_t* block_table, int64_t n_blocks, int64_t pages_per_block,
                            int64_t slot_pages, int64_t page_offset, int32_t* page_table) {
    for (int64_t b = 0; b < n_blocks; ++b)
        for (int64_t j = 0; j < pages_per_block; ++j)
            page_table[b * pages_per_block + j] = (int32_t) ((int64_t) block_table[b] * slot_pages + page_offset + j);
}

void orc_gather_pages(const uint8_t* pool, const int32_t* page_table, int64_t n_pages, uint64_t page_bytes,
                      uint8_t* out) {
    for (int64_t p = 0; p < n_pages; ++p)
        memcpy(out + (uint64_t) p * page_bytes, pool + (uint64_t) page_table[p] * page_bytes, page_bytes);
}

void orc_scatter_pages(const uint8_t* in, const int32_t* page_table, int64_t n_pages, uint64_t page_bytes,
                       uint8_t* pool) {
    for (int64_t p = 0; p < n_pages; ++p)
        memcpy(pool + (uint64_t) page_table[p] * page_bytes, in + (uint64_t) p * page_bytes, page_bytes);
}

/* ---------------------------------------------------------------- snapshot extents */

enum { kPageCells = 4, kIdxBlock = 4, kQk4 = 32, kQ4BlockBytes = 18 };

int orc_kv_layout(int32_t format, int64_t upto, int include_index, int64_t n_head_kv, int64_t head_dim,
                  int64_t idx_key_dim, OrcKvLayout* out) {
    /* conversation_snapshot.cpp:27-67.  format: 0 fp16, 1 int8 (+ fp16 scale per 64), 2 q4_0, 3 hybrid. */
    if (upto < 0 || n_head_kv <= 0 || head_dim <= 0 || idx_key_dim <= 0 || format < 0 || format > 3) return -1;
    const int int8_keys = format == 1 || format == 3;
    if ((format == 2 && head_dim % 32) || (int8_keys && head_dim % 64)) return -1;
    const int64_t cells = ((upto + kPageCells - 1) / kPageCells) * kPageCells;
    const uint64_t q4_per = (uint64_t) (head_dim / kQk4) * kQ4BlockBytes;
    const uint64_t per = format == 2 ? q4_per : (uint64_t) head_dim * (int8_keys ? 1u : 2u);
    const int64_t pooled = include_index && upto > 0 ? upto / kIdxBlock + 1 : 0;
    out->format = format;
    out->cells = cells;
    out->pooled_rows = pooled;
    out->data = (uint64_t) cells * (uint64_t) n_head_kv * per;
    out->scales = int8_keys ? (uint64_t) cells * (uint64_t) n_head_kv * (uint64_t) (head_dim / 64) * 2u : 0u;
    out->pooled = (uint64_t) pooled * (uint64_t) idx_key_dim * 4u;
    out->value_data = format == 3 ? (uint64_t) cells * (uint64_t) n_head_kv * q4_per : out->data;
    out->value_scales = format == 3 ? 0u : out->scales;
    return 0;
}

int orc_state_sizes(int64_t n_layers, int64_t qsa_interval, int64_t ssm_state_size, int64_t ssm_v_heads,
                    int64_t ssm_d_conv, int64_t ssm_conv_channels, int64_t idx_key_dim, OrcStateSizes* out) {
    /* conversation_state.cpp:180-205: a GDN row is S*h_v*S recurrence + C*(d_conv-1) conv floats;
     * PLE history is NG_HIST(9) x NG_HC_DIM(10240) floats; the indexer tail is (idx_block-1) rows. */
    if (n_layers <= 0 || qsa_interval <= 0 || ssm_state_size <= 0 || ssm_v_heads <= 0 || ssm_d_conv <= 0 ||
        ssm_conv_channels <= 0 || idx_key_dim <= 0) return -1;
    const int64_t n_gdn = n_layers - n_layers / qsa_interval;
    const uint64_t row = (uint64_t) ssm_state_size * (uint64_t) ssm_v_heads * (uint64_t) ssm_state_size +
                         (uint64_t) ssm_conv_channels * (uint64_t) (ssm_d_conv - 1);
    out->gdn = (uint64_t) n_gdn * row * 4u;
    out->ple = 9u * 10240u * 4u;
    out->tail = (uint64_t) (kIdxBlock - 1) * (uint64_t) idx_key_dim * 4u;
    out->dead = (uint64_t) idx_key_dim * 4u;
    out->block_pos = 4u;
    return 0;
}

/* ---------------------------------------------------------------- hashes */

uint64_t orc_fnv1a64(const uint8_t* p, uint64_t n, uint64_t seed) {
    uint64_t h = seed;
    for (uint64_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

uint64_t orc_page_checksum(const uint8_t* p, int64_t n_pages, uint64_t page_bytes) {
    uint64_t outer = 1469598103934665603ull;
    for (int64_t i = 0; i < n_pages; ++i) {
        const uint64_t s = orc_fnv1a64(p + (uint64_t) i * page_bytes, page_bytes, 1469598103934665603ull);
        outer = orc_fnv1a64((const uint8_t*) &s, 8, outer);
    }
    return outer;
}

/* ---- the streaming residency resolve, restated sequentially (kv_oracle.h) ---- */
int64_t orc_stream_resolve(int32_t* table, int32_t* slot_block, int32_t* slot_stamp, int32_t* slot_ref, int32_t* ctl,
                           int32_t* miss_block, int32_t* miss_slot, int64_t n_blocks, int64_t n_slots,
                           const int32_t* ids, const int32_t* steps, int64_t n_q, int64_t cap, int64_t page_size) {
    const int32_t epoch = ctl[0] + 1;
    int64_t n_miss = 0, lookups = 0;
    int overflow = 0;
    for (int64_t q = 0; q < n_q; ++q) {
        int64_t width = steps[q * 4 + 3];
        if (width > cap) width = cap;
        const int32_t* qi = ids + q * cap;
        for (int64_t i = 0; i < width; ++i) {
            const int64_t b = qi[i] / page_size;
            if (i > 0 && qi[i - 1] / page_size == b) continue;
            if (b < 0 || b >= n_blocks) continue;
            ++lookups;
            const int32_t sl = table[b];
            if (sl >= 0) {
                slot_stamp[sl] = epoch;
                slot_ref[sl] = 1;
            } else if (sl == -1) {
                if (n_miss < n_slots) {
                    table[b] = -2;
                    miss_block[n_miss] = (int32_t) b;
                } else {
                    overflow = 1;   /* more distinct misses than slots: the block stays evicted */
                }
                ++n_miss;
            }
        }
    }
    const int64_t need = n_miss < n_slots ? n_miss : n_slots;
    int64_t hand = ctl[1], got = 0;
    for (int64_t walked = 0; got < need && walked < 3 * n_slots; ++walked) {
        const int64_t j = hand % n_slots;
        hand = (hand + 1) % n_slots;
        if (slot_stamp[j] == epoch) continue;
        if (slot_block[j] < 0 || slot_ref[j] == 0) {
            miss_slot[got++] = (int32_t) j;
            slot_stamp[j] = epoch;
        } else {
            slot_ref[j] = 0;
        }
    }
    for (int64_t k = 0; k < need; ++k) {
        const int32_t b = miss_block[k];
        if (k >= got) {
            table[b] = -1;
            continue;
        }
        const int32_t sl = miss_slot[k];
        if (slot_block[sl] >= 0) table[slot_block[sl]] = -1;
        slot_block[sl] = b;
        slot_stamp[sl] = epoch;
        slot_ref[sl] = 1;
        table[b] = sl;
    }
    ctl[0] = epoch;
    ctl[1] = (int32_t) hand;
    ctl[2] = (int32_t) got;
    if (got < n_miss || overflow) ctl[3] = 1;
    uint64_t c[3];
    memcpy(c, ctl + 4, sizeof c);
    c[0] += (uint64_t) got;
    c[1] += (uint64_t) lookups;
    c[2] += 1;
    memcpy(ctl + 4, c, sizeof c);
    return got;
}
