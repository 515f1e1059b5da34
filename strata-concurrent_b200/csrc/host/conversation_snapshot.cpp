// conversation_snapshot.cpp - one QSA layer's K/V between device pools and a ConversationKv
// (include/strata_kv/conversation_snapshot.hpp; the reference's src/core/conversation_snapshot.cpp:27-262).
//
// The extents and the refusal rules are the reference's (a layer's snapshot covers whole 4-cell pages up to
// `upto`, K/V data and scales per format, and the indexer's pooled rows including the moving spare row); the
// movement is this build's: every stream is read or written by the copy kernels - through QsaState::page_table
// when the layer lives in a block pool - batched into one launch with the rest of the session
// (snapshot_detail::enqueue_*).  Streamed (kv_mode 1) and ring (kv_mode 2) layers keep their authoritative K/V in
// pinned host memory: a park copies it, a mount writes it back and then evicts every block (mode 1) or refills
// the ring (mode 2), as the reference does (src/core/conversation_snapshot.cpp:190-206).
#include "snapshot_detail.hpp"

#include "kv_stream_detail.h"
#include "skv_internal.h"

#include <algorithm>
#include <array>
#include <cstring>
#include <limits>

namespace strata::core {
namespace snapshot_detail {

bool fail(std::string& error, const char* message) {
    error = std::string("conversation snapshot: ") + message;
    return false;
}

bool checked_product(size_t& out, std::initializer_list<uint64_t> factors) {
    uint64_t v = 1;
    for (uint64_t f : factors) {
        if (f && v > std::numeric_limits<uint64_t>::max() / f) return false;
        v *= f;
    }
    if (v > std::numeric_limits<size_t>::max()) return false;
    out = (size_t) v;
    return true;
}

bool checked_add(size_t& total, size_t n) {
    if (n > std::numeric_limits<size_t>::max() - total) return false;
    total += n;
    return true;
}

bool layer_extent(const QsaState& st, const ModelGeometry& g, int64_t upto, bool index, LayerExtent& x,
                  std::string& error) {
    const auto shapes = strata::kernels::qsa_real_shapes();
    const int64_t ps = shapes.page_size;
    if (upto < 0 || upto > st.max_cells || upto > std::numeric_limits<int64_t>::max() - (ps - 1))
        return fail(error, "invalid K/V extent");
    if (st.kv_hybrid && (st.kv_mode != 0 || st.kv_q4 || st.kv_int8))
        return fail(error, "hybrid K8V4 requires an identity layout and distinct format flags");
    const bool int8_keys = st.kv_int8 || st.kv_hybrid;
    if (g.n_head_kv <= 0 || g.head_dim <= 0 || g.head_dim > INT32_MAX || g.idx_key_dim <= 0 ||
        (st.kv_q4 && g.head_dim % 32) || (int8_keys && !st.kv_q4 && g.head_dim % 64))
        return fail(error, "invalid K/V geometry");
    const uint64_t q4 = strata::kernels::kv_q4_bytes_per_head((int) g.head_dim);
    const uint64_t per = st.kv_q4 ? q4 : (uint64_t) g.head_dim * (int8_keys ? 1u : 2u);
    x = LayerExtent{};
    x.page_size = ps;
    x.cells = ((upto + ps - 1) / ps) * ps;
    x.pooled_rows = index && upto > 0 ? upto / shapes.idx_block + 1 : 0;
    x.format = st.kv_hybrid ? 3 : qsa_kv_format(st);
    const uint64_t scale_per_cell_head = int8_keys && !st.kv_q4 ? (uint64_t) (g.head_dim / 64) * 2 : 0;
    if (!checked_product(x.bytes[0], {(uint64_t) x.cells, (uint64_t) g.n_head_kv, per}) ||
        !checked_product(x.bytes[2], {(uint64_t) x.cells, (uint64_t) g.n_head_kv, scale_per_cell_head}) ||
        !checked_product(x.bytes[4], {(uint64_t) x.pooled_rows, (uint64_t) g.idx_key_dim, sizeof(float)}))
        return fail(error, "K/V byte count overflow");
    x.bytes[1] = x.bytes[0];
    x.bytes[3] = x.bytes[2];
    if (st.kv_hybrid) {
        if (!checked_product(x.bytes[1], {(uint64_t) x.cells, (uint64_t) g.n_head_kv, q4}))
            return fail(error, "hybrid V byte count overflow");
        x.bytes[3] = 0;
    }
    return true;
}

bool layer_usable(const QsaState& st, const LayerExtent& x, int64_t upto, std::string& error) {
    if (upto < 0 || upto > st.max_cells || st.n_pages < 0 || x.cells / x.page_size > st.n_pages || st.kv_mode < 0 ||
        st.kv_mode > 2 || st.n_slots <= 0 || (st.kv_mode == 0 && st.n_slots < st.n_pages) ||
        x.pooled_rows > st.idx_pooled_rows || (st.kv_mode != 0 && !st.host.present()))
        return fail(error, "invalid K/V extent or missing authoritative host pool");
    if (st.kv_mode == 1) {
        const auto& m = st.map;
        if (m.n_blocks != st.n_pages || m.n_slots != st.n_slots || !m.page_table || !m.slot_block || !m.slot_stamp ||
            !m.slot_ref || !m.ctl || !m.miss_block || !m.miss_slot)
            return fail(error, "invalid streaming map");
    }
    if (st.kv_mode == 2 &&
        (!st.page_table || (st.kv_q4      ? !st.k_q4 || !st.v_q4
                            : st.kv_int8 ? !st.k_q || !st.v_q || !st.k_scale || !st.v_scale
                                         : !st.k_pool || !st.v_pool)))
        return fail(error, "invalid draft ring");
    return true;
}

std::array<const void*, 5> layer_sources(const QsaState& st) {
    const bool host = st.kv_mode != 0;
    if (st.kv_hybrid) return {st.k_q, st.v_q4, st.k_scale, nullptr, st.idx_pooled};
    if (st.kv_q4) return {host ? st.host.k_q4 : st.k_q4, host ? st.host.v_q4 : st.v_q4, nullptr, nullptr, st.idx_pooled};
    if (st.kv_int8)
        return {host ? (const void*) st.host.k_q : st.k_q, host ? (const void*) st.host.v_q : st.v_q,
                host ? st.host.k_scale : st.k_scale, host ? st.host.v_scale : st.v_scale, st.idx_pooled};
    return {host ? st.host.k_pool : st.k_pool, host ? st.host.v_pool : st.v_pool, nullptr, nullptr, st.idx_pooled};
}

std::array<const void*, 5> layer_slots(const QsaState& st) {
    if (st.kv_hybrid) return {st.k_q, st.v_q4, st.k_scale, nullptr, st.idx_pooled};
    if (st.kv_q4) return {st.k_q4, st.v_q4, nullptr, nullptr, st.idx_pooled};
    if (st.kv_int8) return {st.k_q, st.v_q, st.k_scale, st.v_scale, st.idx_pooled};
    return {st.k_pool, st.v_pool, nullptr, nullptr, st.idx_pooled};
}

strata::kv::DeviceStream layer_stream(const QsaState& st, const LayerExtent& x, int i, const void* base) {
    strata::kv::DeviceStream s;
    s.base = base;
    // a block-pool layer is addressed through its table; any other resident layer is identity-addressed, which is
    // what the reference assumes of every kv_mode 0 layer
    if (i < 4 && st.kv_mode == 0 && st.page_table && x.cells > 0 && skv::in_block_pool(base)) {
        const int64_t pages = x.cells / x.page_size;
        s.pages = st.page_table;
        s.page_bytes = (uint32_t) (x.bytes[(size_t) i] / (size_t) pages);
        s.page_limit = st.n_slots;
    }
    return s;
}

bool enqueue_kv_save(ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto, bool index,
                     strata::kv::Transfer& t, std::string& error, int64_t unchanged, size_t* reused_bytes) {
    LayerExtent x;
    if (!layer_extent(st, g, upto, index, x, error) || !layer_usable(st, x, upto, error)) return false;
    if (unchanged < 0 || unchanged > upto || unchanged > image.cells) return fail(error, "invalid unchanged prefix");
    const int64_t whole = (unchanged / x.page_size) * x.page_size;
    image.format = x.format;
    image.cells = x.cells;
    image.heads = g.n_head_kv;
    image.head_dim = g.head_dim;
    image.page_size = x.page_size;
    image.pooled_rows = x.pooled_rows;
    image.idx_dim = g.idx_key_dim;
    const auto src = layer_sources(st);
    ConversationBuffer* dst[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    const int64_t idx_block = strata::kernels::qsa_real_shapes().idx_block;
    for (int i = 0; i < 5; ++i) {
        // pages and indexer rows strictly before the first rewritten token are unchanged; re-copy the rest
        const size_t n = x.bytes[(size_t) i];
        const size_t keep = i == 4 ? (index ? (size_t) (unchanged / idx_block) * (size_t) g.idx_key_dim * 4 : 0)
                                   : (x.cells ? (n / (size_t) x.cells) * (size_t) whole : 0);
        if (keep > dst[i]->size()) return fail(error, "missing reusable prefix");
        dst[i]->resize(n);
        if (n > keep) {
            if (!src[(size_t) i]) return fail(error, "missing state buffer");
            if (i < 4 && st.kv_mode != 0)
                t.host_copy(static_cast<const uint8_t*>(src[(size_t) i]), keep, n, *dst[i]);
            else
                t.save(layer_stream(st, x, i, src[(size_t) i]), keep, n, *dst[i]);
        }
        if (reused_bytes) *reused_bytes += keep;
    }
    return true;
}

bool enqueue_kv_restore(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                        bool index, strata::kv::Transfer& t, std::string& error) {
    if (!conversation_kv_validate(image, st, g, upto, index, error)) return false;
    LayerExtent x;
    layer_extent(st, g, upto, index, x, error);
    const auto dst = layer_sources(st);
    const ConversationBuffer* src[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    for (int i = 0; i < 5; ++i) {
        if (!src[i]->size()) continue;
        if (i < 4 && st.kv_mode != 0)
            t.host_restore(*src[i], 0, src[i]->size(), static_cast<uint8_t*>(const_cast<void*>(dst[(size_t) i])));
        else
            t.restore(*src[i], 0, src[i]->size(), layer_stream(st, x, i, dst[(size_t) i]));
    }
    if (st.kv_mode == 1) {
        // the VRAM slots still hold the outgoing conversation: evict every block, resolve refills from the host copy
        const strata::kernels::KvStreamMap map = st.map;
        t.after([map](std::string& err) {
            if (skv::stream_reset(map, nullptr) == SKV_OK) return true;
            err = std::string("conversation snapshot residency restore: ") + skv_last_error();
            return false;
        });
    } else if (st.kv_mode == 2 && x.cells > 0) {
        // the ring holds the last n_slots pages: refill them (page b -> slot b % n_slots) from the restored bytes
        const int64_t end = x.cells / x.page_size, begin = std::max<int64_t>(0, end - st.n_slots);
        const auto slots = layer_slots(st);
        for (int i = 0; i < 4; ++i) {
            if (!src[i]->size()) continue;
            const uint64_t pb = src[i]->size() / (uint64_t) end;
            for (int64_t b = begin; b < end;) {
                const int64_t sl = b % st.n_slots, run = std::min<int64_t>(end - b, st.n_slots - sl);
                // restore(src, from, to, dst) writes image byte `from` at dst.base + from: the base is shifted so
                // that page b lands in slot b % n_slots
                strata::kv::DeviceStream ring;
                ring.base = reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(slots[(size_t) i]) +
                                                          (uint64_t) sl * pb - (uint64_t) b * pb);
                t.restore(*src[i], (uint64_t) b * pb, (uint64_t) (b + run) * pb, ring);
                b += run;
            }
        }
    }
    return true;
}

}  // namespace snapshot_detail

using namespace snapshot_detail;

bool conversation_kv_capture_bytes(const ConversationKv& image, const QsaState& st, const ModelGeometry& g,
                                   int64_t upto, bool index, size_t& bytes, std::string& error) {
    LayerExtent x;
    if (!layer_extent(st, g, upto, index, x, error) || !layer_usable(st, x, upto, error)) return false;
    const ConversationBuffer* b[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    bytes = 0;
    for (int i = 0; i < 5; ++i) {
        const size_t peak = b[i]->allocation_peak(x.bytes[(size_t) i]);
        if (peak == SIZE_MAX || !checked_add(bytes, peak)) return fail(error, "segmented K/V allocation overflow");
    }
    return true;
}

size_t conversation_kv_bytes(const QsaState& st, const ModelGeometry& g, int64_t upto, bool index) {
    size_t bytes = 0;
    std::string error;
    return conversation_kv_capture_bytes({}, st, g, upto, index, bytes, error) ? bytes : 0;
}

bool conversation_kv_save(ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto, bool index,
                          std::string& error, int64_t unchanged_tokens, size_t* reused_bytes) {
    strata::kv::Transfer t;
    if (!enqueue_kv_save(image, st, g, upto, index, t, error, unchanged_tokens, reused_bytes)) return false;
    return t.run(error, "conversation snapshot copy");
}

bool conversation_kv_validate(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                              bool index, std::string& error) {
    return kv_validate_sized(image, st, g, upto, index, error, own_size);
}

bool snapshot_detail::kv_validate_sized(const ConversationKv& image, const QsaState& st, const ModelGeometry& g,
                                        int64_t upto, bool index, std::string& error, const SizeOf& size_of) {
    LayerExtent x;
    if (!layer_extent(st, g, upto, index, x, error) || !layer_usable(st, x, upto, error)) return false;
    if (image.format != x.format || image.cells != x.cells || image.heads != g.n_head_kv ||
        image.head_dim != g.head_dim || image.page_size != x.page_size || image.pooled_rows != x.pooled_rows ||
        image.idx_dim != g.idx_key_dim)
        return fail(error, "incompatible K/V geometry");
    const ConversationBuffer* b[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    for (int i = 0; i < 5; ++i)
        if (size_of(b[i], b[i]->size()) != x.bytes[(size_t) i]) return fail(error, "invalid K/V payload size");
    const auto dst = layer_sources(st);
    for (int i = 0; i < 5; ++i)
        if (x.bytes[(size_t) i] && !dst[(size_t) i]) return fail(error, "missing target state buffer");
    return true;
}

bool conversation_kv_restore(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                             bool index, std::string& error) {
    strata::kv::Transfer t;
    if (!enqueue_kv_restore(image, st, g, upto, index, t, error)) return false;
    return t.run(error, "conversation snapshot copy");
}

bool conversation_kv_verify(const ConversationKv& image, const QsaState& st, const ModelGeometry& g, int64_t upto,
                            bool index, uint64_t& fingerprint, std::string& error) {
    if (!conversation_kv_validate(image, st, g, upto, index, error)) return false;
    LayerExtent x;
    layer_extent(st, g, upto, index, x, error);
    const auto src = layer_sources(st);
    const ConversationBuffer* saved[5] = {&image.k, &image.v, &image.k_scale, &image.v_scale, &image.pooled};
    std::array<ConversationBuffer, 5> back;
    strata::kv::Transfer t;
    for (int i = 0; i < 5; ++i) {
        const size_t n = x.bytes[(size_t) i];
        back[(size_t) i].resize(n);
        if (!n) continue;
        if (i < 4 && st.kv_mode != 0)   // the authoritative host copy
            t.host_copy(static_cast<const uint8_t*>(src[(size_t) i]), 0, n, back[(size_t) i]);
        else
            t.save(layer_stream(st, x, i, src[(size_t) i]), 0, n, back[(size_t) i]);
    }
    // a ring also keeps its last n_slots pages resident: read the slot arrays back too
    std::array<std::vector<uint8_t>, 4> ring;
    const int64_t end = x.page_size ? x.cells / x.page_size : 0;
    if (st.kv_mode == 2 && end > 0) {
        const auto slots = layer_slots(st);
        for (int i = 0; i < 4; ++i) {
            if (!saved[i]->size()) continue;
            const uint64_t pb = saved[i]->size() / (uint64_t) end;
            ring[(size_t) i].resize((size_t) (pb * (uint64_t) st.n_slots));
            strata::kv::DeviceStream d;
            d.base = slots[(size_t) i];
            t.save(d, 0, ring[(size_t) i].size(), ring[(size_t) i].data());
        }
    }
    if (!t.run(error, "conversation snapshot read-back")) return false;
    if (st.kv_mode == 2 && end > 0) {
        const int64_t begin = std::max<int64_t>(0, end - st.n_slots);
        for (int i = 0; i < 4; ++i) {
            if (!saved[i]->size()) continue;
            const uint64_t pb = saved[i]->size() / (uint64_t) end;
            std::vector<uint8_t> page((size_t) pb);
            for (int64_t b = begin; b < end; ++b) {
                if (!saved[i]->read(page.data(), (size_t) ((uint64_t) b * pb), (size_t) pb) ||
                    std::memcmp(page.data(), ring[(size_t) i].data() + (uint64_t) (b % st.n_slots) * pb, (size_t) pb))
                    return fail(error, "restored K/V bytes differ");
            }
        }
    }
    uint64_t hash = 1469598103934665603ull;
    for (int i = 0; i < 5; ++i) {
        if (!(back[(size_t) i] == *saved[i])) return fail(error, "restored K/V bytes differ");
        back[(size_t) i].visit(0, back[(size_t) i].size(), [&](const uint8_t* p, size_t n, size_t) {
            for (size_t j = 0; j < n; ++j) {
                hash ^= p[j];
                hash *= 1099511628211ull;
            }
            return true;
        });
    }
    fingerprint = hash;
    return true;
}

}  // namespace strata::core
