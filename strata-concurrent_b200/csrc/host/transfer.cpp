// transfer.cpp - batched device <-> host moves for the snapshot layer (see transfer.hpp).
#include "transfer.hpp"

#include "strata_kv.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <unordered_map>

namespace strata::kv {
namespace {

std::atomic<TransferFaultHook> g_fault_hook{nullptr};

struct Staging {
    uint8_t* ptr = nullptr;
    uint64_t bytes = 0;
};
std::mutex g_staging_mu;
std::unordered_map<int, Staging> g_staging;

uint64_t round256(uint64_t n) { return (n + 255) & ~uint64_t(255); }

bool cuda_ok(cudaError_t e, std::string& error, const char* what, const char* step) {
    if (e == cudaSuccess) return true;
    (void) cudaGetLastError();
    error = std::string(what) + ": " + step + ": " + cudaGetErrorString(e);
    return false;
}

/// The current device's staging image, at least `bytes` long.
bool staging_for(uint64_t bytes, uint8_t** out, std::string& error, const char* what) {
    int dev = -1;
    if (!cuda_ok(cudaGetDevice(&dev), error, what, "cudaGetDevice")) return false;
    std::lock_guard<std::mutex> lock(g_staging_mu);
    Staging& s = g_staging[dev];
    if (s.bytes < bytes) {
        if (s.ptr) (void) cudaFree(s.ptr);
        s.ptr = nullptr;
        s.bytes = 0;
        const uint64_t want = std::max<uint64_t>(bytes, uint64_t(64) << 20);
        if (!cuda_ok(cudaMalloc(&s.ptr, want), error, what, "staging cudaMalloc")) return false;
        s.bytes = want;
    }
    *out = s.ptr;
    return true;
}

void pieces_of(strata::core::ConversationBuffer& b, uint64_t from, uint64_t to, std::vector<uint8_t*>& ptrs,
               std::vector<uint64_t>& rels, std::vector<uint64_t>& lens) {
    b.visit(from, to - from, [&](uint8_t* p, size_t n, size_t at) {
        ptrs.push_back(p);
        rels.push_back(at - from);
        lens.push_back(n);
        return true;
    });
}

}  // namespace

void set_transfer_fault_hook(TransferFaultHook hook) { g_fault_hook.store(hook); }

bool transfer_fault(TransferStep step) {
    const TransferFaultHook hook = g_fault_hook.load();
    return hook && hook(step);
}

bool transfer_staging(uint64_t bytes, uint8_t** out, std::string& error, const char* what) {
    return staging_for(bytes, out, error, what);
}

uint64_t transfer_staging_bytes(int device) {
    std::lock_guard<std::mutex> lock(g_staging_mu);
    auto it = g_staging.find(device);
    return it == g_staging.end() ? 0 : it->second.bytes;
}

void Transfer::save(const DeviceStream& src, uint64_t from, uint64_t to, strata::core::ConversationBuffer& dst) {
    if (to <= from) return;
    Item it{src, from, to, true, {}};
    std::vector<uint8_t*> p;
    std::vector<uint64_t> r, n;
    pieces_of(dst, from, to, p, r, n);
    for (size_t i = 0; i < p.size(); ++i) it.pieces.push_back(Piece{p[i], r[i], n[i]});
    items_.push_back(std::move(it));
}

void Transfer::save(const DeviceStream& src, uint64_t from, uint64_t to, uint8_t* dst) {
    if (to <= from) return;
    items_.push_back(Item{src, from, to, true, {Piece{dst, 0, to - from}}});
}

void Transfer::restore(const strata::core::ConversationBuffer& src, uint64_t from, uint64_t to, const DeviceStream& dst) {
    if (to <= from) return;
    Item it{dst, from, to, false, {}};
    src.visit(from, to - from, [&](const uint8_t* p, size_t n, size_t at) {
        it.pieces.push_back(Piece{const_cast<uint8_t*>(p), at - from, n});
        return true;
    });
    items_.push_back(std::move(it));
}

void Transfer::restore(const uint8_t* src, uint64_t from, uint64_t to, const DeviceStream& dst) {
    if (to <= from) return;
    items_.push_back(Item{dst, from, to, false, {Piece{const_cast<uint8_t*>(src), 0, to - from}}});
}

void Transfer::host_copy(const uint8_t* src, uint64_t from, uint64_t to, strata::core::ConversationBuffer& dst) {
    if (to > from) host_.push_back(HostCopy{src, from, to, &dst});
}

void Transfer::host_restore(const strata::core::ConversationBuffer& src, uint64_t from, uint64_t to, uint8_t* dst) {
    if (to > from) host_back_.push_back(HostBack{&src, from, to, dst});
}

namespace {
/// cudaMemcpyAsync through the fault seam.
cudaError_t copy_async(void* dst, const void* src, size_t n, cudaMemcpyKind kind, cudaStream_t stream) {
    return transfer_fault(TransferStep::copy) ? cudaErrorInvalidValue : cudaMemcpyAsync(dst, src, n, kind, stream);
}
}  // namespace

bool Transfer::run(std::string& error, const char* what) {
    bool enqueued = false;
    const bool ok = run_queued(error, what, enqueued);
    // a failure part way leaves earlier copies in flight: let them finish before the caller frees or reuses the host
    // memory they read or write (the batch's own result stands; this wait's is of no further use)
    if (!ok && enqueued) (void) cudaStreamSynchronize(nullptr);
    return ok;
}

bool Transfer::run_queued(std::string& error, const char* what, bool& enqueued) {
    const cudaStream_t stream = nullptr;   // the legacy stream: ordered after the caller's earlier device work
    bool saving = true;
    for (size_t i = 0; i < items_.size(); ++i) {
        if (i == 0) saving = items_[0].save;
        if (items_[i].save != saving) {
            error = std::string(what) + ": internal: a transfer batch mixes saves and restores";
            return false;
        }
    }
    if ((!host_.empty() && !host_back_.empty()) || (!items_.empty() && !host_.empty() && !saving) ||
        (!items_.empty() && !host_back_.empty() && saving)) {
        error = std::string(what) + ": internal: a transfer batch mixes saves and restores";
        return false;
    }
    for (const HostBack& h : host_back_) {
        bool ok = true;
        h.src->visit(h.from, h.to - h.from, [&](const uint8_t* p, size_t n, size_t at) {
            ok = cuda_ok(copy_async(h.dst + at, p, n, cudaMemcpyDefault, stream), error, what, "host pool copy");
            enqueued = enqueued || ok;
            return ok;
        });
        if (!ok) return false;
    }
    for (const HostCopy& h : host_) {
        bool ok = true;
        h.dst->visit(h.from, h.to - h.from, [&](uint8_t* p, size_t n, size_t at) {
            ok = cuda_ok(copy_async(p, h.src + at, n, cudaMemcpyDefault, stream), error, what, "host pool copy");
            enqueued = enqueued || ok;
            return ok;
        });
        if (!ok) return false;
    }
    // Contiguous items that are not 16-byte granular (a 4-byte block position, say) cannot go through the copy
    // kernels without touching bytes outside their buffer; the copy engine moves them directly.
    std::vector<const Item*> kernel_items, direct_items;
    bool launched = false;
    for (const Item& it : items_) {
        const uintptr_t at = reinterpret_cast<uintptr_t>(static_cast<const uint8_t*>(it.dev.base) + it.from);
        const bool granular = ((at | (it.to - it.from)) & 15u) == 0;
        if (it.dev.pages || granular) kernel_items.push_back(&it);
        else direct_items.push_back(&it);
    }
    for (const Item* it : direct_items)
        for (const Piece& p : it->pieces) {
            uint8_t* dev = const_cast<uint8_t*>(static_cast<const uint8_t*>(it->dev.base)) + it->from + p.rel;
            const cudaError_t e = it->save ? copy_async(p.host, dev, p.bytes, cudaMemcpyDeviceToHost, stream)
                                           : copy_async(dev, p.host, p.bytes, cudaMemcpyHostToDevice, stream);
            if (!cuda_ok(e, error, what, "running-state copy")) return false;
            enqueued = true;
        }
    if (!kernel_items.empty()) {
        uint64_t total = 0;
        std::vector<uint64_t> off(kernel_items.size());
        for (size_t i = 0; i < kernel_items.size(); ++i) {
            off[i] = total;
            total += round256(kernel_items[i]->to - kernel_items[i]->from);
        }
        uint8_t* staging = nullptr;
        if (!staging_for(total, &staging, error, what)) return false;
        int dev = -1;
        if (!cuda_ok(cudaGetDevice(&dev), error, what, "cudaGetDevice")) return false;
        if (skv_clear_status(dev, stream) != SKV_OK) {
            error = std::string(what) + ": " + skv_last_error();
            return false;
        }
        std::vector<skv_segment> segs;
        segs.reserve(kernel_items.size());
        for (size_t i = 0; i < kernel_items.size(); ++i) {
            const Item& it = *kernel_items[i];
            skv_segment s{};
            uint8_t* stage = staging + off[i];
            const uint8_t* base = static_cast<const uint8_t*>(it.dev.base);
            const int32_t* table = nullptr;
            const uint8_t* dev_at = base + it.from;
            if (it.dev.pages) {
                if (it.dev.page_bytes == 0 || it.from % it.dev.page_bytes || (it.to - it.from) % it.dev.page_bytes) {
                    error = std::string(what) + ": internal: a paged range is not page aligned";
                    return false;
                }
                table = it.dev.pages + it.from / it.dev.page_bytes;
                dev_at = base;
            }
            s.bytes = it.to - it.from;
            s.page_bytes = it.dev.page_bytes;
            if (it.save) {
                s.src = dev_at;
                s.src_pages = table;
                s.src_page_limit = it.dev.page_limit;
                s.dst = stage;
            } else {
                s.src = stage;
                s.dst = const_cast<uint8_t*>(dev_at);
                s.dst_pages = table;
                s.dst_page_limit = it.dev.page_limit;
            }
            segs.push_back(s);
        }
        auto launch = [&]() -> bool {
            for (size_t i = 0; i < segs.size(); i += SKV_COPY_MAX_SEGMENTS) {
                const int n = (int) std::min<size_t>(SKV_COPY_MAX_SEGMENTS, segs.size() - i);
                if (transfer_fault(TransferStep::launch)) {
                    error = std::string(what) + ": copy kernel launch failed (injected)";
                    return false;
                }
                if (skv_copy(segs.data() + i, n, SKV_COPY_AUTO, stream) != SKV_OK) {
                    error = std::string(what) + ": " + skv_last_error();
                    return false;
                }
                enqueued = true;
            }
            return true;
        };
        auto host_moves = [&](bool to_host) -> bool {
            for (size_t i = 0; i < kernel_items.size(); ++i)
                for (const Piece& p : kernel_items[i]->pieces) {
                    uint8_t* stage = staging + off[i] + p.rel;
                    const cudaError_t e =
                        to_host ? copy_async(p.host, stage, p.bytes, cudaMemcpyDeviceToHost, stream)
                                : copy_async(stage, p.host, p.bytes, cudaMemcpyHostToDevice, stream);
                    if (!cuda_ok(e, error, what, to_host ? "device-to-host copy" : "host-to-device copy")) return false;
                    enqueued = true;
                }
            return true;
        };
        if (saving) {
            if (!launch() || !host_moves(true)) return false;
        } else {
            if (!host_moves(false) || !launch()) return false;
        }
        launched = true;
    }
    for (auto& fn : after_) {
        enqueued = true;   // the follow-up work may have enqueued before it refused
        if (!fn(error)) return false;
    }
    cudaError_t synced = cudaStreamSynchronize(stream);
    if (synced == cudaSuccess && transfer_fault(TransferStep::stream_sync)) synced = cudaErrorUnknown;
    if (!cuda_ok(synced, error, what, "synchronize")) return false;
    if (launched) {   // the status word the kernels of this batch reported into
        int dev = -1;
        uint32_t status = 0;
        cudaGetDevice(&dev);
        if (skv_query_status(dev, stream, &status) != SKV_OK) {
            error = std::string(what) + ": " + skv_last_error();
            return false;
        }
        if (status) {
            char bits[16];
            std::snprintf(bits, sizeof bits, "0x%x", (unsigned) status);
            error = std::string(what) + ": the device refused part of the copy (status " + bits +
                    ": a page-table entry outside its pool)";
            return false;
        }
    }
    items_.clear();
    host_.clear();
    host_back_.clear();
    after_.clear();
    return true;
}

}  // namespace strata::kv
