// transfer.hpp - batched device <-> host moves for the snapshot layer (internal to libstrata_kv.so).
//
// A Transfer collects items - one logical byte range of a device stream (paged through a page table, or
// contiguous) paired with host memory (a ConversationBuffer's segments or a contiguous array) - and runs them as
// ONE batch on the device's legacy stream:
//   save:    one gather launch (skv_copy) device streams -> device staging image, then one cudaMemcpyAsync per
//            host piece staging -> host, then one synchronisation and a status-word check;
//   restore: one cudaMemcpyAsync per host piece host -> staging, then one scatter launch, then the same.
// The staging image is a per-device buffer kept between calls and grown on demand.
#pragma once

#include "strata_kv/conversation_buffer.hpp"

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace strata::kv {

/// A device byte stream: logical byte b lives at base + pages[b / page_bytes] * page_bytes + b % page_bytes, or at
/// base + b when `pages` is null.
struct DeviceStream {
    const void* base = nullptr;
    const int32_t* pages = nullptr;   // device int32 page table
    uint32_t page_bytes = 0;
    int64_t page_limit = 0;           // pages addressable from base
};

class Transfer {
public:
    /// Device stream bytes [from, to) -> the same range of `dst` (already sized to at least `to`).
    void save(const DeviceStream& src, uint64_t from, uint64_t to, strata::core::ConversationBuffer& dst);
    /// Device stream bytes [from, to) -> host array `dst` (dst[0] receives byte `from`).
    void save(const DeviceStream& src, uint64_t from, uint64_t to, uint8_t* dst);
    /// Host bytes -> device stream bytes [from, to).
    void restore(const strata::core::ConversationBuffer& src, uint64_t from, uint64_t to, const DeviceStream& dst);
    void restore(const uint8_t* src, uint64_t from, uint64_t to, const DeviceStream& dst);
    /// Host -> host copy run in the same batch (a streamed layer's authoritative host pool).
    void host_copy(const uint8_t* src, uint64_t from, uint64_t to, strata::core::ConversationBuffer& dst);
    /// The reverse: bytes [from, to) of `src` -> the same offsets of host memory `dst`.
    void host_restore(const strata::core::ConversationBuffer& src, uint64_t from, uint64_t to, uint8_t* dst);
    /// Work to enqueue on the batch's stream after every copy of it (a residency reset that must follow the
    /// writes); returns false with `error` set to refuse.
    void after(std::function<bool(std::string& error)> fn) { after_.push_back(std::move(fn)); }

    bool empty() const { return items_.empty() && host_.empty() && host_back_.empty() && after_.empty(); }
    size_t items() const { return items_.size(); }

    /// Run everything queued (saves and restores may not be mixed in one batch).  On failure `error` names the
    /// reason; a restore that failed after its first write has left partial state.  Either way nothing the batch
    /// enqueued is still running when it returns, so the caller may free the host memory at once.
    bool run(std::string& error, const char* what);

private:
    bool run_queued(std::string& error, const char* what, bool& enqueued);
    struct Piece {
        uint8_t* host;
        uint64_t rel;   // offset inside the item's range
        uint64_t bytes;
    };
    struct Item {
        DeviceStream dev;
        uint64_t from = 0, to = 0;
        bool save = true;
        std::vector<Piece> pieces;
    };
    struct HostCopy {
        const uint8_t* src;
        uint64_t from, to;
        strata::core::ConversationBuffer* dst;
    };
    struct HostBack {
        const strata::core::ConversationBuffer* src;
        uint64_t from, to;
        uint8_t* dst;
    };
    std::vector<Item> items_;
    std::vector<HostCopy> host_;
    std::vector<HostBack> host_back_;
    std::vector<std::function<bool(std::string&)>> after_;
};

/// The host-side steps of a batch, and the snapshot layer's device synchronisations, in the order a park or a mount
/// issues them.
enum class TransferStep { device_sync, copy, launch, stream_sync };
/// Test seam (fault injection): when a hook is set, every step above asks it first, and `true` fails that step as
/// if the CUDA runtime had returned an error - a copy or a launch is then not issued; a synchronisation still waits
/// and then reports the error.  No hook is set unless a test sets one.  Process-wide; set it while no batch runs.
using TransferFaultHook = bool (*)(TransferStep step);
void set_transfer_fault_hook(TransferFaultHook hook);
/// True when the hook (if any) fails this step.
bool transfer_fault(TransferStep step);

/// Bytes of the per-device staging image currently held (for tests and telemetry).
uint64_t transfer_staging_bytes(int device);
/// The current device's staging image (kept between calls, grown on demand), at least `bytes` long.  Shared by
/// every batch on that device: one batch at a time per device.
bool transfer_staging(uint64_t bytes, uint8_t** out, std::string& error, const char* what);

}  // namespace strata::kv
