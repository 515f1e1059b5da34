// include/strata_kv/handoff_device.hpp - the split-role hand-off with the payload left in the prefill GPU's HBM.
//
// The reference's split roles hand a finished prefill to the decode instance through a HandoffArena slot that
// holds the whole SR4H payload (include/strata/program/prefill_svc.hpp: CLAIM, SEG, DONE, ACK; the slot is a
// tmpfs file the decode side maps and decodes).  When both instances share a node, this build keeps the slot
// table and the protocol but moves only a 256-byte DEVICE DESCRIPTOR through the slot:
//
//   prefill: claim a slot; conversation_wire_pack_device into a device buffer it exported with CUDA IPC (the
//            same SR4H bytes, now in HBM); write the descriptor (the IPC handle, the payload's size and offset,
//            its identity hashes) into the slot; publish; send DONE.  The prefill may free its pool blocks now.
//   decode:  read_slot (the same checks: nonce, client, pack, geometry); recognise the descriptor by its magic;
//            import the handle (once per exporting allocation, cached); conversation_wire_mount_device straight
//            from the peer's HBM into its own pools over NVLink; send ACK.  The prefill then releases the slot and
//            may reuse the payload buffer.
//
// A slot holds either an SR4H payload or a descriptor; handoff_device_is_descriptor tells them apart, so a
// decode instance serves both (a descriptor from a prefill on its node, a payload from anywhere else).
#pragma once

#include "strata_kv/conversation_wire_device.hpp"
#include "strata_kv/handoff.hpp"

#include <cstdint>
#include <map>
#include <string>

namespace strata::core {

inline constexpr uint64_t kDeviceDescriptorBytes = 256;
inline constexpr char kDeviceDescriptorMagic[8] = {'S', 'R', '4', 'D', 'E', 'V', '0', '1'};
inline constexpr uint32_t kDeviceDescriptorVersion = 1;

/// What the slot carries instead of the payload.
struct HandoffDeviceDescriptor {
    uint8_t ipc_handle[64] = {};   ///< cudaIpcMemHandle_t of the allocation holding the payload
    uint64_t alloc_offset = 0;     ///< the payload's offset inside that allocation
    uint64_t payload_bytes = 0;    ///< the SR4H payload's size
    int32_t device = -1;           ///< the exporting process's CUDA ordinal (informative)
    char pci_bus_id[32] = {};      ///< where the payload lives ("0000:1b:00.0"), for the reader's reachability check
    uint64_t geom_hash = 0, pack_hash = 0;   ///< the payload header's identity
    uint64_t tokens = 0;
    uint64_t payload_fnv = 0;      ///< FNV-1a of the payload when the writer computed it, else 0
};

/// The 256-byte record (little-endian): magic, version, then the fields in declaration order, zero padded.
void handoff_device_encode(const HandoffDeviceDescriptor& d, uint8_t out[kDeviceDescriptorBytes]);
bool handoff_device_decode(const uint8_t* data, uint64_t bytes, HandoffDeviceDescriptor& out, std::string& error);
/// True when a slot's bytes are a device descriptor (by size and magic), false for anything else (an SR4H payload).
bool handoff_device_is_descriptor(const uint8_t* data, uint64_t bytes);

/// Prefill side, after claim(): pack the session into `device_buffer` (at `alloc_offset` inside the allocation
/// whose IPC handle is `ipc_handle`), write the descriptor into the claimed slot and publish it.  `out` gets the
/// pack's plan and sizes.
bool handoff_device_publish(HandoffArena& arena, const HandoffClaim& claim, const ConversationView& view,
                            const SessionState& session, const ConversationStageSet& stages, const ModelGeometry& g,
                            const QsaState& draft, const WireIdentity& identity, uint8_t* device_buffer,
                            uint64_t capacity, const uint8_t ipc_handle[64], uint64_t alloc_offset,
                            WireEncoded& out, std::string& error);

/// Decode side: the imported peer allocations, opened once each and closed with the cache.
class DevicePayloadImports {
public:
    explicit DevicePayloadImports(int device) : device_(device) {}
    ~DevicePayloadImports();
    DevicePayloadImports(const DevicePayloadImports&) = delete;
    DevicePayloadImports& operator=(const DevicePayloadImports&) = delete;
    /// The payload a descriptor names, mapped into this device's address space.
    bool map(const HandoffDeviceDescriptor& d, const uint8_t** payload, std::string& error);
    int device() const { return device_; }

private:
    int device_;
    std::map<std::string, void*> opened_;   // key: the 64 handle bytes
};

/// Decode side, after read_slot(): mount the session a descriptor points at (conversation_wire_mount_device on the
/// peer's HBM).  `expect` is checked against the payload header as in conversation_wire_decode.
ConversationRestore handoff_device_mount(const HandoffPayload& slot, DevicePayloadImports& imports,
                                         SessionState& session, const ConversationStageSet& stages,
                                         const ModelGeometry& g, const QsaState& draft, const WireExpect& expect,
                                         SavedConversation& meta, WireDecoded& info, std::string& error);

}  // namespace strata::core
