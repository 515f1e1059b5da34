// handoff_device.cpp - the device descriptor a hand-off slot carries on one node
// (include/strata_kv/handoff_device.hpp).
#include "strata_kv/handoff_device.hpp"

#include "strata_kv.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

namespace strata::core {
namespace {

bool dfail(std::string& error, const std::string& why) {
    error = "device hand-off: " + why;
    return false;
}
void put64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t) (v >> (8 * i));
}
void put32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t) (v >> (8 * i));
}
uint64_t get64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= (uint64_t) p[i] << (8 * i);
    return v;
}
uint32_t get32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t) p[i] << (8 * i);
    return v;
}

// the record layout
constexpr size_t kOffVersion = 8, kOffHeaderBytes = 12, kOffHandle = 16, kOffAllocOffset = 80, kOffPayloadBytes = 88,
                 kOffDevice = 96, kOffBusId = 100, kOffGeom = 136, kOffPack = 144, kOffTokens = 152, kOffFnv = 160,
                 kOffEnd = 168;
static_assert(kOffBusId + 32 <= kOffGeom && kOffEnd <= kDeviceDescriptorBytes);

}  // namespace

void handoff_device_encode(const HandoffDeviceDescriptor& d, uint8_t out[kDeviceDescriptorBytes]) {
    std::memset(out, 0, kDeviceDescriptorBytes);
    std::memcpy(out, kDeviceDescriptorMagic, 8);
    put32(out + kOffVersion, kDeviceDescriptorVersion);
    put32(out + kOffHeaderBytes, (uint32_t) kDeviceDescriptorBytes);
    std::memcpy(out + kOffHandle, d.ipc_handle, 64);
    put64(out + kOffAllocOffset, d.alloc_offset);
    put64(out + kOffPayloadBytes, d.payload_bytes);
    put32(out + kOffDevice, (uint32_t) d.device);
    std::memcpy(out + kOffBusId, d.pci_bus_id, 31);
    put64(out + kOffGeom, d.geom_hash);
    put64(out + kOffPack, d.pack_hash);
    put64(out + kOffTokens, d.tokens);
    put64(out + kOffFnv, d.payload_fnv);
}

bool handoff_device_is_descriptor(const uint8_t* data, uint64_t bytes) {
    return data && bytes == kDeviceDescriptorBytes && std::memcmp(data, kDeviceDescriptorMagic, 8) == 0;
}

bool handoff_device_decode(const uint8_t* p, uint64_t bytes, HandoffDeviceDescriptor& d, std::string& error) {
    if (!p || bytes != kDeviceDescriptorBytes)
        return dfail(error, "a descriptor is " + std::to_string(kDeviceDescriptorBytes) + " bytes, not " +
                                std::to_string(bytes));
    if (std::memcmp(p, kDeviceDescriptorMagic, 8) != 0) return dfail(error, "not a device descriptor (bad magic)");
    if (get32(p + kOffVersion) != kDeviceDescriptorVersion)
        return dfail(error, "descriptor version " + std::to_string(get32(p + kOffVersion)) + "; this build reads 1");
    if (get32(p + kOffHeaderBytes) != kDeviceDescriptorBytes) return dfail(error, "descriptor header_bytes is not 256");
    for (size_t i = kOffEnd; i < kDeviceDescriptorBytes; ++i)
        if (p[i]) return dfail(error, "the descriptor's reserved bytes are not zero");
    if (p[kOffBusId + 31]) return dfail(error, "the descriptor's bus id is not terminated");
    HandoffDeviceDescriptor out;
    std::memcpy(out.ipc_handle, p + kOffHandle, 64);
    out.alloc_offset = get64(p + kOffAllocOffset);
    out.payload_bytes = get64(p + kOffPayloadBytes);
    out.device = (int32_t) get32(p + kOffDevice);
    std::memcpy(out.pci_bus_id, p + kOffBusId, 32);
    out.geom_hash = get64(p + kOffGeom);
    out.pack_hash = get64(p + kOffPack);
    out.tokens = get64(p + kOffTokens);
    out.payload_fnv = get64(p + kOffFnv);
    if (out.payload_bytes < kWireHeaderRecordBytes) return dfail(error, "the descriptor names a payload shorter than a header");
    if (out.alloc_offset % 256) return dfail(error, "the payload does not start on a 256-byte boundary of its allocation");
    d = out;
    return true;
}

bool handoff_device_publish(HandoffArena& arena, const HandoffClaim& claim, const ConversationView& view,
                            const SessionState& ss, const ConversationStageSet& stages, const ModelGeometry& g,
                            const QsaState& draft, const WireIdentity& identity, uint8_t* device_buffer,
                            uint64_t capacity, const uint8_t ipc_handle[64], uint64_t alloc_offset, WireEncoded& out,
                            std::string& error) {
    if (!device_buffer || !ipc_handle) return dfail(error, "no device buffer or no IPC handle");
    WirePlan plan;
    if (!conversation_wire_pack_device(view, ss, stages, g, draft, identity, device_buffer, capacity, plan, out, error))
        return false;
    HandoffDeviceDescriptor d;
    std::memcpy(d.ipc_handle, ipc_handle, 64);
    d.alloc_offset = alloc_offset;
    d.payload_bytes = out.bytes;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, device_buffer) != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
        (void) cudaGetLastError();
        return dfail(error, "the payload buffer is not device memory");
    }
    d.device = attr.device;
    if (cudaDeviceGetPCIBusId(d.pci_bus_id, (int) sizeof d.pci_bus_id - 1, attr.device) != cudaSuccess) {
        (void) cudaGetLastError();
        return dfail(error, "cannot name the payload's PCI bus id");
    }
    d.geom_hash = identity.geom_hash;
    d.pack_hash = identity.pack_hash;
    d.tokens = view.ids.size();
    uint8_t rec[kDeviceDescriptorBytes];
    handoff_device_encode(d, rec);
    return arena.write_payload(claim, 0, rec, sizeof rec, error) &&
           arena.publish(claim, d.tokens, sizeof rec, fnv1a64(rec, sizeof rec), error);
}

DevicePayloadImports::~DevicePayloadImports() {
    for (auto& [key, ptr] : opened_) (void) skv_ipc_close(ptr);
}

bool DevicePayloadImports::map(const HandoffDeviceDescriptor& d, const uint8_t** payload, std::string& error) {
    const std::string key(reinterpret_cast<const char*>(d.ipc_handle), 64);
    auto it = opened_.find(key);
    if (it == opened_.end()) {
        void* base = nullptr;
        if (skv_ipc_import(device_, d.ipc_handle, &base) != SKV_OK)
            return dfail(error, std::string("cannot import the payload's allocation (from ") + d.pci_bus_id +
                                    "): " + skv_last_error());
        it = opened_.emplace(key, base).first;
    }
    *payload = static_cast<const uint8_t*>(it->second) + d.alloc_offset;
    return true;
}

ConversationRestore handoff_device_mount(const HandoffPayload& slot, DevicePayloadImports& imports, SessionState& ss,
                                         const ConversationStageSet& stages, const ModelGeometry& g,
                                         const QsaState& draft, const WireExpect& expect, SavedConversation& meta,
                                         WireDecoded& info, std::string& error) {
    HandoffDeviceDescriptor d;
    if (!slot.valid() || !handoff_device_decode(slot.data, slot.payload_bytes, d, error))
        return ConversationRestore::invalid;
    if (expect.check_hashes && (d.geom_hash != expect.geom_hash || d.pack_hash != expect.pack_hash)) {
        dfail(error, "the descriptor's identity differs from this instance's");
        return ConversationRestore::invalid;
    }
    const uint8_t* payload = nullptr;
    if (!imports.map(d, &payload, error)) return ConversationRestore::invalid;
    return conversation_wire_mount_device(payload, d.payload_bytes, ss, stages, g, draft, expect, meta, info, error);
}

}  // namespace strata::core
