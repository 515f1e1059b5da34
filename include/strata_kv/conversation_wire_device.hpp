// include/strata_kv/conversation_wire_device.hpp - the SR4H payload packed straight from device state.
//
// The reference parks a conversation in two passes: conversation_snapshot_save copies every buffer from the GPU
// into a host image, then conversation_wire_encode copies the image again into the payload
// (include/strata/core/conversation_wire.hpp:24-81 for the format).  This pack produces the SAME bytes in one
// pass: the header and record stream are built on the host from the session's metadata, and every blob (each
// layer's K/V through its page table, indexer rows, running state) is gathered by the sm_100a copy kernels
// straight into its 64-byte-aligned place in the blob pool.  The result decodes with conversation_wire_decode
// (this build's or the reference's) and equals conversation_wire_encode(conversation_snapshot_save(...)) byte
// for byte.
//
// Destination: host memory (pinned for full PCIe speed; the pool goes down as one device-to-host copy per run of
// blobs that share a device), or device memory on the device that holds every device-resident blob (for a
// payload that then moves over NVLink or CUDA IPC as one contiguous buffer).  The mount side,
// conversation_wire_mount_device, takes such a device payload (a peer's, through CUDA IPC) straight into the
// decode session's pools.
#pragma once

#include "strata_kv/conversation_snapshot.hpp"
#include "strata_kv/conversation_wire.hpp"

#include <string>

namespace strata::core {

struct WireDeviceOptions {
    /// Fold the FNV-1a over the written payload into WireEncoded::payload_hash.  FNV-1a is a sequential chain,
    /// so this is a host pass over the payload; false leaves payload_hash 0.  Ignored (0) for a device target.
    bool hash = true;
    int max_checkpoint_depth = kWireMaxCheckpointDepth;
};

/// Validates the session exactly as conversation_snapshot_save would and plans its payload (plan.total_bytes is
/// the destination size a pack needs).  Nothing moves.
bool conversation_wire_pack_plan(const ConversationView& view, const SessionState& session,
                                 const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                 WirePlan& plan, std::string& error, const WireDeviceOptions& options = {});
bool conversation_wire_pack_plan(const ConversationView& view, const SessionState& session, const ModelGeometry& g,
                                 const QsaState& draft, WirePlan& plan, std::string& error,
                                 const WireDeviceOptions& options = {});

/// Packs the live session into `dst` (`capacity` bytes, at least plan.total_bytes).  On failure nothing of the
/// session changes and `dst` holds no valid payload.
bool conversation_wire_pack_device(const ConversationView& view, const SessionState& session,
                                   const ConversationStageSet& stages, const ModelGeometry& g, const QsaState& draft,
                                   const WireIdentity& identity, uint8_t* dst, uint64_t capacity, WirePlan& plan,
                                   WireEncoded& out, std::string& error, const WireDeviceOptions& options = {});
bool conversation_wire_pack_device(const ConversationView& view, const SessionState& session, const ModelGeometry& g,
                                   const QsaState& draft, const WireIdentity& identity, uint8_t* dst,
                                   uint64_t capacity, WirePlan& plan, WireEncoded& out, std::string& error,
                                   const WireDeviceOptions& options = {});

/// Mounts a session straight from an SR4H payload that lies in DEVICE memory - this device's, or a peer GPU's
/// mapped through CUDA IPC (the prefill instance's packed payload on the same node).  The header and records are
/// copied to the host and decoded with every check of conversation_wire_decode except the payload hash (the blobs
/// are never read by the host); the whole image is validated against the session exactly as
/// conversation_snapshot_restore validates it; then every blob goes from the payload to its place - K/V through
/// the destination layer's table, the running state, the draft, the layer-split stages - by the copy kernels
/// (NVLink loads for a peer payload), with the streamed / ring residency fix-ups of a mount.  `meta` receives the
/// image's metadata and its retained checkpoints (host copies); its K/V buffers and live running state stay empty,
/// because their bytes went to the device.  Returns invalid (nothing written) or transfer_failed like
/// conversation_snapshot_restore.
ConversationRestore conversation_wire_mount_device(const uint8_t* payload, uint64_t bytes, SessionState& session,
                                                   const ConversationStageSet& stages, const ModelGeometry& g,
                                                   const QsaState& draft, const WireExpect& expect,
                                                   SavedConversation& meta, WireDecoded& info, std::string& error);
ConversationRestore conversation_wire_mount_device(const uint8_t* payload, uint64_t bytes, SessionState& session,
                                                   const ModelGeometry& g, const QsaState& draft,
                                                   const WireExpect& expect, SavedConversation& meta,
                                                   WireDecoded& info, std::string& error);

/// Host-clock phases of this thread's last successful conversation_wire_pack_device or
/// conversation_wire_mount_device, in milliseconds.  prepare: validation, planning, the header and record stream
/// (written, or read from the payload and decoded), and the wait for work already queued on the session's devices;
/// issue: enqueueing every copy (for a host destination the per-device copies are waited for here too); complete:
/// waiting for the device copies to land and reading the status word (for a host destination: the payload hash).
struct WireDevicePhases {
    double prepare_ms = 0, issue_ms = 0, complete_ms = 0, total_ms = 0;
};
WireDevicePhases conversation_wire_device_last_phases();

}  // namespace strata::core
