// wire_detail.hpp - the SR4H encoder's plan and record passes, reusable on a shape image (internal).
//
// A shape image is a SavedConversation whose metadata (geometry, ids, image keys, extents, nesting) is real but
// whose byte buffers may be empty: `size_of(buffer, its size())` supplies the byte count each buffer stands for.
// The device-side pack builds one from live device state, plans the payload with it, writes the header and
// records on the host and gathers every blob straight from the device pools into its place in the blob pool.
#pragma once

#include "strata_kv/conversation_wire.hpp"

#include <functional>
#include <string>
#include <unordered_map>
#include <vector>

namespace strata::core::wire_detail {

/// key = the ConversationBuffer or std::vector<uint8_t> inside the image; real = its size().
using SizeOf = std::function<uint64_t(const void* key, uint64_t real)>;

/// One non-empty blob in pool order: `rel` is its offset inside the blob pool.
struct PlannedBlob {
    const void* key = nullptr;
    uint64_t rel = 0;
    uint64_t bytes = 0;
};

bool plan(const SavedConversation& image, int max_depth, const SizeOf& size_of, WirePlan& plan,
          std::vector<PlannedBlob>& blobs, std::string& error);

/// Writes bytes [0, plan.blob_pool_off) of the payload - the header record, the record stream and the zero pad
/// up to the blob pool - into `out`.
bool write_records(const SavedConversation& image, const WireIdentity& identity, const WirePlan& plan,
                   const std::vector<PlannedBlob>& blobs, const SizeOf& size_of, uint8_t* out, std::string& error);

/// Where a blob lies in a payload.
struct BlobAt {
    uint64_t off = 0;
    uint64_t bytes = 0;
};
using BlobTable = std::unordered_map<const void*, BlobAt>;

/// Decode the record stream of `source` into a SHAPE image, in place: every metadata field real, every blob left
/// empty and recorded in `blobs` under the address of its buffer or vector inside `image`.  Every check of a full
/// decode runs except the payload hash; no blob byte is read, so `source` only has to serve the records (its size
/// is the whole payload's).
bool decode_shape(const WireSource& source, SavedConversation& image, WireDecoded& info, const WireExpect& expect,
                  BlobTable& blobs, std::string& error);

}  // namespace strata::core::wire_detail
