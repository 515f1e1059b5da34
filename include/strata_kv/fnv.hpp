// include/strata_kv/fnv.hpp - FNV-1a 64, the content hash of hand-off payloads and arena slots.
#pragma once

#include <cstdint>

namespace strata::core {

/// The public FNV-1a 64 algorithm (offset basis 1469598103934665603, prime 1099511628211) over [p, p + n),
/// continuing from `seed`; the reference's engine uses the same function (src/core/pinned.cu:594-601).
uint64_t fnv1a64(const uint8_t* p, uint64_t n, uint64_t seed = 1469598103934665603ull);

}  // namespace strata::core
