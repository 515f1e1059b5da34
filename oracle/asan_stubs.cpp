// oracle/asan_stubs.cpp - TEST INFRASTRUCTURE for the sanitizer builds of the reference's host-only suites.
//
// The snapshot layer (conversation_snapshot.cpp) calls two internals of libstrata_kv.so that the library does not
// export: the streamed-layer reset mover and the block-pool registry.  The host-only suites stop at validation and
// never reach a transfer, so a call to the mover here is a harness error and aborts; no pool is registered in
// these programs, so the registry answers "not in a block pool" (identity addressing).
#include "kv_stream_detail.h"

#include <cstdio>
#include <cstdlib>

namespace skv {

int stream_reset(const strata::kernels::KvStreamMap&, cudaStream_t) {
    std::fprintf(stderr, "asan_stubs: stream_reset reached from a host-only suite\n");
    std::abort();
}

bool in_block_pool(const void*) { return false; }

}  // namespace skv
