// kv_stream_detail.h - status-returning forms of the block movers (internal to libstrata_kv.so).  The public
// strata::kernels functions (include/strata_kv/kv_stream.hpp) wrap these and end the process on a CUDA failure
// like the reference's; the snapshot layer calls these and reports the failure instead.
#pragma once

#include "strata_kv/kv_stream.hpp"

#include <cuda_runtime.h>

namespace skv {

int stream_reset(const strata::kernels::KvStreamMap& m, cudaStream_t stream);
int ring_table(int32_t* table, int64_t n_blocks, int64_t n_slots, cudaStream_t stream);
int ring_restore(const strata::kernels::QsaAttnPools& slots, const strata::kernels::KvHostPools& host, int fmt,
                 int64_t b0, int64_t b1, int64_t n_slots, const strata::kernels::QsaShapes& s, cudaStream_t stream);
int stage_from_host(const strata::kernels::QsaAttnPools& stage, const strata::kernels::KvHostPools& host, int fmt,
                    int64_t n_blocks, const strata::kernels::QsaShapes& s, cudaStream_t stream);
int stream_resolve(const strata::kernels::KvStreamMap& m, const strata::kernels::QsaAttnPools& slots,
                   const strata::kernels::KvHostPools& host, int fmt, const int32_t* ids, const int32_t* steps,
                   int64_t n_q, int64_t cap, const strata::kernels::QsaShapes& s, cudaStream_t stream);

}  // namespace skv
