// chunk_tc.cuh — tensor-core (tcgen05) chunkwise WY prefill for bf16 inputs.
#pragma once

#include "common.cuh"

namespace dc {

// Whether the tensor-core kernel serves this request.
inline bool tc_applies(int64_t dk, int64_t dv, int32_t in_dtype, uint32_t flags) {
    (void)dk; (void)dv; (void)in_dtype; (void)flags;
    return false;
}

inline int tc_last_error() { return 0; }

inline int launch_chunk_tc(const CoreParams &, int32_t, int32_t, cudaStream_t) { return 5; }

}  // namespace dc
