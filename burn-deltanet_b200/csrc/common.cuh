// common.cuh — element access and launch parameters shared by the delta-rule kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dc {

__device__ __forceinline__ float ld(const float *p) { return *p; }
__device__ __forceinline__ float ld(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st(float *p, float v) { *p = v; }
__device__ __forceinline__ void st(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// Everything a delta-rule kernel reads, in the reference's layouts
// (src/delta/path.rs:120-141).  `seq` counts tokens; k, v, erase and write
// carry seq * u rows (the micro-step fold), q and g carry seq rows.
struct CoreParams {
    int64_t batch, seq, heads, dk, dv;
    int32_t u;                 // n_householder
    int32_t ew, ww, gw;        // gate widths: erase {1, dk}, write {1, dv}, g {0, 1, dk}
    // Rows between consecutive batches, for the decode tick only: of k, v,
    // erase, write (u for one token; seq * u when the tick walks a sequence in
    // place) and of q, g, y (1 for one token; seq for a sequence).
    int64_t kv_bstride, q_bstride;
    float scale;
    int32_t stall;             // test hook (DC_FLAG_TEST_STALL): issue no tile loads
    const void *q, *k, *v, *erase, *write, *g;
    const float *state_in;
    void *y;
    float *state_out;
    // The plain output norm fused into the read-out (dc_chunk_fwd_out_norm; the fused tensor-core kernel
    // only): y <- y / sqrt(mean(y^2) + norm_eps) * norm_weight over each row of dv values.
    int32_t norm;              // 0: y as is; 1: normalised
    float norm_eps;
    const float *norm_weight;  // [dv] float32
};

}  // namespace dc
