// out_norm.cuh — the per-head output normalisation that follows the delta rule's read-out
// (src/common/norm.rs:106-144, OutNorm): over each (batch, token, head) row of y [.., dv],
//
//   gated:  out = y / sqrt(mean(y^2) + eps) * w (.) silu(gate),   silu(x) = x sigma(x)
//   plain:  out = y / sqrt(mean(y^2) + eps) * w
//
// the RmsNormGated / RmsNorm modules of burn-stack (rev 984d42d3, not vendored in the reference tree; the
// gated form is the post-normalisation modulation norm.rs:108-113 describes).  fp32 arithmetic, bf16 or
// fp32 in and out.  One warp per row, two rows per warp in flight; HBM-bound (reads y and gate once,
// writes out once).
#pragma once

#include "common.cuh"

namespace dc {
namespace onorm {

constexpr int kThreads = 256;
constexpr int kRowsPerWarp = 2;
constexpr int kMaxPer = 8;  // dv <= 32 * kMaxPer (kernels for PER = 4 and 8 elements per lane)

struct Params {
    int64_t rows;
    int32_t dv;
    float eps;
    const void *y, *gate;  // [rows, dv]; gate may be null (plain)
    const float *weight;   // [dv]
    void *out;             // [rows, dv]
};

template <typename TI, typename TO, int PER>
__global__ void __launch_bounds__(kThreads) out_norm_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
    const int dv = p.dv, per = (dv + 31) / 32;
    const TI *Y = static_cast<const TI *>(p.y), *Gt = static_cast<const TI *>(p.gate);
    TO *O = static_cast<TO *>(p.out);
    const TI *Gb = Gt ? Gt : Y;  // the gate's loads read y when there is no gate (and are not used)
    float w[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) w[e] = (e < per && lane + 32 * e < dv) ? p.weight[lane + 32 * e] : 0.f;
    const float inv_dv = 1.f / (float)dv;
    for (int64_t r0 = ((int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * kRowsPerWarp; r0 < p.rows;
         r0 += warps * kRowsPerWarp) {
        float y[kRowsPerWarp][PER], g[kRowsPerWarp][PER];
        // every load of both rows first, unconditional (an element past the row reads element 0) so that
        // they all issue before the first use
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q) {
            const int64_t r = r0 + q;
            const bool in = r < p.rows;
#pragma unroll
            for (int e = 0; e < PER; ++e) {
                const int d = lane + 32 * e;
                const bool ok = in && e < per && d < dv;
                const int64_t o = ok ? r * dv + d : 0;
                const float yv = ld(Y + o), gv = ld(Gb + o);
                y[q][e] = ok ? yv : 0.f;
                g[q][e] = gv;
            }
        }
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q) {
            const int64_t r = r0 + q;
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < PER; ++e) ss = fmaf(y[q][e], y[q][e], ss);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = rsqrtf(fmaf(ss, inv_dv, p.eps));
            if (r >= p.rows) continue;
#pragma unroll
            for (int e = 0; e < PER; ++e) {
                const int d = lane + 32 * e;
                if (e < per && d < dv) {
                    float v = y[q][e] * inv * w[e];
                    if (Gt) v *= g[q][e] / (1.f + expf(-g[q][e]));
                    st(O + r * dv + d, v);
                }
            }
        }
    }
}

}  // namespace onorm
}  // namespace dc
