// out_norm.cuh — the per-head output normalisation that follows the delta rule's read-out
// (src/common/norm.rs:106-144, OutNorm): over each (batch, token, head) row of y [.., dv],
//
//   gated:  out = y / sqrt(mean(y^2) + eps) * w (.) silu(gate),   silu(x) = x sigma(x) (fast exponential
//           and division intrinsics: a few ulp)
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
                    if (Gt) v *= __fdividef(g[q][e], 1.f + __expf(-g[q][e]));
                    st(O + r * dv + d, v);
                }
            }
        }
    }
}

// 16-byte vector access: VEC = 16 / sizeof(T) elements.
__device__ __forceinline__ void load16(const float *p, float (&v)[4]) {
    const float4 t = *reinterpret_cast<const float4 *>(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
}
__device__ __forceinline__ void load16(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 t = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
        v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
}
template <int N>
__device__ __forceinline__ void store_vec(float *p, const float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 4) *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}
template <int N>
__device__ __forceinline__ void store_vec(__nv_bfloat16 *p, const float (&v)[N]) {
    uint32_t w[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
    if constexpr (N == 8) *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    else *reinterpret_cast<uint2 *>(p) = make_uint2(w[0], w[1]);
}

// The same normalisation with 16-byte loads and stores: a row is LPR lanes of VEC = 16 / sizeof(TI)
// consecutive elements each (dv = LPR VEC, LPR a power of two <= 32), a warp holds 32 / LPR rows per slot
// and kSlots slots per iteration, all of them loaded before the first use.  Needs 16-byte-aligned rows.
constexpr int kSlots = 4;
// slots per warp iteration by input width: 2-byte inputs hold twice the elements per 16 bytes, so two
// slots keep their registers (and occupancy) in line with 4-byte inputs at four
template <typename TI> __host__ __device__ constexpr int slots_for() { return sizeof(TI) == 2 ? 2 : kSlots; }

template <typename TI, typename TO, int LPR>
__global__ void __launch_bounds__(kThreads) out_norm_vec_kernel(const Params p) {
    constexpr int VEC = 16 / sizeof(TI), RPS = 32 / LPR, NS = slots_for<TI>();
    const int lane = threadIdx.x & 31, sub = lane % LPR, srow = lane / LPR, col = sub * VEC;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
    const int dv = p.dv;
    const TI *Y = static_cast<const TI *>(p.y), *Gt = static_cast<const TI *>(p.gate);
    const TI *Gb = Gt ? Gt : Y;  // the gate's loads read y when there is no gate (and are not used)
    TO *O = static_cast<TO *>(p.out);
    float w[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) w[e] = p.weight[col + e];
    const float inv_dv = 1.f / (float)dv;
    for (int64_t r0 = ((int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * (RPS * NS); r0 < p.rows;
         r0 += warps * (RPS * NS)) {
        float y[NS][VEC], g[NS][VEC];
#pragma unroll
        for (int q = 0; q < NS; ++q) {
            const int64_t r = r0 + q * RPS + srow;
            const int64_t o = (r < p.rows ? r : 0) * dv + col;
            load16(Y + o, y[q]);
            load16(Gb + o, g[q]);
        }
#pragma unroll
        for (int q = 0; q < NS; ++q) {
            const int64_t r = r0 + q * RPS + srow;
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < VEC; ++e) ss = fmaf(y[q][e], y[q][e], ss);
#pragma unroll
            for (int o = LPR / 2; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = rsqrtf(fmaf(ss, inv_dv, p.eps));
            float v[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                v[e] = y[q][e] * inv * w[e];
                if (Gt) v[e] *= __fdividef(g[q][e], 1.f + __expf(-g[q][e]));
            }
            if (r < p.rows) store_vec(O + r * dv + col, v);
        }
    }
}

}  // namespace onorm
}  // namespace dc
