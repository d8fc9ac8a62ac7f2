// step.cuh — the fused decode tick (replaces delta_step, src/delta/recurrent.rs:41-99).
//
// One pass over the state: each CTA owns a [dk x CW] column tile of one head's
// fp32 state S, keeps it in registers, and for each of the token's u
// micro-steps applies
//
//     S-  = exp(g) (.) S                 (key axis; micro-step 0 only)
//     u_j = w_j v_j - sum_i (b_i k_i) S-_ij
//     S   = S- + k u^T
//     y_j = sum_i (scale q_i) S_ij       (last micro-step, after the write)
//
// The readout needs no second pass: y = (sq^T S-) + (sq . k) u, so both
// column reductions run on the same registers before the write.  S is read
// once and written once per call (2 * dk * dv * 4 bytes per head), which is
// the HBM roofline of the tick; the reference's five separate tensor ops
// touch it about five times.
//
// Thread layout: TPR = CW / VEC threads cover one row's column tile with
// VEC-wide (float4) accesses; the 128 threads cover RPP = 128 / TPR rows per
// pass and NP passes cover dk <= NP * RPP.  Column sums reduce with warp
// shuffles across the rows of a warp, then across the 4 warps in shared memory.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

// Phase timestamps for performance work (a timing build defines DC_STEP_MARK(id); a no-op here).
#ifndef DC_STEP_MARK
#define DC_STEP_MARK(id)
#endif

namespace dc {

constexpr int kStepThreads = 128;
constexpr int kMaxHouseholder = 8;
constexpr int kMaxDk = 256;

template <int VEC>
struct VecF;
template <>
struct VecF<4> {
    __device__ __forceinline__ static void load(float *dst, const float *src) {
        float4 t = *reinterpret_cast<const float4 *>(src);
        dst[0] = t.x; dst[1] = t.y; dst[2] = t.z; dst[3] = t.w;
    }
    __device__ __forceinline__ static void store(float *dst, const float *src) {
        *reinterpret_cast<float4 *>(dst) = make_float4(src[0], src[1], src[2], src[3]);
    }
};
template <>
struct VecF<1> {
    __device__ __forceinline__ static void load(float *dst, const float *src) { dst[0] = *src; }
    __device__ __forceinline__ static void store(float *dst, const float *src) { *dst = src[0]; }
};

// Shared-memory bytes for one CTA of the step kernel.
__host__ __device__ inline size_t step_smem_bytes(int dk, int u, int cw) {
    // kk[u][dk], ke[u][dk], decay[dk], sq[dk], wv[u][cw], red[2][4][2][cw], sqk
    return sizeof(float) * ((size_t)2 * u * dk + 2 * dk + (size_t)u * cw + 2 * 4 * 2 * cw + 4);
}

template <typename TI, typename TG, typename TO, int VEC, int CW, int NP>
__global__ void __launch_bounds__(kStepThreads) step_kernel(CoreParams p) {
    constexpr int TPR = CW / VEC;             // threads per row
    constexpr int RPP = kStepThreads / TPR;   // rows per pass
    static_assert(32 % TPR == 0, "a row's threads must sit inside one warp");

    extern __shared__ float smem[];
    const int dk = (int)p.dk, dv = (int)p.dv, u = p.u;
    float *kk = smem;                 // [u][dk]   k
    float *ke = kk + u * dk;          // [u][dk]   erase (.) k
    float *decay = ke + u * dk;       // [dk]      exp(g)
    float *sq = decay + dk;           // [dk]      scale * q
    float *wv = sq + dk;              // [u][CW]   write (.) v for this column tile
    float *red = wv + u * CW;         // [2][4][2][CW] per-warp column partials
    float *sqk = red + 2 * 4 * 2 * CW;

    const int64_t bh = blockIdx.x;
    const int64_t b = bh / p.heads, h = bh % p.heads;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cv = tid % TPR, r0 = tid / TPR;
    const int col_base = blockIdx.y * CW;
    const int col = col_base + cv * VEC;
    const bool col_ok = col < dv;  // VEC divides dv whenever VEC > 1
    const TI *q = static_cast<const TI *>(p.q);
    const TI *k = static_cast<const TI *>(p.k);
    const TI *v = static_cast<const TI *>(p.v);
    const TG *erase = static_cast<const TG *>(p.erase);
    const TG *write = static_cast<const TG *>(p.write);
    const TG *g = static_cast<const TG *>(p.g);
    const int64_t H = p.heads;
    const int64_t qrow = b * p.q_bstride * H + h;  // row of q, g and y
    const bool one = u == 1 && dk <= kStepThreads;

    // Consecutive ticks: the next tick's CTAs may be scheduled now; this tick reads nothing before the
    // previous kernel in the stream has finished (programmatic dependent launch, see the launcher).  The
    // token's input lines are only pulled into L2 before that wait: a prefetch returns no data, and a
    // line the previous kernel is still writing is updated in L2 (the point of coherence) by that write.
    DC_STEP_MARK(0);
    ptx::launch_dependents();
    if (one) {
        const int64_t row = (b * p.kv_bstride) * H + h;
        if (tid < dk) {
            ptx::prefetch_l2(k + row * dk + tid);
            ptx::prefetch_l2(q + qrow * dk + tid);
            ptx::prefetch_l2(erase + row * p.ew + (p.ew == 1 ? 0 : tid));
            if (p.gw) ptx::prefetch_l2(g + qrow * p.gw + (p.gw == 1 ? 0 : tid));
        }
        if (tid < CW && col_base + tid < dv) {
            ptx::prefetch_l2(v + row * dv + col_base + tid);
            ptx::prefetch_l2(write + row * p.ww + (p.ww == 1 ? 0 : col_base + tid));
        }
    }
    ptx::grid_dependency_wait();
    DC_STEP_MARK(1);

    // ---- the state tile into registers (issued first: the long-latency loads) ----
    float s[NP][VEC];
    const float *S_in = p.state_in + bh * (int64_t)dk * dv;
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) {
        const int row = r0 + pp * RPP;
        if (row < dk && col_ok) {
            VecF<VEC>::load(s[pp], S_in + (int64_t)row * dv + col);
        } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) s[pp][e] = 0.f;
        }
    }

    // ---- this token's inputs into shared memory ----
    if (one) {
        // One micro-step: thread i < dk takes key channel i, thread j < CW value column j.  Every load is
        // issued before any shared-memory write, so the tick pays one global latency instead of one per
        // input loop.
        const int64_t row = (b * p.kv_bstride) * H + h;
        const int c = col_base + tid;
        const bool kt = tid < dk, vt = tid < CW && c < dv;
        const float kv = kt ? ld(k + row * dk + tid) : 0.f;
        const float ev = kt ? ld(erase + row * p.ew + (p.ew == 1 ? 0 : tid)) : 0.f;
        const float gv = (kt && p.gw) ? ld(g + qrow * p.gw + (p.gw == 1 ? 0 : tid)) : 0.f;
        const float qv = kt ? ld(q + qrow * dk + tid) : 0.f;
        const float vv = vt ? ld(v + row * dv + c) : 0.f;
        const float wv_ = vt ? ld(write + row * p.ww + (p.ww == 1 ? 0 : c)) : 0.f;
        if (kt) {
            kk[tid] = kv;
            ke[tid] = kv * ev;
            decay[tid] = p.gw ? expf(gv) : 1.f;
            sq[tid] = p.scale * qv;
        }
        if (tid < CW) wv[tid] = vv * wv_;
    } else {
    for (int idx = tid; idx < u * dk; idx += kStepThreads) {
        const int m = idx / dk, i = idx % dk;
        const int64_t row = (b * p.kv_bstride + m) * H + h;  // [batch, u, heads, .]
        const float kv = ld(k + row * dk + i);
        const float ev = ld(erase + row * p.ew + (p.ew == 1 ? 0 : i));
        kk[idx] = kv;
        ke[idx] = kv * ev;
    }
    for (int i = tid; i < dk; i += kStepThreads) {
        decay[i] = p.gw ? expf(ld(g + qrow * p.gw + (p.gw == 1 ? 0 : i))) : 1.f;
        sq[i] = p.scale * ld(q + qrow * dk + i);
    }
    for (int idx = tid; idx < u * CW; idx += kStepThreads) {
        const int m = idx / CW, j = idx % CW, c = col_base + j;
        float val = 0.f;
        if (c < dv) {
            const int64_t row = (b * p.kv_bstride + m) * H + h;
            val = ld(v + row * dv + c) * ld(write + row * p.ww + (p.ww == 1 ? 0 : c));
        }
        wv[idx] = val;
    }
    }
    __syncthreads();
    DC_STEP_MARK(2);
    // (scale q) . k of the last micro-step: the readout's share of the write.
    if (warp == 0) {
        float acc = 0.f;
        for (int i = lane; i < dk; i += 32) acc += sq[i] * kk[(u - 1) * dk + i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) sqk[0] = acc;
    }

    TO *y = static_cast<TO *>(p.y);
    for (int m = 0; m < u; ++m) {
        const bool last = (m == u - 1);
        if (m == 0 && p.gw) {
#pragma unroll
            for (int pp = 0; pp < NP; ++pp) {
                const int row = r0 + pp * RPP;
                const float a = row < dk ? decay[row] : 0.f;
#pragma unroll
                for (int e = 0; e < VEC; ++e) s[pp][e] *= a;
            }
        }
        float ret[VEC], qs[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) ret[e] = qs[e] = 0.f;
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
            const int row = r0 + pp * RPP;
            if (row < dk) {
                const float kr = ke[m * dk + row];
                const float qr = last ? sq[row] : 0.f;
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    ret[e] = fmaf(kr, s[pp][e], ret[e]);
                    qs[e] = fmaf(qr, s[pp][e], qs[e]);
                }
            }
        }
#pragma unroll
        for (int off = TPR; off < 32; off <<= 1) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                ret[e] += __shfl_xor_sync(0xffffffffu, ret[e], off);
                qs[e] += __shfl_xor_sync(0xffffffffu, qs[e], off);
            }
        }
        float *buf = red + (m & 1) * (4 * 2 * CW);
        if (lane < TPR) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                buf[(warp * 2 + 0) * CW + cv * VEC + e] = ret[e];
                buf[(warp * 2 + 1) * CW + cv * VEC + e] = qs[e];
            }
        }
        __syncthreads();
        float du[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            const int j = cv * VEC + e;
            float r = 0.f, qq = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                r += buf[(w * 2 + 0) * CW + j];
                qq += buf[(w * 2 + 1) * CW + j];
            }
            du[e] = wv[m * CW + j] - r;
            qs[e] = qq;
        }
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
            const int row = r0 + pp * RPP;
            const float kr = row < dk ? kk[m * dk + row] : 0.f;
#pragma unroll
            for (int e = 0; e < VEC; ++e) s[pp][e] = fmaf(kr, du[e], s[pp][e]);
        }
        if (last && r0 == 0 && col_ok) {
            const float c = sqk[0];
#pragma unroll
            for (int e = 0; e < VEC; ++e) st(y + qrow * dv + col + e, fmaf(c, du[e], qs[e]));
        }
    }

    DC_STEP_MARK(3);
    float *S_out = p.state_out + bh * (int64_t)dk * dv;
#pragma unroll
    for (int pp = 0; pp < NP; ++pp) {
        const int row = r0 + pp * RPP;
        if (row < dk && col_ok) VecF<VEC>::store(S_out + (int64_t)row * dv + col, s[pp]);
    }
    DC_STEP_MARK(4);
}

}  // namespace dc
