// bwd_recurrent.cuh — the backward of the delta-rule core (the gradients the reference's custom
// autodiff node returns, src/delta/chunk_recalculated/combined_backward.rs:72-190), walked token by
// token on the CUDA cores in fp32.
//
// The forward it differentiates is the recurrence (src/delta/recurrent.rs:41-142), micro-step n of
// token t = n / u (n_householder u, the fold of src/delta_product/delta_product.rs:178-228):
//
//   S-  = diag(alpha_n) S_{n-1}        alpha_n = e^{g_t} on micro-step 0 (key axis), else 1
//   u_n = w_n (.) v_n - S-^T (b_n (.) k_n)
//   S_n = S- + k_n u_n^T
//   y_t = S_n^T (s q_t)                 on micro-step u - 1
//
// and, for L = <y, dy> + <S_final, dS_final>, one step back with dS = dL/dS_n:
//
//   (read-out step)  dS += (s q_t) dy_t^T;   dq_t = s S_n dy_t = s (S- dy_t + k_n (u_n . dy_t))
//   du   = dS^T k_n
//   dk_n = dS u_n - b_n (.) (S- du);        db_n = -k_n (.) (S- du)
//   dv_n = w_n (.) du;                      dw_n = v_n (.) du
//   dS-  = dS - (b_n (.) k_n) du^T
//   (decay step)     dg_t = sum_j dS-_ij S-_ij;   dS_{n-1} = diag(alpha_n) dS-
//
// with gate gradients summed over the broadcast axis when a gate has width 1.  The chunkwise
// backward of the reference computes the same derivatives in a different order; this is their
// definition, and every gradient element is written exactly once (no atomics: deterministic).
//
// The reverse walk needs S-_n at every step, and running the recurrence backwards would divide by
// alpha.  So the kernel stores the state at the start of every block of kBlk micro-steps (a forward
// pass), then for each block from the last: replays the block forward from its checkpoint, keeping
// each step's S- in a scratch, and walks the block back.  One CTA (256 threads) per (batch, head,
// slice of 32 value columns), its slices of S and dS in shared memory (~42 KB at dk = 128: several
// CTAs per SM hide each other's latency); dk, dv <= 128.
#pragma once

#include "common.cuh"

namespace dc {
namespace bwd {

constexpr int kThreads = 256;
constexpr int kBlk = 16;    // micro-steps per checkpoint block
constexpr int kMaxD = 128;  // dk, dv
constexpr int kSlice = 32;  // value columns per CTA

// The value columns of S evolve independently (recurrent.rs:41-99 acts on S column by column); only
// the gradients that sum over them (dq, dk, d_erase, d_g, and d_write at width 1) couple the slices.
// With several slices each CTA writes its share of those into a partial buffer [slice][...], and
// reduce_partials adds the slices up in a fixed order (deterministic); with one slice they go straight
// to the outputs.
struct Params {
    CoreParams f;           // the forward call: dims, widths, scale, q, k, v, erase, write, g, state_in
    const float *dy;        // [batch, seq, heads, dv]
    const float *dS_final;  // [batch, heads, dk, dv] or null (zero)
    float *dv, *dw_full;    // [batch, seq*u, heads, dv]: dv, and d_write when write_w == dv
    float *dS0;             // [batch, heads, dk, dv]
    // column-summed gradients: base and the stride between slices (0 with one slice)
    float *dq, *dk, *de, *dg, *dw1;
    int64_t sq, sk, se, sg, sw1;
    float *ckpt;            // [batch*heads][nslice][nblk][dk][kSlice]
    float *scratch;         // [batch*heads][nslice][kBlk][dk][kSlice]
    int64_t nblk;
    int32_t nslice;
};

// Shared-memory layout (floats): S and dS ([dk][kSlice + 1]), then the step's vectors and the partial
// sums of the reductions.
struct Layout {
    int dk, P;
    int S, dS, kx, bk, ex, al, qs, r1, r2, vx, wx, uu, du, dy, red, scal, total;
    __host__ __device__ explicit Layout(int dk_) : dk(dk_), P(kSlice + 1) {
        S = 0;
        dS = S + dk * P;
        kx = dS + dk * P;
        bk = kx + kMaxD;
        ex = bk + kMaxD;
        al = ex + kMaxD;
        qs = al + kMaxD;
        r1 = qs + kMaxD;
        r2 = r1 + kMaxD;
        vx = r2 + kMaxD;
        wx = vx + kSlice;
        uu = wx + kSlice;
        du = uu + kSlice;
        dy = du + kSlice;
        red = dy + kSlice;        // [kThreads]
        scal = red + kThreads;    // [8] block-reduction slots
        total = scal + 32;
    }
};

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads) bwd_recurrent_kernel(const Params p) {
    extern __shared__ float sm[];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, u = f.u;
    const Layout L(dk);
    const int P = L.P;
    float *S = sm + L.S, *dS = sm + L.dS;
    float *kx = sm + L.kx, *bk = sm + L.bk, *ex = sm + L.ex, *al = sm + L.al, *qs = sm + L.qs;
    float *r1 = sm + L.r1, *r2 = sm + L.r2, *vx = sm + L.vx, *wx = sm + L.wx, *uu = sm + L.uu;
    float *du = sm + L.du, *dyv = sm + L.dy, *red = sm + L.red, *scal = sm + L.scal;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh % f.heads;
    const int sl = blockIdx.y, c0 = sl * kSlice, ws = (dv - c0) < kSlice ? (dv - c0) : kSlice;  // this slice's columns
    const int64_t N = f.seq * u;  // micro-steps
    const int64_t selems = (int64_t)dk * kSlice;
    const bool gated = f.gw > 0;
    // Element sweeps over a [dk][ws] matrix: thread (er, ec) takes column ec of rows er, er + kRows, ...
    constexpr int kRows = kThreads / kSlice;
    const int er = tid / kSlice, ec = tid % kSlice;
    const bool sweeper = ec < ws;

    const TI *Q = static_cast<const TI *>(f.q), *K = static_cast<const TI *>(f.k), *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *W = static_cast<const TG *>(f.write), *G = static_cast<const TG *>(f.g);
    auto row_n = [&](int64_t n) { return (b * N + n) * f.heads + h; };       // micro-step rows
    auto row_t = [&](int64_t t) { return (b * f.seq + t) * f.heads + h; };   // token rows

    // ---- block-wide helpers (all threads; each ends with a barrier) ----
    // out[j] = sum_i M[i][j] x[i], j < ws: kRows row groups, then their partial sums added
    auto col_product = [&](const float *M, const float *x, float *out) {
        float a0 = 0.f, a1 = 0.f;
        if (sweeper) {
            int i = er;
            for (; i + kRows < dk; i += 2 * kRows) {
                a0 = fmaf(M[i * P + ec], x[i], a0);
                a1 = fmaf(M[(i + kRows) * P + ec], x[i + kRows], a1);
            }
            if (i < dk) a0 = fmaf(M[i * P + ec], x[i], a0);
        }
        red[tid] = a0 + a1;
        __syncthreads();
        if (tid < ws) {
            float sum = 0.f;
#pragma unroll
            for (int g = 0; g < kRows; ++g) sum += red[g * kSlice + tid];
            out[tid] = sum;
        }
        __syncthreads();
    };
    // out[i] = sum_{j < ws} M[i][j] x[j]   (x == nullptr: sum_j M[i][j] M2[i][j])
    auto row_product = [&](const float *M, const float *x, const float *M2, float *out) {
        const int i = tid & 127, half = tid >> 7, hc = (ws + 1) >> 1;
        const int c0h = half * hc, c1h = half ? ws : hc;
        if (i < dk) {
            float a0 = 0.f, a1 = 0.f;
            int j = c0h;
            if (x) {
                for (; j + 1 < c1h; j += 2) {
                    a0 = fmaf(M[i * P + j], x[j], a0);
                    a1 = fmaf(M[i * P + j + 1], x[j + 1], a1);
                }
                if (j < c1h) a0 = fmaf(M[i * P + j], x[j], a0);
            } else {
                for (; j + 1 < c1h; j += 2) {
                    a0 = fmaf(M[i * P + j], M2[i * P + j], a0);
                    a1 = fmaf(M[i * P + j + 1], M2[i * P + j + 1], a1);
                }
                if (j < c1h) a0 = fmaf(M[i * P + j], M2[i * P + j], a0);
            }
            red[half * kMaxD + i] = a0 + a1;
        }
        __syncthreads();
        if (tid < dk) out[tid] = red[tid] + red[kMaxD + tid];
        __syncthreads();
    };
    // M[i][j] += sign a[i] b[j]
    auto rank1 = [&](float *M, const float *a, const float *bvec, float sign) {
        if (sweeper) {
            const float bj = sign * bvec[ec];
            for (int i = er; i < dk; i += kRows) M[i * P + ec] = fmaf(a[i], bj, M[i * P + ec]);
        }
        __syncthreads();
    };
    auto scale_rows = [&](float *M, const float *a) {
        if (sweeper)
            for (int i = er; i < dk; i += kRows) M[i * P + ec] *= a[i];
        __syncthreads();
    };
    // sum over the block of one value per thread
    auto block_sum = [&](float v) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) scal[warp] = v;
        __syncthreads();
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) s += scal[w];
        __syncthreads();
        return s;
    };
    // this slice of a [dk][dv] state in global memory <-> shared; checkpoints are [dk][kSlice]
    auto store_full = [&](const float *M, float *dst) {
        if (sweeper)
            for (int i = er; i < dk; i += kRows) dst[i * dv + c0 + ec] = M[i * P + ec];
    };
    auto load_full = [&](float *M, const float *src) {
        if (sweeper)
            for (int i = er; i < dk; i += kRows) M[i * P + ec] = src ? src[i * dv + c0 + ec] : 0.f;
        __syncthreads();
    };
    auto store_local = [&](const float *M, float *dst) {
        if (sweeper)
            for (int i = er; i < dk; i += kRows) dst[i * kSlice + ec] = M[i * P + ec];
    };
    auto load_local = [&](float *M, const float *src) {
        if (sweeper)
            for (int i = er; i < dk; i += kRows) M[i * P + ec] = src[i * kSlice + ec];
        __syncthreads();
    };

    // The inputs of micro-step n into the shared vectors: k, b (.) k, the erase row (width-expanded),
    // the decay alpha (1 unless micro-step 0 of a gated token), and this slice's v, w.
    auto load_step = [&](int64_t n) {
        const int64_t t = n / u, m = n % u;
        const int64_t rn = row_n(n);
        const bool decay = gated && m == 0;
        if (tid < dk) {
            const float kk = ld(K + rn * dk + tid);
            const float e = ld(E + rn * f.ew + (f.ew == 1 ? 0 : tid));
            kx[tid] = kk;
            ex[tid] = e;
            bk[tid] = e * kk;
            al[tid] = decay ? __expf(ld(G + row_t(t) * f.gw + (f.gw == 1 ? 0 : tid))) : 1.f;
        } else if (tid >= 128 && tid - 128 < ws) {
            const int j = tid - 128;
            vx[j] = ld(V + rn * dv + c0 + j);
            wx[j] = ld(W + rn * f.ww + (f.ww == 1 ? 0 : c0 + j));
        }
        __syncthreads();
        return decay;
    };
    // One forward micro-step on S (after load_step): S- = diag(alpha) S, u = w v - S-^T bk, S = S- + k u^T.
    // `keep` (if not null) receives S-.
    auto forward_step = [&](bool decay, float *keep) {
        if (decay) scale_rows(S, al);
        if (keep) store_local(S, keep);
        col_product(S, bk, uu);
        if (tid < ws) uu[tid] = wx[tid] * vx[tid] - uu[tid];
        __syncthreads();
        rank1(S, kx, uu, 1.f);
    };

    const int64_t cta = bh * p.nslice + sl;
    float *ckpt = p.ckpt + cta * p.nblk * selems;
    float *scratch = p.scratch + cta * (int64_t)kBlk * selems;
    float *dq = p.dq + sl * p.sq, *dkp = p.dk + sl * p.sk, *dep = p.de + sl * p.se;
    float *dgp = gated ? p.dg + sl * p.sg : nullptr, *dw1 = p.dw1 ? p.dw1 + sl * p.sw1 : nullptr;

    // ---- pass 1: the state at the start of every block ----
    load_full(S, f.state_in + bh * (int64_t)dk * dv);
    for (int64_t blk = 0; blk < p.nblk; ++blk) {
        store_local(S, ckpt + blk * selems);
        const int64_t n1 = (blk + 1) * kBlk < N ? (blk + 1) * kBlk : N;
        for (int64_t n = blk * kBlk; n < n1; ++n) forward_step(load_step(n), nullptr);
    }

    // ---- pass 2: block by block from the last, replay forward (keeping S-) and walk back ----
    load_full(dS, p.dS_final ? p.dS_final + bh * (int64_t)dk * dv : nullptr);
    for (int64_t blk = p.nblk - 1; blk >= 0; --blk) {
        const int64_t n0 = blk * kBlk, n1 = (n0 + kBlk) < N ? (n0 + kBlk) : N;
        __syncthreads();
        load_local(S, ckpt + blk * selems);
        for (int64_t n = n0; n < n1; ++n) {
            const bool decay = load_step(n);
            forward_step(decay, scratch + (n - n0) * selems);
        }
        __syncthreads();
        for (int64_t n = n1 - 1; n >= n0; --n) {
            const int64_t t = n / u, m = n % u, rn = row_n(n);
            const bool decay = load_step(n);
            load_local(S, scratch + (n - n0) * selems);  // S-_n
            col_product(S, bk, uu);                     // u_n = w v - S-^T bk (this slice)
            if (tid < ws) uu[tid] = wx[tid] * vx[tid] - uu[tid];
            __syncthreads();
            if (m == u - 1) {  // the read-out step of token t
                const int64_t rt = row_t(t);
                if (tid < dk) qs[tid] = f.scale * ld(Q + rt * dk + tid);
                if (tid < ws) dyv[tid] = p.dy[rt * dv + c0 + tid];
                __syncthreads();
                row_product(S, dyv, nullptr, r1);  // S- dy
                const float udy = block_sum(tid < ws ? uu[tid] * dyv[tid] : 0.f);
                if (tid < dk) dq[rt * dk + tid] = f.scale * (r1[tid] + kx[tid] * udy);
                rank1(dS, qs, dyv, 1.f);
            }
            col_product(dS, kx, du);            // du = dS^T k
            row_product(S, du, nullptr, r1);    // S- du
            row_product(dS, uu, nullptr, r2);   // dS u
            if (tid < dk) dkp[rn * dk + tid] = r2[tid] - ex[tid] * r1[tid];
            if (f.ew != 1) {
                if (tid < dk) dep[rn * dk + tid] = -kx[tid] * r1[tid];
            } else {
                const float s = block_sum(tid < dk ? -kx[tid] * r1[tid] : 0.f);
                if (tid == 0) dep[rn] = s;
            }
            if (tid < ws) p.dv[rn * dv + c0 + tid] = wx[tid] * du[tid];
            if (f.ww != 1) {
                if (tid < ws) p.dw_full[rn * dv + c0 + tid] = vx[tid] * du[tid];
            } else {
                const float s = block_sum(tid < ws ? vx[tid] * du[tid] : 0.f);
                if (tid == 0) dw1[rn] = s;
            }
            rank1(dS, bk, du, -1.f);            // dS-
            if (decay) {
                row_product(dS, nullptr, S, r1);  // sum_j dS-_ij S-_ij
                const int64_t rt = row_t(t);
                if (f.gw != 1) {
                    if (tid < dk) dgp[rt * dk + tid] = r1[tid];
                } else {
                    const float s = block_sum(tid < dk ? r1[tid] : 0.f);
                    if (tid == 0) dgp[rt] = s;
                }
                scale_rows(dS, al);
            }
        }
    }
    __syncthreads();
    store_full(dS, p.dS0 + bh * (int64_t)dk * dv);
}

// out[e] = sum over `nslice` slices (stride `stride`) of part[e], in slice order.
__global__ void reduce_partials(const float *part, int64_t stride, int nslice, float *out, int64_t n) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        float s = part[e];
        for (int k = 1; k < nslice; ++k) s += part[k * stride + e];
        out[e] = s;
    }
}

}  // namespace bwd
}  // namespace dc
