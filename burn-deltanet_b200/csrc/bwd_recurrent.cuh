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
// each step's S- in a per-(batch, head) scratch, and walks the block back.  S and dS live in shared
// memory; one CTA (256 threads) per (batch, head); dk, dv <= 128.
#pragma once

#include "common.cuh"

namespace dc {
namespace bwd {

constexpr int kThreads = 256;
constexpr int kBlk = 16;    // micro-steps per checkpoint block
constexpr int kMaxD = 128;  // dk, dv

struct Params {
    CoreParams f;           // the forward call: dims, widths, scale, q, k, v, erase, write, g, state_in
    const float *dy;        // [batch, seq, heads, dv]
    const float *dS_final;  // [batch, heads, dk, dv] or null (zero)
    float *dq, *dk, *dv;    // [batch, seq, heads, dk]; [batch, seq*u, heads, dk]; [batch, seq*u, heads, dv]
    float *de, *dw;         // [batch, seq*u, heads, erase_w]; [batch, seq*u, heads, write_w]
    float *dg;              // [batch, seq, heads, g_w] (g_w > 0)
    float *dS0;             // [batch, heads, dk, dv]
    float *ckpt;            // [batch*heads][nblk][dk][dv]
    float *scratch;         // [batch*heads][kBlk][dk][dv]
    int64_t nblk;
};

// Shared-memory layout (floats): S and dS with a row pitch of dv + 1 (row and column sweeps both
// conflict-free), then the step's vectors and two rows of partial sums.
struct Layout {
    int dk, dv, P;
    int S, dS, kx, bk, ex, al, qs, r1, r2, vx, wx, uu, du, dy, red, scal, total;
    __host__ __device__ Layout(int dk_, int dv_) : dk(dk_), dv(dv_), P(dv_ + 1) {
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
        wx = vx + kMaxD;
        uu = wx + kMaxD;
        du = uu + kMaxD;
        dy = du + kMaxD;
        red = dy + kMaxD;         // [2][kMaxD]
        scal = red + 2 * kMaxD;   // [8] block-reduction slots
        total = scal + 8 * 32;
    }
};

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads) bwd_recurrent_kernel(const Params p) {
    extern __shared__ float sm[];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, u = f.u;
    const Layout L(dk, dv);
    const int P = L.P;
    float *S = sm + L.S, *dS = sm + L.dS;
    float *kx = sm + L.kx, *bk = sm + L.bk, *ex = sm + L.ex, *al = sm + L.al, *qs = sm + L.qs;
    float *r1 = sm + L.r1, *r2 = sm + L.r2, *vx = sm + L.vx, *wx = sm + L.wx, *uu = sm + L.uu;
    float *du = sm + L.du, *dyv = sm + L.dy, *red = sm + L.red, *scal = sm + L.scal;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh % f.heads;
    const int64_t N = f.seq * u;  // micro-steps
    const int64_t elems = (int64_t)dk * dv;
    const bool gated = f.gw > 0;
    // Element sweeps over a [dk][dv] matrix: thread (er, ec) takes column ec of rows er, er + rstep, ...
    const int rstep = kThreads / dv, er = tid / dv, ec = tid - er * dv;
    const bool sweeper = er < rstep;

    const TI *Q = static_cast<const TI *>(f.q), *K = static_cast<const TI *>(f.k), *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *W = static_cast<const TG *>(f.write), *G = static_cast<const TG *>(f.g);
    auto row_n = [&](int64_t n) { return (b * N + n) * f.heads + h; };       // micro-step rows
    auto row_t = [&](int64_t t) { return (b * f.seq + t) * f.heads + h; };   // token rows

    // ---- block-wide helpers (all threads; each ends with a barrier) ----
    // out[j] = sum_i M[i][j] x[i]
    auto col_product = [&](const float *M, const float *x, float *out) {
        const int j = tid & 127, half = tid >> 7, h0 = half * ((dk + 1) >> 1), h1 = half ? dk : ((dk + 1) >> 1);
        if (j < dv) {
            float a0 = 0.f, a1 = 0.f;
            int i = h0;
            for (; i + 1 < h1; i += 2) {
                a0 = fmaf(M[i * P + j], x[i], a0);
                a1 = fmaf(M[(i + 1) * P + j], x[i + 1], a1);
            }
            if (i < h1) a0 = fmaf(M[i * P + j], x[i], a0);
            red[half * kMaxD + j] = a0 + a1;
        }
        __syncthreads();
        if (tid < dv) out[tid] = red[tid] + red[kMaxD + tid];
        __syncthreads();
    };
    // out[i] = sum_j M[i][j] x[j]   (x == nullptr: out[i] = sum_j M[i][j] N2[i][j])
    auto row_product = [&](const float *M, const float *x, const float *M2, float *out) {
        const int i = tid & 127, half = tid >> 7, c0 = half * ((dv + 1) >> 1), c1 = half ? dv : ((dv + 1) >> 1);
        if (i < dk) {
            float a0 = 0.f, a1 = 0.f;
            int j = c0;
            if (x) {
                for (; j + 1 < c1; j += 2) {
                    a0 = fmaf(M[i * P + j], x[j], a0);
                    a1 = fmaf(M[i * P + j + 1], x[j + 1], a1);
                }
                if (j < c1) a0 = fmaf(M[i * P + j], x[j], a0);
            } else {
                for (; j + 1 < c1; j += 2) {
                    a0 = fmaf(M[i * P + j], M2[i * P + j], a0);
                    a1 = fmaf(M[i * P + j + 1], M2[i * P + j + 1], a1);
                }
                if (j < c1) a0 = fmaf(M[i * P + j], M2[i * P + j], a0);
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
            for (int i = er; i < dk; i += rstep) M[i * P + ec] = fmaf(a[i], bj, M[i * P + ec]);
        }
        __syncthreads();
    };
    auto scale_rows = [&](float *M, const float *a) {
        if (sweeper)
            for (int i = er; i < dk; i += rstep) M[i * P + ec] *= a[i];
        __syncthreads();
    };
    // sum over the block of one value per thread (threads beyond `n` pass 0)
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
    // global <-> shared state copies ([dk][dv] contiguous in global memory)
    auto store_state = [&](const float *M, float *dst) {
        if (sweeper)
            for (int i = er; i < dk; i += rstep) dst[i * dv + ec] = M[i * P + ec];
    };
    auto load_state = [&](float *M, const float *src) {
        if (sweeper)
            for (int i = er; i < dk; i += rstep) M[i * P + ec] = src ? src[i * dv + ec] : 0.f;
        __syncthreads();
    };

    // The inputs of micro-step n into the shared vectors: k, b (.) k, the erase row (width-expanded),
    // the decay alpha (1 unless micro-step 0 of a gated token), v, w.
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
        }
        if (tid < dv) {
            vx[tid] = ld(V + rn * dv + tid);
            wx[tid] = ld(W + rn * f.ww + (f.ww == 1 ? 0 : tid));
        }
        __syncthreads();
        return decay;
    };
    // One forward micro-step on S (after load_step): S- = diag(alpha) S, u = w v - S-^T bk, S = S- + k u^T.
    // `keep` (if not null) receives S-.
    auto forward_step = [&](bool decay, float *keep) {
        if (decay) scale_rows(S, al);
        if (keep) store_state(S, keep);
        col_product(S, bk, uu);
        if (tid < dv) uu[tid] = wx[tid] * vx[tid] - uu[tid];
        __syncthreads();
        rank1(S, kx, uu, 1.f);
    };

    float *ckpt = p.ckpt + bh * p.nblk * elems;
    float *scratch = p.scratch + bh * (int64_t)kBlk * elems;

    // ---- pass 1: the state at the start of every block ----
    load_state(S, f.state_in + bh * elems);
    for (int64_t blk = 0; blk < p.nblk; ++blk) {
        store_state(S, ckpt + blk * elems);
        const int64_t n1 = (blk + 1) * kBlk < N ? (blk + 1) * kBlk : N;
        for (int64_t n = blk * kBlk; n < n1; ++n) forward_step(load_step(n), nullptr);
    }

    // ---- pass 2: block by block from the last, replay forward (keeping S-) and walk back ----
    load_state(dS, p.dS_final ? p.dS_final + bh * elems : nullptr);
    for (int64_t blk = p.nblk - 1; blk >= 0; --blk) {
        const int64_t n0 = blk * kBlk, n1 = (n0 + kBlk) < N ? (n0 + kBlk) : N;
        __syncthreads();
        load_state(S, ckpt + blk * elems);
        for (int64_t n = n0; n < n1; ++n) {
            const bool decay = load_step(n);
            forward_step(decay, scratch + (n - n0) * elems);
        }
        __syncthreads();
        for (int64_t n = n1 - 1; n >= n0; --n) {
            const int64_t t = n / u, m = n % u, rn = row_n(n);
            const bool decay = load_step(n);
            load_state(S, scratch + (n - n0) * elems);  // S-_n
            col_product(S, bk, uu);                    // u_n = w v - S-^T bk
            if (tid < dv) uu[tid] = wx[tid] * vx[tid] - uu[tid];
            __syncthreads();
            if (m == u - 1) {  // the read-out step of token t
                const int64_t rt = row_t(t);
                if (tid < dk) qs[tid] = f.scale * ld(Q + rt * dk + tid);
                if (tid < dv) dyv[tid] = p.dy[rt * dv + tid];
                __syncthreads();
                row_product(S, dyv, nullptr, r1);  // S- dy
                const float udy = block_sum(tid < dv ? uu[tid] * dyv[tid] : 0.f);
                if (tid < dk) p.dq[rt * dk + tid] = f.scale * (r1[tid] + kx[tid] * udy);
                rank1(dS, qs, dyv, 1.f);
            }
            col_product(dS, kx, du);            // du = dS^T k
            row_product(S, du, nullptr, r1);    // S- du
            row_product(dS, uu, nullptr, r2);   // dS u
            if (tid < dk) p.dk[rn * dk + tid] = r2[tid] - ex[tid] * r1[tid];
            if (f.ew != 1) {
                if (tid < dk) p.de[rn * dk + tid] = -kx[tid] * r1[tid];
            } else {
                const float s = block_sum(tid < dk ? -kx[tid] * r1[tid] : 0.f);
                if (tid == 0) p.de[rn] = s;
            }
            if (tid < dv) p.dv[rn * dv + tid] = wx[tid] * du[tid];
            if (f.ww != 1) {
                if (tid < dv) p.dw[rn * dv + tid] = vx[tid] * du[tid];
            } else {
                const float s = block_sum(tid < dv ? vx[tid] * du[tid] : 0.f);
                if (tid == 0) p.dw[rn] = s;
            }
            rank1(dS, bk, du, -1.f);            // dS-
            if (decay) {
                row_product(dS, nullptr, S, r1);  // sum_j dS-_ij S-_ij
                const int64_t rt = row_t(t);
                if (f.gw != 1) {
                    if (tid < dk) p.dg[rt * dk + tid] = r1[tid];
                } else {
                    const float s = block_sum(tid < dk ? r1[tid] : 0.f);
                    if (tid == 0) p.dg[rt] = s;
                }
                scale_rows(dS, al);
            }
        }
    }
    __syncthreads();
    store_state(dS, p.dS0 + bh * elems);
}

}  // namespace bwd
}  // namespace dc
