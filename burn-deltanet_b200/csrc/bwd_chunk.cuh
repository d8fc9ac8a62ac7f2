// bwd_chunk.cuh — the backward of the delta-rule core chunk by chunk, for a log-decay per head or none
// (g width 0 or 1), any erase / write width and any n_householder: the gradients the reference's custom
// autodiff node returns (src/delta/chunk_recalculated/combined_backward.rs:72-190).
//
// The forward runs on the folded sequence (micro-step n of token t = n / u; q and dy sit on micro-step
// u - 1 and g on micro-step 0, src/delta_product/delta_product.rs:178-228), cut into chunks of kBL
// micro-steps; zero rows pad the last chunk, an exact identity (src/delta/chunk.rs:16-24).  Per chunk,
// with S the state at its start, the chunk algorithm (src/delta/chunk.rs:103-205) is
//
//   G = cumsum(g), gam = e^G, D_ij = e^{G_i - G_j}
//   A = strict_lower((b (.) k) k^T (.) D),  T = (I + A)^-1
//   W = T (b (.) k (.) gam),  U = T (w (.) v)
//   att = lower(s q k^T (.) D) (diagonal kept),  Q' = s q (.) gam,  K^ = k (.) e^{G_L - G}
//   V' = U - W S,  y = Q' S + att V',  S_next = gam_L S + K^^T V'
//
// For L = <y, dy> + <S_final, dS_final>, walking the chunks back with dS = dL/dS_next:
//
//   dV' = att^T dy + K^ dS,  dS <- gam_L dS + Q'^T dy - W^T dV'
//
// and then, chunk-parallel once every chunk's S and dS_next are known:
//
//   dQ' = dy S^T,  dW = -dV' S^T,  dK^ = V' dS_next^T,  dgam_L = <dS_next, S>,  datt = lower(dy V'^T)
//   dT = dV' (w (.) v)^T + dW (b (.) k (.) gam)^T,  d(w (.) v) = T^T dV',  d(b (.) k (.) gam) = T^T dW
//   dA = strict_lower(-T^T dT T^T)
//
// followed by the chain rule through the elementwise products and D; dg is the reverse cumulative sum of
// dG within the chunk.  Per-channel log-decays put D inside the key-channel sums and take the
// token-by-token backward (bwd_recurrent.cuh) instead.
//
// Three kernels, fp32 on the CUDA cores (register-tiled products over shared memory), every output
// element written once (deterministic):
//   prep_kernel  one CTA per (batch x head, chunk): T, A, att, W, U, Q', K^, gam_L into the workspace;
//   scan_kernel  one CTA per (batch x head, 32 value columns): the forward pass over the chunks, storing
//                each chunk's starting S (transposed) and V', then the reverse pass, storing dS_next
//                (transposed) and dV', and finally dS0;
//   grad_kernel  one CTA per (batch x head, chunk): every input gradient of the chunk's rows.
#pragma once

#include "common.cuh"

namespace dc {
namespace bwdc {

constexpr int kBL = 32;          // micro-steps per chunk (one warp's width: the gate scans are warp scans)
constexpr int kThreads = 256;
constexpr int kMaxD = 128;       // dk, dv
constexpr int kLD = kMaxD + 4;   // row stride of a [kBL][kLD] token tile (floats)
constexpr int kLS = kBL + 4;     // row stride of [kBL][kLS] chunk squares and [kMaxD][kLS] state slices
constexpr int kSlice = 32;       // scan: value columns per CTA

struct Params {
    CoreParams f;                // the forward call
    const float *dy;             // [batch, seq, heads, dv]
    const float *dS_final;       // [batch, heads, dk, dv] or null (zero)
    float *dq, *dk, *dv, *de, *dw, *dg, *dS0;
    // workspace, per chunk ch = bh * nc + c (dkp, dvp: dk, dv rounded up to a multiple of 4)
    float *W, *Kh, *Qp;          // [ch][kBL][dkp]
    float *U, *Vp, *dVp;         // [ch][kBL][dvp]
    float *att, *T, *A;          // [ch][kBL][kBL]
    float *gl;                   // [ch]: gam_L
    float *ST, *dSnT;            // [ch][dvp][dkp]: S at the chunk's start and dS_next, transposed
    int64_t nc;                  // chunks per (batch, head)
    int32_t dkp, dvp, nslice;
};

// ---------------------------------------------------------------------------------------------------
// Register-tiled products.  acc[r][c] += sum_{k<K} A(i0 + r, k) B(k, j0 + c) with
// A(i, k) = A[i * AI + k * AK] and B(k, j) = B[k * BK + j * BJ]; K is a multiple of 4, and the loads
// are float4 / float2 wherever the layout puts consecutive elements together (16-byte aligned bases,
// strides that are multiples of 4 floats).
// ---------------------------------------------------------------------------------------------------
template <int TM, int TN, int AI, int AK, int BK, int BJ>
__device__ __forceinline__ void tile_madd(float (&acc)[TM][TN], int i0, int j0, int K, const float *__restrict__ A,
                                          const float *__restrict__ B) {
    const float *a = A + i0 * AI, *b = B + j0 * BJ;
#pragma unroll 2
    for (int k = 0; k < K; k += 4) {
        float av[TM][4], bv[4][TN];
        if constexpr (AK == 1) {
#pragma unroll
            for (int r = 0; r < TM; ++r) {
                const float4 t = *reinterpret_cast<const float4 *>(a + r * AI + k);
                av[r][0] = t.x, av[r][1] = t.y, av[r][2] = t.z, av[r][3] = t.w;
            }
        } else if constexpr (AI == 1 && TM == 4) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 t = *reinterpret_cast<const float4 *>(a + (k + kk) * AK);
                av[0][kk] = t.x, av[1][kk] = t.y, av[2][kk] = t.z, av[3][kk] = t.w;
            }
        } else if constexpr (AI == 1 && TM == 2) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float2 t = *reinterpret_cast<const float2 *>(a + (k + kk) * AK);
                av[0][kk] = t.x, av[1][kk] = t.y;
            }
        } else {
#pragma unroll
            for (int r = 0; r < TM; ++r)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) av[r][kk] = a[r * AI + (k + kk) * AK];
        }
        if constexpr (BJ == 1 && TN == 4) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 t = *reinterpret_cast<const float4 *>(b + (k + kk) * BK);
                bv[kk][0] = t.x, bv[kk][1] = t.y, bv[kk][2] = t.z, bv[kk][3] = t.w;
            }
        } else if constexpr (BJ == 1 && TN == 2) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float2 t = *reinterpret_cast<const float2 *>(b + (k + kk) * BK);
                bv[kk][0] = t.x, bv[kk][1] = t.y;
            }
        } else if constexpr (BK == 1) {
#pragma unroll
            for (int c = 0; c < TN; ++c) {
                const float4 t = *reinterpret_cast<const float4 *>(b + c * BJ + k);
                bv[0][c] = t.x, bv[1][c] = t.y, bv[2][c] = t.z, bv[3][c] = t.w;
            }
        } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                for (int c = 0; c < TN; ++c) bv[kk][c] = b[(k + kk) * BK + c * BJ];
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int r = 0; r < TM; ++r)
#pragma unroll
                for (int c = 0; c < TN; ++c) acc[r][c] = fmaf(av[r][kk], bv[kk][c], acc[r][c]);
    }
}

// Every output (i, j), i < M, j < N (multiples of TM, TN) of the product above, tiles dealt round robin
// over the CTA's threads; epi(i, j, value) consumes each once.
template <int TM, int TN, int AI, int AK, int BK, int BJ, class Epi>
__device__ __forceinline__ void product(int M, int N, int K, const float *A, const float *B, Epi &&epi) {
    const int tn = N / TN, tiles = (M / TM) * tn;
    for (int t = threadIdx.x; t < tiles; t += kThreads) {
        const int i0 = t / tn * TM, j0 = t % tn * TN;
        float acc[TM][TN];
#pragma unroll
        for (int r = 0; r < TM; ++r)
#pragma unroll
            for (int c = 0; c < TN; ++c) acc[r][c] = 0.f;
        tile_madd<TM, TN, AI, AK, BK, BJ>(acc, i0, j0, K, A, B);
#pragma unroll
        for (int r = 0; r < TM; ++r)
#pragma unroll
            for (int c = 0; c < TN; ++c) epi(i0 + r, j0 + c, acc[r][c]);
    }
}

// rows [kBL] x cols (a multiple of 4) from global (row stride `ls` floats) into shared (row stride `ld`)
__device__ __forceinline__ void load_rows(float *dst, int ld, const float *src, int64_t ls, int cols) {
    const int c4 = cols >> 2;
    for (int idx = threadIdx.x; idx < kBL * c4; idx += kThreads) {
        const int r = idx / c4, q = idx - r * c4;
        *reinterpret_cast<float4 *>(dst + r * ld + 4 * q) = *reinterpret_cast<const float4 *>(src + r * ls + 4 * q);
    }
}

// G = inclusive cumsum over the chunk of its log-decays (warp 0; kBL == 32), gam = e^G, eL = e^{G_L - G}.
// Folded row n carries token n / u's log-decay on micro-step 0 only.
template <typename TG>
__device__ __forceinline__ void gate_scan(const CoreParams &f, const TG *Gp, int64_t b, int64_t h, int64_t c, float *sG,
                                          float *sgam, float *seL) {
    static_assert(kBL == 32, "the gate scans are warp scans");
    const int lane = threadIdx.x;
    const int64_t N = f.seq * f.u, n = c * kBL + lane;
    float g = 0.f;
    if (f.gw > 0 && n < N && n % f.u == 0) g = ld(Gp + ((b * f.seq + n / f.u) * f.heads + h));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float x = __shfl_up_sync(0xffffffffu, g, o);
        if (lane >= o) g += x;
    }
    const float gl = __shfl_sync(0xffffffffu, g, 31);
    sG[lane] = g;
    sgam[lane] = expf(g);
    seL[lane] = expf(gl - g);
}

// The chunk's token rows into shared memory: k, b (.) k (and optionally q) over dkp columns, w (.) v
// over dvp columns; zero outside the sequence and the heads' widths.
template <typename TI, typename TG>
__device__ __forceinline__ void load_chunk_inputs(const CoreParams &f, int64_t b, int64_t h, int64_t c, int dkp, int dvp,
                                                  float *sq, float *sk, float *ske, float *svw) {
    const int dk = (int)f.dk, dv = (int)f.dv, u = f.u;
    const int64_t N = f.seq * u;
    const TI *Q = static_cast<const TI *>(f.q), *K = static_cast<const TI *>(f.k), *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *Wr = static_cast<const TG *>(f.write);
    for (int idx = threadIdx.x; idx < kBL * dkp; idx += kThreads) {
        const int r = idx / dkp, d = idx - r * dkp;
        const int64_t n = c * kBL + r;
        float kv = 0.f, ev = 0.f, qv = 0.f;
        if (n < N && d < dk) {
            const int64_t rn = (b * N + n) * f.heads + h;
            kv = ld(K + rn * dk + d);
            ev = ld(E + rn * f.ew + (f.ew == 1 ? 0 : d));
            if (sq && n % u == u - 1) qv = ld(Q + ((b * f.seq + n / u) * f.heads + h) * dk + d);
        }
        sk[r * kLD + d] = kv;
        ske[r * kLD + d] = ev * kv;
        if (sq) sq[r * kLD + d] = qv;
    }
    for (int idx = threadIdx.x; idx < kBL * dvp; idx += kThreads) {
        const int r = idx / dvp, d = idx - r * dvp;
        const int64_t n = c * kBL + r;
        float x = 0.f;
        if (n < N && d < dv) {
            const int64_t rn = (b * N + n) * f.heads + h;
            x = ld(V + rn * dv + d) * ld(Wr + rn * f.ww + (f.ww == 1 ? 0 : d));
        }
        svw[r * kLD + d] = x;
    }
}

// ---------------------------------------------------------------------------------------------------
// prep_kernel: one CTA per chunk (blockIdx.x = bh * nc + c)
// ---------------------------------------------------------------------------------------------------
constexpr int kPrepSmemFloats = 4 * kBL * kLD + 3 * kBL * kLS + 3 * kBL;

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads) prep_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    const CoreParams &f = p.f;
    const int dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t ch = blockIdx.x, bh = ch / p.nc, c = ch - bh * p.nc, b = bh / f.heads, h = bh - b * f.heads;
    float *sq = sm, *sk = sq + kBL * kLD, *ske = sk + kBL * kLD, *svw = ske + kBL * kLD;
    float *sA = svw + kBL * kLD, *sT = sA + kBL * kLS, *sTg = sT + kBL * kLS;
    float *sG = sTg + kBL * kLS, *sgam = sG + kBL, *seL = sgam + kBL;

    load_chunk_inputs<TI, TG>(f, b, h, c, dkp, dvp, sq, sk, ske, svw);
    if (tid < 32) gate_scan(f, static_cast<const TG *>(f.g), b, h, c, sG, sgam, seL);
    __syncthreads();

    float *gA = p.A + ch * kBL * kBL, *gatt = p.att + ch * kBL * kBL;
    // A = strict_lower((b k) k^T D), att = lower(s q k^T D)
    product<2, 2, kLD, 1, 1, kLD>(kBL, kBL, dkp, ske, sk, [&](int i, int j, float a) {
        const float v = j < i ? a * expf(sG[i] - sG[j]) : 0.f;
        sA[i * kLS + j] = v;
        gA[i * kBL + j] = v;
    });
    product<2, 2, kLD, 1, 1, kLD>(kBL, kBL, dkp, sq, sk, [&](int i, int j, float a) {
        gatt[i * kBL + j] = j <= i ? f.scale * a * expf(sG[i] - sG[j]) : 0.f;
    });
    __syncthreads();
    // T = (I + A)^-1 by forward substitution, lane j owning column j (it reads back only its own writes)
    if (tid < 32) {
        const int j = tid;
        for (int i = 0; i < kBL; ++i) {
            float a0 = i == j ? 1.f : 0.f, a1 = 0.f;
            int k = 0;
            for (; k + 1 < i; k += 2) {
                a0 = fmaf(-sA[i * kLS + k], sT[k * kLS + j], a0);
                a1 = fmaf(-sA[i * kLS + k + 1], sT[(k + 1) * kLS + j], a1);
            }
            if (k < i) a0 = fmaf(-sA[i * kLS + k], sT[k * kLS + j], a0);
            sT[i * kLS + j] = i >= j ? a0 + a1 : 0.f;
        }
    }
    __syncthreads();
    float *gT = p.T + ch * kBL * kBL;
    for (int idx = tid; idx < kBL * kBL; idx += kThreads) {
        const int i = idx / kBL, j = idx - i * kBL;
        const float t = sT[i * kLS + j];
        sTg[i * kLS + j] = t * sgam[j];
        gT[idx] = t;
    }
    __syncthreads();
    // W = (T diag(gam)) (b k),  U = T (w v)
    float *gW = p.W + ch * kBL * dkp, *gU = p.U + ch * kBL * dvp;
    product<4, 4, kLS, 1, kLD, 1>(kBL, dkp, kBL, sTg, ske, [&](int i, int d, float a) { gW[i * dkp + d] = a; });
    product<4, 4, kLS, 1, kLD, 1>(kBL, dvp, kBL, sT, svw, [&](int i, int d, float a) { gU[i * dvp + d] = a; });
    float *gQ = p.Qp + ch * kBL * dkp, *gK = p.Kh + ch * kBL * dkp;
    for (int idx = tid; idx < kBL * dkp; idx += kThreads) {
        const int i = idx / dkp, d = idx - i * dkp;
        gQ[idx] = f.scale * sq[i * kLD + d] * sgam[i];
        gK[idx] = sk[i * kLD + d] * seL[i];
    }
    if (tid == 0) p.gl[ch] = sgam[kBL - 1];
}

// ---------------------------------------------------------------------------------------------------
// scan_kernel: one CTA per (batch x head = blockIdx.x, value slice = blockIdx.y)
// ---------------------------------------------------------------------------------------------------
constexpr int kScanSmemFloats = kMaxD * kLS + 3 * kBL * kLD + 3 * kBL * kLS;

__global__ void __launch_bounds__(kThreads) scan_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float s_gl;
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, u = f.u, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh - b * f.heads, N = f.seq * u, nc = p.nc;
    const int c0 = blockIdx.y * kSlice, wsl = dvp - c0 < kSlice ? dvp - c0 : kSlice;  // a multiple of 4
    float *sX = sm;                        // [kMaxD][kLS]: this slice of S, then of dS
    float *sW = sX + kMaxD * kLS, *sKh = sW + kBL * kLD, *sQp = sKh + kBL * kLD;
    float *satt = sQp + kBL * kLD, *sU = satt + kBL * kLS, *sV = sU + kBL * kLS;
    const int64_t sbase = bh * (int64_t)dk * dv;

    // the slice of a [dk][dv] state in global memory -> sX (zero outside dk x dv)
    auto load_state = [&](const float *src) {
        for (int idx = tid; idx < dkp * wsl; idx += kThreads) {
            const int d = idx / wsl, j = idx - d * wsl;
            sX[d * kLS + j] = (src && d < dk && c0 + j < dv) ? src[sbase + (int64_t)d * dv + c0 + j] : 0.f;
        }
    };
    // sX -> dst[ch][c0 + j][d] (transposed)
    auto store_T = [&](float *dst) {
        for (int idx = tid; idx < wsl * dkp; idx += kThreads) {
            const int j = idx / dkp, d = idx - j * dkp;
            dst[(int64_t)(c0 + j) * dkp + d] = sX[d * kLS + j];
        }
    };

    // ---- forward: S_c, V'_c ----
    load_state(f.state_in);
    for (int64_t c = 0; c < nc; ++c) {
        const int64_t ch = bh * nc + c;
        load_rows(sW, kLD, p.W + ch * kBL * dkp, dkp, dkp);
        load_rows(sKh, kLD, p.Kh + ch * kBL * dkp, dkp, dkp);
        load_rows(sU, kLS, p.U + ch * kBL * dvp + c0, dvp, wsl);
        if (tid == 0) s_gl = p.gl[ch];
        __syncthreads();
        store_T(p.ST + ch * (int64_t)dvp * dkp);
        float *gV = p.Vp + ch * kBL * dvp + c0;
        product<2, 2, kLD, 1, kLS, 1>(kBL, wsl, dkp, sW, sX, [&](int i, int j, float a) {  // V' = U - W S
            const float v = sU[i * kLS + j] - a;
            sV[i * kLS + j] = v;
            gV[i * dvp + j] = v;
        });
        __syncthreads();
        const float gl = s_gl;
        product<4, 4, 1, kLD, kLS, 1>(dkp, wsl, kBL, sKh, sV, [&](int d, int j, float a) {  // S = gam_L S + K^^T V'
            sX[d * kLS + j] = fmaf(gl, sX[d * kLS + j], a);
        });
        __syncthreads();
    }

    // ---- reverse: dS_next_c, dV'_c, then dS0 ----
    load_state(p.dS_final);
    for (int64_t c = nc - 1; c >= 0; --c) {
        const int64_t ch = bh * nc + c;
        load_rows(sW, kLD, p.W + ch * kBL * dkp, dkp, dkp);
        load_rows(sKh, kLD, p.Kh + ch * kBL * dkp, dkp, dkp);
        load_rows(sQp, kLD, p.Qp + ch * kBL * dkp, dkp, dkp);
        load_rows(satt, kLS, p.att + ch * kBL * kBL, kBL, kBL);
        for (int idx = tid; idx < kBL * wsl; idx += kThreads) {  // dy rows: the read-out micro-steps only
            const int r = idx / wsl, j = idx - r * wsl;
            const int64_t n = c * kBL + r;
            float x = 0.f;
            if (n < N && n % u == u - 1 && c0 + j < dv) x = p.dy[((b * f.seq + n / u) * f.heads + h) * dv + c0 + j];
            sU[r * kLS + j] = x;
        }
        if (tid == 0) s_gl = p.gl[ch];
        __syncthreads();
        store_T(p.dSnT + ch * (int64_t)dvp * dkp);
        float *gdV = p.dVp + ch * kBL * dvp + c0;
        // dV' = att^T dy + K^ dS
        for (int t = tid; t < (kBL / 2) * (wsl / 2); t += kThreads) {
            const int i0 = t / (wsl / 2) * 2, j0 = t % (wsl / 2) * 2;
            float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            tile_madd<2, 2, 1, kLS, kLS, 1>(acc, i0, j0, kBL, satt, sU);
            tile_madd<2, 2, kLD, 1, kLS, 1>(acc, i0, j0, dkp, sKh, sX);
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    sV[(i0 + r) * kLS + j0 + q] = acc[r][q];
                    gdV[(i0 + r) * dvp + j0 + q] = acc[r][q];
                }
        }
        __syncthreads();
        // dS = gam_L dS + Q'^T dy - W^T dV'
        const float gl = s_gl;
        for (int t = tid; t < (dkp / 4) * (wsl / 4); t += kThreads) {
            const int d0 = t / (wsl / 4) * 4, j0 = t % (wsl / 4) * 4;
            float ap[4][4], an[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) ap[r][q] = an[r][q] = 0.f;
            tile_madd<4, 4, 1, kLD, kLS, 1>(ap, d0, j0, kBL, sQp, sU);
            tile_madd<4, 4, 1, kLD, kLS, 1>(an, d0, j0, kBL, sW, sV);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float *x = sX + (d0 + r) * kLS + j0 + q;
                    *x = fmaf(gl, *x, ap[r][q] - an[r][q]);
                }
        }
        __syncthreads();
    }
    for (int idx = tid; idx < dk * wsl; idx += kThreads) {
        const int d = idx / wsl, j = idx - d * wsl;
        if (c0 + j < dv) p.dS0[sbase + (int64_t)d * dv + c0 + j] = sX[d * kLS + j];
    }
}

// ---------------------------------------------------------------------------------------------------
// grad_kernel: one CTA per chunk (blockIdx.x = bh * nc + c)
// ---------------------------------------------------------------------------------------------------
constexpr int kGradSmemFloats = 8 * kBL * kLD + 7 * kBL * kLS + 3 * kBL * (kBL + 1) + 6 * kBL + 16;

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads) grad_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, u = f.u, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t ch = blockIdx.x, bh = ch / p.nc, c = ch - bh * p.nc, b = bh / f.heads, h = bh - b * f.heads;
    const int64_t N = f.seq * u;
    constexpr int kTile = kBL * kLD, kSq = kBL * kLS, kRed = kBL + 1;
    float *t0 = sm, *t1 = t0 + kTile, *t2 = t1 + kTile, *t3 = t2 + kTile, *t4 = t3 + kTile;
    float *t5 = t4 + kTile, *t6 = t5 + kTile, *t7 = t6 + kTile;
    float *sT = t7 + kTile, *sA = sT + kSq, *satt = sA + kSq, *sdatt = satt + kSq, *sdT = sdatt + kSq;
    float *sX = sdT + kSq, *sM = sX + kSq;
    float *redG = sM + kSq, *redE = redG + kBL * kRed, *redW = redE + kBL * kRed;
    float *sG = redW + kBL * kRed, *sgam = sG + kBL, *seL = sgam + kBL, *sdG = seL + kBL;
    float *se1 = sdG + kBL, *sw1 = se1 + kBL, *sscal = sw1 + kBL;

    const TI *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *Wr = static_cast<const TG *>(f.write);
    auto row_n = [&](int64_t n) { return (b * N + n) * f.heads + h; };
    auto row_t = [&](int64_t t) { return (b * f.seq + t) * f.heads + h; };

    // This thread's 4 x 4 tile of every [kBL][dkp] result (tnd column groups of 4).
    const int tnd = dkp >> 2;
    const bool own = tid < (kBL / 4) * tnd;
    const int ti0 = own ? tid / tnd * 4 : 0, tg = own ? tid % tnd : 0, td0 = tg * 4;

    // ---- inputs that phase 1 does not touch: k, b k, w v, the gates, T, A, att ----
    load_chunk_inputs<TI, TG>(f, b, h, c, dkp, dvp, nullptr, t5, t6, t7);
    load_rows(sT, kLS, p.T + ch * kBL * kBL, kBL, kBL);
    load_rows(sA, kLS, p.A + ch * kBL * kBL, kBL, kBL);
    load_rows(satt, kLS, p.att + ch * kBL * kBL, kBL, kBL);
    if (tid < 32) {
        gate_scan(f, static_cast<const TG *>(f.g), b, h, c, sG, sgam, seL);
        const int64_t n = c * kBL + tid;
        const bool in = n < N;
        se1[tid] = (in && f.ew == 1) ? ld(E + row_n(n)) : 0.f;
        sw1[tid] = (in && f.ww == 1) ? ld(Wr + row_n(n)) : 0.f;
    }
    // ---- phase 1: the products with S and dS_next ----
    // dy -> t0 (read-out micro-steps only), V' -> t1, dV' -> t2
    for (int idx = tid; idx < kBL * dvp; idx += kThreads) {
        const int r = idx / dvp, j = idx - r * dvp;
        const int64_t n = c * kBL + r;
        t0[r * kLD + j] = (n < N && n % u == u - 1 && j < dv) ? p.dy[row_t(n / u) * dv + j] : 0.f;
    }
    load_rows(t1, kLD, p.Vp + ch * kBL * dvp, dvp, dvp);
    load_rows(t2, kLD, p.dVp + ch * kBL * dvp, dvp, dvp);
    float aq[4][4], aw[4][4], ak[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) aq[r][q] = aw[r][q] = ak[r][q] = 0.f;
    float dgl_part = 0.f;
    const float *gST = p.ST + ch * (int64_t)dvp * dkp, *gdS = p.dSnT + ch * (int64_t)dvp * dkp;
    for (int jb = 0; jb < dvp; jb += kBL) {
        const int jn = dvp - jb < kBL ? dvp - jb : kBL;
        __syncthreads();
        const int c4 = dkp >> 2;
        for (int idx = tid; idx < jn * c4; idx += kThreads) {  // S^T, dS_next^T rows jb.. -> t3, t4
            const int r = idx / c4, q = idx - r * c4;
            const float4 x = *reinterpret_cast<const float4 *>(gST + (int64_t)(jb + r) * dkp + 4 * q);
            const float4 y = *reinterpret_cast<const float4 *>(gdS + (int64_t)(jb + r) * dkp + 4 * q);
            *reinterpret_cast<float4 *>(t3 + r * kLD + 4 * q) = x;
            *reinterpret_cast<float4 *>(t4 + r * kLD + 4 * q) = y;
            dgl_part += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
        }
        __syncthreads();
        if (own) {
            tile_madd<4, 4, kLD, 1, kLD, 1>(aq, ti0, td0, jn, t0 + jb, t3);  // dy S^T
            tile_madd<4, 4, kLD, 1, kLD, 1>(aw, ti0, td0, jn, t2 + jb, t3);  // dV' S^T
            tile_madd<4, 4, kLD, 1, kLD, 1>(ak, ti0, td0, jn, t1 + jb, t4);  // V' dS_next^T
        }
    }
    // datt = lower(dy V'^T)
    product<2, 2, kLD, 1, 1, kLD>(kBL, kBL, dvp, t0, t1, [&](int i, int j, float a) {
        sdatt[i * kLS + j] = j <= i ? a : 0.f;
    });
    // <dS_next, S> over the CTA
    {
        float v = dgl_part;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((tid & 31) == 0) sscal[tid >> 5] = v;
    }
    __syncthreads();
    // park dQ' -> t0, dW = -dV' S^T -> t1, dK^ -> t3; q -> t4
    if (own) {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int o = (ti0 + r) * kLD + td0 + q;
                t0[o] = aq[r][q];
                t1[o] = -aw[r][q];
                t3[o] = ak[r][q];
            }
    }
    {
        const TI *Q = static_cast<const TI *>(f.q);
        for (int idx = tid; idx < kBL * dkp; idx += kThreads) {
            const int r = idx / dkp, d = idx - r * dkp;
            const int64_t n = c * kBL + r;
            t4[r * kLD + d] = (n < N && n % u == u - 1 && d < dk) ? ld(Q + row_t(n / u) * dk + d) : 0.f;
        }
    }
    __syncthreads();

    // ---- phase 2 ----
    // dT = dV' (w v)^T + dW (b k)^T diag(gam)
    for (int t = tid; t < (kBL / 2) * (kBL / 2); t += kThreads) {
        const int i0 = t / (kBL / 2) * 2, j0 = t % (kBL / 2) * 2;
        float a1[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, a2[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        tile_madd<2, 2, kLD, 1, 1, kLD>(a1, i0, j0, dvp, t2, t7);
        tile_madd<2, 2, kLD, 1, 1, kLD>(a2, i0, j0, dkp, t1, t6);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int q = 0; q < 2; ++q) sdT[(i0 + r) * kLS + j0 + q] = fmaf(sgam[j0 + q], a2[r][q], a1[r][q]);
    }
    // d(w v) = T^T dV'  ->  d_v = w d(wv), d_write = v d(wv)
    {
        const int tnv = dvp >> 2;
        for (int t = tid; t < (kBL / 4) * tnv; t += kThreads) {
            const int j0 = t / tnv * 4, g = t % tnv, d0 = g * 4;
            float acc[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;
            tile_madd<4, 4, 1, kLS, kLD, 1>(acc, j0, d0, kBL, sT, t2);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int64_t n = c * kBL + j0 + r;
                float part = 0.f;
                if (n < N) {
                    const int64_t rn = row_n(n);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int d = d0 + q;
                        if (d < dv) {
                            const float wv = f.ww == 1 ? sw1[j0 + r] : ld(Wr + rn * dv + d);
                            const float vv = ld(V + rn * dv + d);
                            p.dv[rn * dv + d] = wv * acc[r][q];
                            if (f.ww == 1) part = fmaf(vv, acc[r][q], part);
                            else p.dw[rn * dv + d] = vv * acc[r][q];
                        }
                    }
                }
                if (f.ww == 1) redW[(j0 + r) * kRed + g] = part;
            }
        }
    }
    // d(b k gam) = T^T dW: its part of d(b k) and of dG
    float ake[4][4], dGp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) ake[r][q] = 0.f;
    if (own) {
        tile_madd<4, 4, 1, kLS, kLD, 1>(ake, ti0, td0, kBL, sT, t1);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float gm = sgam[ti0 + r];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                dGp[r] = fmaf(ake[r][q], t6[(ti0 + r) * kLD + td0 + q], dGp[r]);
                ake[r][q] *= gm;
            }
            dGp[r] *= gm;
        }
    }
    __syncthreads();
    // dA = strict_lower(-T^T dT T^T): X = T^T dT, then dA = -X T^T; Fa = dA D -> sdT, dA A -> sM
    product<2, 2, 1, kLS, kLS, 1>(kBL, kBL, kBL, sT, sdT, [&](int i, int j, float a) { sX[i * kLS + j] = a; });
    __syncthreads();
    product<2, 2, kLS, 1, 1, kLS>(kBL, kBL, kBL, sX, sT, [&](int i, int j, float a) {
        const float da = j < i ? -a : 0.f;
        sdT[i * kLS + j] = j < i ? da * expf(sG[i] - sG[j]) : 0.f;
        sM[i * kLS + j] = da * sA[i * kLS + j];
    });
    // attention: F = s datt D -> sdatt, datt att -> satt
    for (int idx = tid; idx < kBL * kBL; idx += kThreads) {
        const int i = idx / kBL, j = idx - i * kBL;
        const float dd = sdatt[i * kLS + j];
        sdatt[i * kLS + j] = j <= i ? f.scale * dd * expf(sG[i] - sG[j]) : 0.f;
        satt[i * kLS + j] = dd * satt[i * kLS + j];
    }
    __syncthreads();
    // dG from the squares: row sums minus column sums of dA A + datt att
    if (tid < kBL) {
        float s = 0.f;
        for (int j = 0; j < kBL; ++j)
            s += (sM[tid * kLS + j] + satt[tid * kLS + j]) - (sM[j * kLS + tid] + satt[j * kLS + tid]);
        sdG[tid] = s;
    }
    // d_q, d_k, d_erase
    float khat_part = 0.f;
    if (own) {
        float aqk[4][4], akk[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) aqk[r][q] = akk[r][q] = 0.f;
        tile_madd<4, 4, kLS, 1, kLD, 1>(aqk, ti0, td0, kBL, sdatt, t5);  // F k
        tile_madd<4, 4, 1, kLS, kLD, 1>(akk, ti0, td0, kBL, sdatt, t4);  // F^T q
        tile_madd<4, 4, 1, kLS, kLD, 1>(akk, ti0, td0, kBL, sdT, t6);    // Fa^T (b k)
        tile_madd<4, 4, kLS, 1, kLD, 1>(ake, ti0, td0, kBL, sdT, t5);    // Fa k
        float epart[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = ti0 + r;
            const int64_t n = c * kBL + i;
            const float sg = f.scale * sgam[i], el = seL[i];
            const bool in = n < N;
            const int64_t rn = in ? row_n(n) : 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int d = td0 + q, o = i * kLD + d;
                const float dqp = t0[o], dkh = t3[o], qv = t4[o], kv = t5[o];
                aqk[r][q] = fmaf(sg, dqp, aqk[r][q]);
                dGp[r] += sg * dqp * qv;
                const float kh = el * dkh * kv;
                dGp[r] -= kh;
                khat_part += kh;
                float ev = 0.f;
                if (in && d < dk) ev = f.ew == 1 ? se1[i] : ld(E + rn * dk + d);
                akk[r][q] = fmaf(el, dkh, fmaf(ev, ake[r][q], akk[r][q]));
                const float de = kv * ake[r][q];
                if (f.ew == 1) epart[r] += de;
                else if (in && d < dk) p.de[rn * dk + d] = de;
                if (in && d < dk) {
                    p.dk[rn * dk + d] = akk[r][q];
                    if (n % u == u - 1) p.dq[row_t(n / u) * dk + d] = aqk[r][q];
                }
            }
            redG[i * kRed + tg] = dGp[r];
            if (f.ew == 1) redE[i * kRed + tg] = epart[r];
        }
    }
    {
        float v = khat_part;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((tid & 31) == 0) sscal[8 + (tid >> 5)] = v;
    }
    __syncthreads();
    // row totals (in column-group order), dG at the last row, and the reverse cumsum -> d_g
    if (tid < 32) {
        const int i = tid;
        const int64_t n = c * kBL + i;
        float dG = sdG[i];
        for (int g = 0; g < tnd; ++g) dG += redG[i * kRed + g];
        if (i == kBL - 1) {
            float dgl = 0.f, kh = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) dgl += sscal[w], kh += sscal[8 + w];
            dG += kh + sgam[kBL - 1] * dgl;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float x = __shfl_down_sync(0xffffffffu, dG, o);
            if (i + o < 32) dG += x;
        }
        if (n < N) {
            const int64_t rn = row_n(n);
            if (f.gw > 0 && n % u == 0) p.dg[row_t(n / u)] = dG;
            if (f.ew == 1) {
                float s = 0.f;
                for (int g = 0; g < tnd; ++g) s += redE[i * kRed + g];
                p.de[rn] = s;
            }
            if (f.ww == 1) {
                float s = 0.f;
                for (int g = 0; g < (dvp >> 2); ++g) s += redW[i * kRed + g];
                p.dw[rn] = s;
            }
        }
    }
}

}  // namespace bwdc
}  // namespace dc
