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
// Three kernels over fp32 data, every product on the tensor cores as three mma.sync tf32 products of
// split operands (about fp32 accuracy), every output element written once (deterministic):
//   prep_kernel  one CTA per (batch x head, chunk): T, A, att, W, U, Q', K^, gam_L into the workspace;
//   scan_kernel  one CTA per (batch x head, 32 value columns): the forward pass over the chunks, storing
//                each chunk's starting S (transposed) and V', then the reverse pass, storing dS_next
//                (transposed) and dV', and finally dS0 (scan_wide_kernel: the same over every value
//                column of a head, when the slices would not fit on the SMs in one wave);
//   grad_kernel  one CTA per (batch x head, chunk): every input gradient of the chunk's rows.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace dc {
namespace bwdc {

constexpr int kBL = 32;          // micro-steps per chunk (one warp's width: the gate scans are warp scans)
constexpr int kThreads = 256;
constexpr int kMaxD = 128;       // dk, dv
constexpr int kLD = kMaxD + 4;   // row stride of a [kBL][kLD] token tile (floats)
constexpr int kLS = kBL + 8;     // row stride of [kBL][kLS] chunk squares and [kMaxD][kLS] state slices
constexpr int kSlice = 32;       // scan: value columns per CTA
constexpr int kWS = kMaxD + 8;   // row stride of full-width tiles read as B (rows t, columns g) or as a
                                 // transposed A (AI = 1): 8 mod 32, so a warp's fragment hits 32 banks
constexpr int kAS = kBL + 4;     // row stride of a [kBL][kBL] square read as A (rows g, columns t)
constexpr int kWideThreads = 512;  // the full-width scans: 16 warps, four per SM sub-partition

struct Params {
    CoreParams f;                // the forward call
    const float *dy;             // [batch, seq, heads, dv]
    const float *dS_final;       // [batch, heads, dk, dv] or null (zero)
    float *dq, *dk, *dv, *de, *dw, *dg, *dS0;
    // workspace, per chunk ch = bh * nc + c (dkp, dvp: dk, dv rounded up to a multiple of 8)
    float *W, *Kh, *Qp;          // [ch][kBL][dkp]
    float *U, *Vp, *dVp;         // [ch][kBL][dvp]
    float *att, *T, *A;          // [ch][kBL][kBL]
    float *gl;                   // [ch]: gam_L
    float *ST, *dSnT;            // [ch][dvp][dkp]: S at the chunk's start and dS_next, transposed
    int64_t nc;                  // chunks per (batch, head)
    int32_t dkp, dvp, nslice;
    int32_t dy_vec;              // dy rows are 16-byte aligned (dv % 4 == 0): copied by cp.async
};

// One warp on the tensor cores: acc[n], the 16 x 8 tile at rows i0.., columns j0 + 8n.., += A(i, k) B(k, j)
// over k < K (a multiple of 8), with A(i, k) = A[i * AI + k * AK] and B(k, j) = B[k * BK + j * BJ].  Each
// operand is split into a tf32-exact big part and a small remainder, and big x big + big x small +
// small x big (three mma.sync m16n8k8) recovers ~fp32 accuracy.  Fragment of lane (g = lane / 4,
// t = lane % 4): acc[n] = {C(i0+g, j0+8n+2t), C(i0+g, j0+8n+2t+1), C(i0+g+8, j0+8n+2t), C(i0+g+8, j0+8n+2t+1)}.
// Rows and columns past the caller's extents may be read (they must lie inside the buffers); their
// outputs are the caller's to drop.
// UNR: the k loop's unroll factor (1 where a kernel's code size costs more than the lost overlap: the
// grad kernel's many products).
template <int NT, int AI, int AK, int BK, int BJ, int UNR = 2>
__device__ __forceinline__ void warp_mma3(float (&acc)[NT][4], int i0, int j0, int K, const float *__restrict__ A,
                                          const float *__restrict__ B) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float *a = A + (i0 + g) * AI + t * AK;
    const float *b = B + t * BK + (j0 + g) * BJ;
#pragma unroll UNR
    for (int k = 0; k < K; k += 8) {
        uint32_t ab[4], as[4];
        ptx::split_tf32(a[k * AK], ab[0], as[0]);
        ptx::split_tf32(a[8 * AI + k * AK], ab[1], as[1]);
        ptx::split_tf32(a[(k + 4) * AK], ab[2], as[2]);
        ptx::split_tf32(a[8 * AI + (k + 4) * AK], ab[3], as[3]);
        uint32_t bb[NT][2], bs[NT][2];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            ptx::split_tf32(b[k * BK + 8 * n * BJ], bb[n][0], bs[n][0]);
            ptx::split_tf32(b[(k + 4) * BK + 8 * n * BJ], bb[n][1], bs[n][1]);
        }
        // term by term over the NT tiles (each accumulator still takes its three products in order)
#pragma unroll
        for (int n = 0; n < NT; ++n) ptx::mma_tf32_16x8x8(acc[n], as, bb[n]);
#pragma unroll
        for (int n = 0; n < NT; ++n) ptx::mma_tf32_16x8x8(acc[n], ab, bs[n]);
#pragma unroll
        for (int n = 0; n < NT; ++n) ptx::mma_tf32_16x8x8(acc[n], ab, bb[n]);
    }
}

// acc[m][n] (the 16 x 8 tile at rows i0 + RS m, columns j0 + 8 n) += A(i, k) B(k, j) over k < K (a multiple
// of 8), with A(i, k) = A[i * AI + k * AK] and B(k, j) = B[k * BK + j * BJ]; three-part tf32 products as in
// warp_mma3.  The MT row blocks share each B fragment, the NT column blocks each A fragment.
template <int MT, int RS, int NT, int AI, int AK, int BK, int BJ = 1>
__device__ __forceinline__ void warp_mma3_block(float (&acc)[MT][NT][4], int i0, int j0, int K,
                                                const float *__restrict__ A, const float *__restrict__ B) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float *a = A + (i0 + g) * AI + t * AK;
    const float *b = B + t * BK + (j0 + g) * BJ;
#pragma unroll 2
    for (int k = 0; k < K; k += 8) {
        uint32_t ab[MT][4], as[MT][4];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float *am = a + m * RS * AI + k * AK;
            ptx::split_tf32(am[0], ab[m][0], as[m][0]);
            ptx::split_tf32(am[8 * AI], ab[m][1], as[m][1]);
            ptx::split_tf32(am[4 * AK], ab[m][2], as[m][2]);
            ptx::split_tf32(am[8 * AI + 4 * AK], ab[m][3], as[m][3]);
        }
        uint32_t bb[NT][2], bs[NT][2];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            ptx::split_tf32(b[k * BK + 8 * n * BJ], bb[n][0], bs[n][0]);
            ptx::split_tf32(b[(k + 4) * BK + 8 * n * BJ], bb[n][1], bs[n][1]);
        }
        // term by term over every tile, so that the three products into one accumulator are MT x NT
        // issues apart (the tensor pipe works on the other tiles' products meanwhile)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int m = 0; m < MT; ++m) ptx::mma_tf32_16x8x8(acc[m][n], as[m], bb[n]);
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int m = 0; m < MT; ++m) ptx::mma_tf32_16x8x8(acc[m][n], ab[m], bs[n]);
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int m = 0; m < MT; ++m) ptx::mma_tf32_16x8x8(acc[m][n], ab[m], bb[n]);
    }
}

// epi(i, j, value) for the in-range elements (i < M, j < N) of the tile's fragments.
template <int MT, int RS, int NT, class Epi>
__device__ __forceinline__ void block_store(const float (&acc)[MT][NT][4], int i0, int j0, int M, int N, Epi &&epi) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = i0 + RS * m + g + (q >> 1) * 8, j = j0 + 8 * n + 2 * t + (q & 1);
                if (i < M && j < N) epi(i, j, acc[m][n][q]);
            }
}

// Calls f(i0, j0) for the 16 x (8 NT) warp tiles of an M x N output, dealt round robin over the warps.
template <int NT, class F>
__device__ __forceinline__ void for_warp_tiles(int M, int N, F &&f) {
    const int tn = (N + 8 * NT - 1) / (8 * NT), tiles = ((M + 15) >> 4) * tn;
    for (int w = threadIdx.x >> 5; w < tiles; w += kThreads / 32) f(w / tn * 16, w % tn * (8 * NT));
}

// epi(i, j, value) for the in-range elements (i < M, j < N) of a warp tile's fragments.
template <int NT, class Epi>
__device__ __forceinline__ void frag_store(const float (&acc)[NT][4], int i0, int j0, int M, int N, Epi &&epi) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = i0 + g + (q >> 1) * 8, j = j0 + 8 * n + 2 * t + (q & 1);
            if (i < M && j < N) epi(i, j, acc[n][q]);
        }
}

// copy_rows_async for a CTA of NTHR threads.
template <int NTHR>
__device__ __forceinline__ void copy_rows(float *dst, int ld, const float *src, int64_t ls, int cols) {
    const int c4 = cols >> 2;
    for (int idx = threadIdx.x; idx < kBL * c4; idx += NTHR) {
        const int r = idx / c4, q = idx - r * c4;
        ptx::cp_async16(ptx::smem_u32(dst + r * ld + 4 * q), src + r * ls + 4 * q, 16u);
    }
}

// Workspace rows [kBL] x cols (a multiple of 4 floats) from global (row stride `ls` floats) into shared
// (row stride `ld`) by 16-byte asynchronous copies; the caller commits, waits and synchronises.
__device__ __forceinline__ void copy_rows_async(float *dst, int ld, const float *src, int64_t ls, int cols) {
    const int c4 = cols >> 2;
    for (int idx = threadIdx.x; idx < kBL * c4; idx += kThreads) {
        const int r = idx / c4, q = idx - r * c4;
        ptx::cp_async16(ptx::smem_u32(dst + r * ld + 4 * q), src + r * ls + 4 * q, 16u);
    }
}

// dst[r * lds + d] = x(r, d) for r < kBL, d < width, zero for width <= d < widthp (widthp <= kMaxD), with
// x = a[off_a(r, d)] (times b[off_b(r, d)] when TWO); an offset below zero stands for a zero.  The loads
// are unconditional (a dropped element reads the base) and branch-free, and each thread issues all of
// its loads before its first store, so their latencies overlap.
template <bool TWO, typename TA, typename TB, class OffA, class OffB>
__device__ __forceinline__ void gather_rows(float *dst, int lds, int width, int widthp, const TA *a, OffA &&off_a,
                                            const TB *b, OffB &&off_b) {
    constexpr int kPer = kBL * kMaxD / kThreads;
    float xa[kPer], xb[kPer];
    int at[kPer];
    bool keep[kPer];
    const int total = kBL * widthp;
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
        const int idx = threadIdx.x + m * kThreads;
        const int r = idx / widthp, d = idx - r * widthp;
        const bool in = idx < total;
        const int64_t oa = (in && d < width) ? off_a(r, d) : -1;
        at[m] = in ? r * lds + d : -1;
        keep[m] = oa >= 0;
        xa[m] = ld(a + (keep[m] ? oa : 0));
        if constexpr (TWO) xb[m] = ld(b + (keep[m] ? off_b(r, d) : 0));
    }
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
        float v = xa[m];
        if constexpr (TWO) v *= xb[m];
        if (at[m] >= 0) dst[at[m]] = keep[m] ? v : 0.f;
    }
}

// As gather_rows<true>, writing both factors' product to dst_ab and the first factor alone to dst_a (k and
// b (.) k from one pass over k).
template <typename TA, typename TB, class OffA, class OffB>
__device__ __forceinline__ void gather_rows_pair(float *dst_a, float *dst_ab, int lds, int width, int widthp,
                                                 const TA *a, OffA &&off_a, const TB *b, OffB &&off_b) {
    constexpr int kPer = kBL * kMaxD / kThreads;
    float xa[kPer], xb[kPer];
    int at[kPer];
    bool keep[kPer];
    const int total = kBL * widthp;
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
        const int idx = threadIdx.x + m * kThreads;
        const int r = idx / widthp, d = idx - r * widthp;
        const bool in = idx < total;
        const int64_t oa = (in && d < width) ? off_a(r, d) : -1;
        at[m] = in ? r * lds + d : -1;
        keep[m] = oa >= 0;
        xa[m] = ld(a + (keep[m] ? oa : 0));
        xb[m] = ld(b + (keep[m] ? off_b(r, d) : 0));
    }
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
        if (at[m] >= 0) {
            dst_a[at[m]] = keep[m] ? xa[m] : 0.f;
            dst_ab[at[m]] = keep[m] ? xa[m] * xb[m] : 0.f;
        }
    }
}

// Row indices (of the [batch, rows, heads, .] layouts) of chunk c's micro-steps, one lane of warp 0 per
// row: rn for k / v / erase / write (-1 past the sequence); rt for q / dy (-1 unless a read-out
// micro-step); rg for g (-1 unless micro-step 0 of a gated token).
struct ChunkRows {
    int64_t rn, rt, rg;
};
__device__ __forceinline__ ChunkRows chunk_rows(const CoreParams &f, int64_t b, int64_t h, int64_t c, int r) {
    const int64_t N = f.seq * f.u, n = c * kBL + r;
    ChunkRows o{-1, -1, -1};
    if (n < N) {
        const int64_t t = n / f.u, m = n - t * f.u;
        o.rn = (b * N + n) * f.heads + h;
        if (m == f.u - 1) o.rt = (b * f.seq + t) * f.heads + h;
        if (m == 0 && f.gw > 0) o.rg = (b * f.seq + t) * f.heads + h;
    }
    return o;
}

// G = inclusive cumsum over the chunk of its log-decays (warp 0; kBL == 32), gam = e^G, eL = e^{G_L - G}.
template <typename TG>
__device__ __forceinline__ void gate_scan(const TG *Gp, int64_t rg, float *sG, float *sgam, float *seL) {
    static_assert(kBL == 32, "the gate scans are warp scans");
    const int lane = threadIdx.x;
    float g = rg >= 0 ? ld(Gp + rg) : 0.f;
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

// The chunk's token rows into shared memory: k and b (.) k (and q, if sq) over dkp columns, w (.) v over
// dvp columns; zero outside the sequence and the heads' widths.  rn / rt: the chunk's row indices.
template <typename TI, typename TG>
__device__ __forceinline__ void load_chunk_inputs(const CoreParams &f, const int64_t *rn, const int64_t *rt, int dkp,
                                                  int dvp, float *sq, float *sk, float *ske, float *svw) {
    const int dk = (int)f.dk, dv = (int)f.dv;
    const TI *Q = static_cast<const TI *>(f.q), *K = static_cast<const TI *>(f.k), *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *Wr = static_cast<const TG *>(f.write);
    const TG *none = nullptr;
    auto krow = [&](int r, int d) -> int64_t { return rn[r] < 0 ? -1 : rn[r] * dk + d; };
    auto erow = [&](int r, int d) -> int64_t { return rn[r] * f.ew + (f.ew == 1 ? 0 : d); };
    auto vrow = [&](int r, int d) -> int64_t { return rn[r] < 0 ? -1 : rn[r] * dv + d; };
    auto wrow = [&](int r, int d) -> int64_t { return rn[r] * f.ww + (f.ww == 1 ? 0 : d); };
    gather_rows_pair(sk, ske, kLD, dk, dkp, K, krow, E, erow);
    if (sq)
        gather_rows<false>(sq, kLD, dk, dkp, Q,
                           [&](int r, int d) -> int64_t { return rt[r] < 0 ? -1 : rt[r] * dk + d; }, none, krow);
    gather_rows<true>(svw, kLD, dv, dvp, V, vrow, Wr, wrow);
}

// ---------------------------------------------------------------------------------------------------
// prep_kernel: one CTA per chunk (blockIdx.x = bh * nc + c)
// ---------------------------------------------------------------------------------------------------
constexpr int kPrepSmemFloats = 4 * kBL * kLD + 3 * kBL * kLS + 3 * kBL;

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads, 2) prep_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int64_t s_rn[kBL], s_rt[kBL];
    const CoreParams &f = p.f;
    const int dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t ch = blockIdx.x, bh = ch / p.nc, c = ch - bh * p.nc, b = bh / f.heads, h = bh - b * f.heads;
    float *sq = sm, *sk = sq + kBL * kLD, *ske = sk + kBL * kLD, *svw = ske + kBL * kLD;
    float *sA = svw + kBL * kLD, *sT = sA + kBL * kLS, *sTg = sT + kBL * kLS;
    float *sG = sTg + kBL * kLS, *sgam = sG + kBL, *seL = sgam + kBL;

    if (tid < 32) {
        const ChunkRows o = chunk_rows(f, b, h, c, tid);
        s_rn[tid] = o.rn;
        s_rt[tid] = o.rt;
        gate_scan(static_cast<const TG *>(f.g), o.rg, sG, sgam, seL);
    }
    __syncthreads();
    load_chunk_inputs<TI, TG>(f, s_rn, s_rt, dkp, dvp, sq, sk, ske, svw);
    __syncthreads();

    // A and T are the backward's alone: the forward (chunk_f32.cuh) passes them as null
    float *gA = p.A ? p.A + ch * kBL * kBL : nullptr, *gatt = p.att + ch * kBL * kBL;
    // A = strict_lower((b k) k^T D), att = lower(s q k^T D): q and b k (64 rows apart in shared memory)
    // as one stacked A operand, so each k fragment feeds both
    for_warp_tiles<1>(kBL, kBL, [&](int i0, int j0) {
        float a2[2][1][4] = {};
        warp_mma3_block<2, 2 * kBL, 1, kLD, 1, 1, kLD>(a2, i0, j0, dkp, sq, sk);
        const float(&aq)[1][4] = a2[0];
        const float(&aa)[1][4] = a2[1];
        frag_store(aa, i0, j0, kBL, kBL, [&](int i, int j, float a) {
            const float v = j < i ? a * expf(sG[i] - sG[j]) : 0.f;
            sA[i * kLS + j] = v;
            if (gA) gA[i * kBL + j] = v;
        });
        frag_store(aq, i0, j0, kBL, kBL, [&](int i, int j, float a) {
            gatt[i * kBL + j] = j <= i ? f.scale * a * expf(sG[i] - sG[j]) : 0.f;
        });
    });
    __syncthreads();
    // T = (I + A)^-1 by forward substitution down the rows, every column at once: the 8 threads of group
    // j = tid / 8 own column j, thread l holding T[l + 8m][j] (m < 4) in registers.  Row i's sum over k < i
    // of A[i][k] T[k][j] is split over the group (k = l mod 8; rows not yet reached still hold zero, and
    // A is zero on and above the diagonal) and closed with three shuffles.
    {
        const int j = tid >> 3, l = tid & 7;
        float tr[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < kBL; ++i) {
            float part = 0.f;
#pragma unroll
            for (int m = 0; m < 4; ++m) part = fmaf(sA[i * kLS + l + 8 * m], tr[m], part);
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            part += __shfl_xor_sync(0xffffffffu, part, 4);
            if (l == (i & 7)) tr[i >> 3] = (i == j ? 1.f : 0.f) - part;
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) sT[(l + 8 * m) * kLS + j] = tr[m];
    }
    __syncthreads();
    float *gT = p.T ? p.T + ch * kBL * kBL : nullptr;
    for (int idx = tid; idx < kBL * kBL; idx += kThreads) {
        const int i = idx / kBL, j = idx - i * kBL;
        const float t = sT[i * kLS + j];
        sTg[i * kLS + j] = t * sgam[j];
        if (gT) gT[idx] = t;
    }
    __syncthreads();
    // W = (T diag(gam)) (b k),  U = T (w v)
    float *gW = p.W + ch * kBL * dkp, *gU = p.U + ch * kBL * dvp;
    for_warp_tiles<4>(kBL, dkp, [&](int i0, int j0) {
        float acc[4][4] = {};
        warp_mma3<4, kLS, 1, kLD, 1>(acc, i0, j0, kBL, sTg, ske);
        frag_store(acc, i0, j0, kBL, dkp, [&](int i, int d, float a) { gW[i * dkp + d] = a; });
    });
    for_warp_tiles<4>(kBL, dvp, [&](int i0, int j0) {
        float acc[4][4] = {};
        warp_mma3<4, kLS, 1, kLD, 1>(acc, i0, j0, kBL, sT, svw);
        frag_store(acc, i0, j0, kBL, dvp, [&](int i, int d, float a) { gU[i * dvp + d] = a; });
    });
    float *gQ = p.Qp + ch * kBL * dkp, *gK = p.Kh + ch * kBL * dkp;
    for (int idx = tid; idx < kBL * dkp; idx += kThreads) {
        const int i = idx / dkp, d = idx - i * dkp;
        gQ[idx] = f.scale * sq[i * kLD + d] * sgam[i];
        gK[idx] = sk[i * kLD + d] * seL[i];
    }
    if (tid == 0) p.gl[ch] = sgam[kBL - 1];
}

// ---------------------------------------------------------------------------------------------------
// scan_kernel: one CTA per (batch x head = blockIdx.x, value slice = blockIdx.y).  Each chunk's operands
// are copied in asynchronously while the previous chunk still computes: a buffer is refilled for chunk
// c + 1 (forward) or c - 1 (reverse) as soon as its last reader of chunk c is done.
// ---------------------------------------------------------------------------------------------------
constexpr int kScanSmemFloats = kMaxD * kLS + 3 * kBL * kLD + 4 * kBL * kLS;

__global__ void __launch_bounds__(kThreads) scan_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh - b * f.heads, nc = p.nc;
    const int c0 = blockIdx.y * kSlice, wsl = dvp - c0 < kSlice ? dvp - c0 : kSlice;  // a multiple of 4
    float *sX = sm;                        // [kMaxD][kLS]: this slice of S, then of dS
    float *sW = sX + kMaxD * kLS, *sKh = sW + kBL * kLD, *sQp = sKh + kBL * kLD;
    float *satt = sQp + kBL * kLD, *sU = satt + kBL * kLS, *sV = sU + kBL * kLS, *sY1 = sV + kBL * kLS;
    auto sY = [&](int64_t c) { return (c & 1) ? sY1 : sU; };  // reverse: dy of even / odd chunks
    const int64_t sbase = bh * (int64_t)dk * dv;

    // the slice of a [dk][dv] state in global memory -> sX (zero outside dk x dv)
    auto load_state = [&](const float *src) {
        for (int idx = tid; idx < dkp * wsl; idx += kThreads) {
            const int d = idx / wsl, j = idx - d * wsl;
            sX[d * kLS + j] = (src && d < dk && c0 + j < dv) ? src[sbase + (int64_t)d * dv + c0 + j] : 0.f;
        }
    };
    // sX -> dst[c0 + j][d] (transposed): each thread reads 4 value columns of one key row (float4, no bank
    // conflicts) and writes them to 4 rows of dst, consecutive threads on consecutive keys (coalesced)
    auto store_T = [&](float *dst) {
        for (int idx = tid; idx < (wsl >> 2) * dkp; idx += kThreads) {
            const int jq = idx / dkp, d = idx - jq * dkp;
            const float4 x = *reinterpret_cast<const float4 *>(sX + d * kLS + 4 * jq);
            float *o = dst + (int64_t)(c0 + 4 * jq) * dkp + d;
            o[0] = x.x, o[dkp] = x.y, o[2 * dkp] = x.z, o[3 * dkp] = x.w;
        }
    };
    // chunk c's dy rows (this slice; zero off the read-out micro-steps) into `dst`
    auto issue_dy = [&](int64_t c, float *dst) {
        const int q4 = wsl >> 2;
        if (p.dy_vec) {
            for (int idx = tid; idx < kBL * q4; idx += kThreads) {
                const int r = idx / q4, q = idx - r * q4;
                const ChunkRows o = chunk_rows(f, b, h, c, r);
                const bool in = o.rt >= 0 && c0 + 4 * q < dv;  // the quads past dv (dvp > dv) read nothing
                const float *src = in ? p.dy + o.rt * dv + c0 + 4 * q : p.dy;
                ptx::cp_async16(ptx::smem_u32(dst + r * kLS + 4 * q), src, in ? 16u : 0u);
            }
        } else {
            for (int idx = tid; idx < kBL * wsl; idx += kThreads) {
                const int r = idx / wsl, j = idx - r * wsl;
                const ChunkRows o = chunk_rows(f, b, h, c, r);
                dst[r * kLS + j] = (o.rt >= 0 && c0 + j < dv) ? p.dy[o.rt * dv + c0 + j] : 0.f;
            }
        }
    };

    // ---- forward: S_c, V'_c.  Groups: [W, U](c), [K^](c) ----
    load_state(f.state_in);
    if (nc > 0) {
        copy_rows_async(sW, kLD, p.W + bh * nc * kBL * dkp, dkp, dkp);
        copy_rows_async(sU, kLS, p.U + bh * nc * kBL * dvp + c0, dvp, wsl);
        ptx::cp_async_commit();
        copy_rows_async(sKh, kLD, p.Kh + bh * nc * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    }
    for (int64_t c = 0; c < nc; ++c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        ptx::cp_async_wait<1>();  // W, U of chunk c
        __syncthreads();
        store_T(p.ST + ch * (int64_t)dvp * dkp);
        float *gV = p.Vp + ch * kBL * dvp + c0;
        for_warp_tiles<1>(kBL, wsl, [&](int i0, int j0) {  // V' = U - W S
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
            warp_mma3<1, kLD, 1, kLS, 1>(acc, i0, j0, dkp, sW, sX);
            frag_store(acc, i0, j0, kBL, wsl, [&](int i, int j, float a) {
                const float v = sU[i * kLS + j] - a;
                sV[i * kLS + j] = v;
                gV[i * dvp + j] = v;
            });
        });
        __syncthreads();
        if (c + 1 < nc) {
            copy_rows_async(sW, kLD, p.W + (ch + 1) * kBL * dkp, dkp, dkp);
            copy_rows_async(sU, kLS, p.U + (ch + 1) * kBL * dvp + c0, dvp, wsl);
        }
        ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // K^ of chunk c
        __syncthreads();
        for_warp_tiles<4>(dkp, wsl, [&](int d0, int j0) {  // S = gam_L S + K^^T V'
            float acc[4][4] = {};
            warp_mma3<4, 1, kLD, kLS, 1>(acc, d0, j0, kBL, sKh, sV);
            frag_store(acc, d0, j0, dkp, wsl, [&](int d, int j, float a) { sX[d * kLS + j] = fmaf(gl, sX[d * kLS + j], a); });
        });
        __syncthreads();
        if (c + 1 < nc) copy_rows_async(sKh, kLD, p.Kh + (ch + 1) * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    __syncthreads();

    // ---- reverse: dS_next_c, dV'_c, then dS0.  Groups: [att, K^, dy](c), [Q', W](c) ----
    load_state(p.dS_final);
    auto issue_a = [&](int64_t c) {
        const int64_t ch = bh * nc + c;
        copy_rows_async(satt, kLS, p.att + ch * kBL * kBL, kBL, kBL);
        copy_rows_async(sKh, kLD, p.Kh + ch * kBL * dkp, dkp, dkp);
        issue_dy(c, sY(c));
        ptx::cp_async_commit();
    };
    auto issue_b = [&](int64_t c) {
        const int64_t ch = bh * nc + c;
        copy_rows_async(sQp, kLD, p.Qp + ch * kBL * dkp, dkp, dkp);
        copy_rows_async(sW, kLD, p.W + ch * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    };
    if (nc > 0) {
        issue_a(nc - 1);
        issue_b(nc - 1);
    }
    for (int64_t c = nc - 1; c >= 0; --c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        const float *sy = sY(c);
        ptx::cp_async_wait<1>();  // att, K^, dy of chunk c
        __syncthreads();
        store_T(p.dSnT + ch * (int64_t)dvp * dkp);
        float *gdV = p.dVp + ch * kBL * dvp + c0;
        // dV' = att^T dy + K^ dS
        for_warp_tiles<1>(kBL, wsl, [&](int i0, int j0) {
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
            warp_mma3<1, 1, kLS, kLS, 1>(acc, i0, j0, kBL, satt, sy);
            warp_mma3<1, kLD, 1, kLS, 1>(acc, i0, j0, dkp, sKh, sX);
            frag_store(acc, i0, j0, kBL, wsl, [&](int i, int j, float a) {
                sV[i * kLS + j] = a;
                gdV[i * dvp + j] = a;
            });
        });
        __syncthreads();
        if (c > 0) issue_a(c - 1);
        else ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // Q', W of chunk c
        __syncthreads();
        // dS = gam_L dS + Q'^T dy - W^T dV'
        for_warp_tiles<4>(dkp, wsl, [&](int d0, int j0) {
            float ap[4][4] = {}, an[4][4] = {};
            warp_mma3<4, 1, kLD, kLS, 1>(ap, d0, j0, kBL, sQp, sy);
            warp_mma3<4, 1, kLD, kLS, 1>(an, d0, j0, kBL, sW, sV);
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int q = 0; q < 4; ++q) ap[n][q] -= an[n][q];
            frag_store(ap, d0, j0, dkp, wsl, [&](int d, int j, float a) { sX[d * kLS + j] = fmaf(gl, sX[d * kLS + j], a); });
        });
        __syncthreads();
        if (c > 0) issue_b(c - 1);
        else ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    for (int idx = tid; idx < dk * wsl; idx += kThreads) {
        const int d = idx / wsl, j = idx - d * wsl;
        if (c0 + j < dv) p.dS0[sbase + (int64_t)d * dv + c0 + j] = sX[d * kLS + j];
    }
}

// ---------------------------------------------------------------------------------------------------
// scan_wide_kernel: one 16-warp CTA per (batch x head = blockIdx.x) over every value column, for calls with
// more (head, slice) pairs than two per SM.  The same passes, products and stores as scan_kernel, every
// output element accumulated in the same order (so both forms give the same bits); each chunk operand is
// read once per head instead of once per slice, and the warp tiles are larger.
// ---------------------------------------------------------------------------------------------------
constexpr int kScanWideSmemFloats = kMaxD * kWS + 6 * kBL * kWS + kBL * kLS;

__global__ void __launch_bounds__(kWideThreads, 1) scan_wide_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int warp = tid >> 5;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh - b * f.heads, nc = p.nc;
    float *sX = sm;                                    // [kMaxD][kWS]: S, then dS
    float *sW = sX + kMaxD * kWS, *sQp = sW + kBL * kWS, *sKh = sQp + kBL * kWS;
    float *sU = sKh + kBL * kWS, *sY1 = sU + kBL * kWS, *sV = sY1 + kBL * kWS;
    float *satt = sV + kBL * kWS;                      // [kBL][kLS]
    auto sY = [&](int64_t c) { return (c & 1) ? sY1 : sU; };  // reverse: dy of even / odd chunks
    const int64_t sbase = bh * (int64_t)dk * dv;

    auto load_state = [&](const float *src) {
        for (int idx = tid; idx < dkp * dvp; idx += kWideThreads) {
            const int d = idx / dvp, j = idx - d * dvp;
            sX[d * kWS + j] = (src && d < dk && j < dv) ? src[sbase + (int64_t)d * dv + j] : 0.f;
        }
    };
    // sX -> dst[j][d] (transposed, [dvp][dkp]): float4 reads of 4 value columns of one key row,
    // consecutive threads on consecutive keys (coalesced writes)
    auto store_T = [&](float *dst) {
        for (int idx = tid; idx < (dvp >> 2) * dkp; idx += kWideThreads) {
            const int jq = idx / dkp, d = idx - jq * dkp;
            const float4 x = *reinterpret_cast<const float4 *>(sX + d * kWS + 4 * jq);
            float *o = dst + (int64_t)(4 * jq) * dkp + d;
            o[0] = x.x, o[dkp] = x.y, o[2 * dkp] = x.z, o[3 * dkp] = x.w;
        }
    };
    auto issue_dy = [&](int64_t c, float *dst) {
        const int q4 = dvp >> 2;
        if (p.dy_vec) {
            for (int idx = tid; idx < kBL * q4; idx += kWideThreads) {
                const int r = idx / q4, q = idx - r * q4;
                const ChunkRows o = chunk_rows(f, b, h, c, r);
                const bool in = o.rt >= 0 && 4 * q < dv;
                const float *src = in ? p.dy + o.rt * dv + 4 * q : p.dy;
                ptx::cp_async16(ptx::smem_u32(dst + r * kWS + 4 * q), src, in ? 16u : 0u);
            }
        } else {
            for (int idx = tid; idx < kBL * dvp; idx += kWideThreads) {
                const int r = idx / dvp, j = idx - r * dvp;
                const ChunkRows o = chunk_rows(f, b, h, c, r);
                dst[r * kWS + j] = (o.rt >= 0 && j < dv) ? p.dy[o.rt * dv + j] : 0.f;
            }
        }
    };

    // [kBL x dvp] tiles (V', dV'): rows r0, 16 columns from c1; [dkp x dvp] tiles (S, dS): 32 x 32
    const int ncb = (dvp + 15) >> 4;
    const bool t1 = warp < 2 * ncb;
    const int r0 = (warp & 1) * 16, c1 = (warp >> 1) * 16;
    const int nsb = (dvp + 31) >> 5;
    const bool t3 = warp < ((dkp + 31) >> 5) * nsb;
    const int d0 = (warp / nsb) * 32, c3 = (warp % nsb) * 32;

    // ---- forward: S_c, V'_c.  Groups: [W (rows), U](c), [K^ (transposed)](c) ----
    load_state(f.state_in);
    copy_rows<kWideThreads>(sW, kLD, p.W + bh * nc * kBL * dkp, dkp, dkp);
    copy_rows<kWideThreads>(sU, kWS, p.U + bh * nc * kBL * dvp, dvp, dvp);
    ptx::cp_async_commit();
    copy_rows<kWideThreads>(sKh, kWS, p.Kh + bh * nc * kBL * dkp, dkp, dkp);
    ptx::cp_async_commit();
    for (int64_t c = 0; c < nc; ++c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        ptx::cp_async_wait<1>();  // W, U of chunk c
        __syncthreads();
        store_T(p.ST + ch * (int64_t)dvp * dkp);
        float *gV = p.Vp + ch * kBL * dvp;
        if (t1) {  // V' = U - W S
            float acc[1][2][4] = {};
            warp_mma3_block<1, 16, 2, kLD, 1, kWS>(acc, r0, c1, dkp, sW, sX);
            block_store<1, 16, 2>(acc, r0, c1, kBL, dvp, [&](int i, int j, float a) {
                const float v = sU[i * kWS + j] - a;
                sV[i * kWS + j] = v;
                gV[i * dvp + j] = v;
            });
        }
        __syncthreads();
        if (c + 1 < nc) {
            copy_rows<kWideThreads>(sW, kLD, p.W + (ch + 1) * kBL * dkp, dkp, dkp);
            copy_rows<kWideThreads>(sU, kWS, p.U + (ch + 1) * kBL * dvp, dvp, dvp);
        }
        ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // K^ of chunk c
        __syncthreads();
        if (t3) {  // S = gam_L S + K^^T V'
            float a3[2][4][4] = {};
            warp_mma3_block<2, 16, 4, 1, kWS, kWS>(a3, d0, c3, kBL, sKh, sV);
            block_store<2, 16, 4>(a3, d0, c3, dkp, dvp,
                                  [&](int d, int j, float a) { sX[d * kWS + j] = fmaf(gl, sX[d * kWS + j], a); });
        }
        __syncthreads();
        if (c + 1 < nc) copy_rows<kWideThreads>(sKh, kWS, p.Kh + (ch + 1) * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    __syncthreads();

    // ---- reverse: dS_next_c, dV'_c, then dS0.  Groups: [att, K^ (rows), dy](c), [Q', W (transposed)](c) ----
    load_state(p.dS_final);
    auto issue_a = [&](int64_t c) {
        const int64_t ch = bh * nc + c;
        copy_rows<kWideThreads>(satt, kLS, p.att + ch * kBL * kBL, kBL, kBL);
        copy_rows<kWideThreads>(sKh, kLD, p.Kh + ch * kBL * dkp, dkp, dkp);
        issue_dy(c, sY(c));
        ptx::cp_async_commit();
    };
    auto issue_b = [&](int64_t c) {
        const int64_t ch = bh * nc + c;
        copy_rows<kWideThreads>(sQp, kWS, p.Qp + ch * kBL * dkp, dkp, dkp);
        copy_rows<kWideThreads>(sW, kWS, p.W + ch * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    };
    if (nc > 0) {
        issue_a(nc - 1);
        issue_b(nc - 1);
    }
    for (int64_t c = nc - 1; c >= 0; --c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        const float *sy = sY(c);
        ptx::cp_async_wait<1>();  // att, K^, dy of chunk c
        __syncthreads();
        store_T(p.dSnT + ch * (int64_t)dvp * dkp);
        float *gdV = p.dVp + ch * kBL * dvp;
        if (t1) {  // dV' = att^T dy + K^ dS
            float acc[1][2][4] = {};
            warp_mma3_block<1, 16, 2, 1, kLS, kWS>(acc, r0, c1, kBL, satt, sy);
            warp_mma3_block<1, 16, 2, kLD, 1, kWS>(acc, r0, c1, dkp, sKh, sX);
            block_store<1, 16, 2>(acc, r0, c1, kBL, dvp, [&](int i, int j, float a) {
                sV[i * kWS + j] = a;
                gdV[i * dvp + j] = a;
            });
        }
        __syncthreads();
        if (c > 0) issue_a(c - 1);
        else ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // Q', W of chunk c
        __syncthreads();
        if (t3) {  // dS = gam_L dS + Q'^T dy - W^T dV', in two 32 x 16 halves (two accumulators each)
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                const int cj = c3 + 16 * hf;
                float ap[2][2][4] = {}, an[2][2][4] = {};
                warp_mma3_block<2, 16, 2, 1, kWS, kWS>(ap, d0, cj, kBL, sQp, sy);
                warp_mma3_block<2, 16, 2, 1, kWS, kWS>(an, d0, cj, kBL, sW, sV);
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int n = 0; n < 2; ++n)
#pragma unroll
                        for (int q = 0; q < 4; ++q) ap[m][n][q] -= an[m][n][q];
                block_store<2, 16, 2>(ap, d0, cj, dkp, dvp,
                                      [&](int d, int j, float a) { sX[d * kWS + j] = fmaf(gl, sX[d * kWS + j], a); });
            }
        }
        __syncthreads();
        if (c > 0) issue_b(c - 1);
        else ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    __syncthreads();
    for (int idx = tid; idx < dk * dv; idx += kWideThreads) {
        const int d = idx / dv, j = idx - d * dv;
        p.dS0[sbase + (int64_t)d * dv + j] = sX[d * kWS + j];
    }
}

// ---------------------------------------------------------------------------------------------------
// grad_kernel: one CTA per chunk (blockIdx.x = bh * nc + c)
// ---------------------------------------------------------------------------------------------------
constexpr int kGradSmemFloats = 10 * kBL * kLD + 7 * kBL * kLS + 3 * kBL * (kBL + 1) + 6 * kBL + 16;

template <typename TI, typename TG>
__global__ void __launch_bounds__(kThreads) grad_kernel(const Params p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int64_t s_rn[kBL], s_rt[kBL];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int64_t ch = blockIdx.x, bh = ch / p.nc, c = ch - bh * p.nc, b = bh / f.heads, h = bh - b * f.heads;
    constexpr int kTile = kBL * kLD, kSq = kBL * kLS, kRed = kBL + 1;
    float *t0 = sm, *t1 = t0 + kTile, *t2 = t1 + kTile, *t3 = t2 + kTile, *t4 = t3 + kTile;
    float *t5 = t4 + kTile, *t6 = t5 + kTile, *t7 = t6 + kTile, *t8 = t7 + kTile, *t9 = t8 + kTile;
    float *sT = t9 + kTile, *sA = sT + kSq, *satt = sA + kSq, *sdatt = satt + kSq, *sdT = sdatt + kSq;
    float *sX = sdT + kSq, *sM = sX + kSq;
    float *redG = sM + kSq, *redE = redG + kBL * kRed, *redW = redE + kBL * kRed;
    float *sG = redW + kBL * kRed, *sgam = sG + kBL, *seL = sgam + kBL, *sdG = seL + kBL;
    float *se1 = sdG + kBL, *sw1 = se1 + kBL, *sscal = sw1 + kBL;

    const TI *V = static_cast<const TI *>(f.v);
    const TG *E = static_cast<const TG *>(f.erase), *Wr = static_cast<const TG *>(f.write);

    // 32-column groups of the [kBL][dkp] and [kBL][dvp] results (the row-sum tables' columns)
    const int ngk = (dkp + 31) >> 5, ngv = (dvp + 31) >> 5;

    // ---- asynchronous: V', dV', T, A, att and the first block of S^T / dS_next^T ----
    const float *gST = p.ST + ch * (int64_t)dvp * dkp, *gdS = p.dSnT + ch * (int64_t)dvp * dkp;
    auto issue_block = [&](int kb) {
        const int jb = kb * kBL, jn = dvp - jb < kBL ? dvp - jb : kBL, c4 = dkp >> 2;
        float *bs = (kb & 1) ? t8 : t3, *bd = (kb & 1) ? t9 : t4;
        for (int idx = tid; idx < jn * c4; idx += kThreads) {
            const int r = idx / c4, q = idx - r * c4;
            ptx::cp_async16(ptx::smem_u32(bs + r * kLD + 4 * q), gST + (int64_t)(jb + r) * dkp + 4 * q, 16u);
            ptx::cp_async16(ptx::smem_u32(bd + r * kLD + 4 * q), gdS + (int64_t)(jb + r) * dkp + 4 * q, 16u);
        }
    };
    copy_rows_async(t1, kLD, p.Vp + ch * kBL * dvp, dvp, dvp);
    copy_rows_async(t2, kLD, p.dVp + ch * kBL * dvp, dvp, dvp);
    copy_rows_async(sT, kLS, p.T + ch * kBL * kBL, kBL, kBL);
    copy_rows_async(sA, kLS, p.A + ch * kBL * kBL, kBL, kBL);
    copy_rows_async(satt, kLS, p.att + ch * kBL * kBL, kBL, kBL);
    issue_block(0);
    ptx::cp_async_commit();

    if (tid < 32) {
        const ChunkRows o = chunk_rows(f, b, h, c, tid);
        s_rn[tid] = o.rn;
        s_rt[tid] = o.rt;
        gate_scan(static_cast<const TG *>(f.g), o.rg, sG, sgam, seL);
        se1[tid] = (o.rn >= 0 && f.ew == 1) ? ld(E + o.rn) : 0.f;
        sw1[tid] = (o.rn >= 0 && f.ww == 1) ? ld(Wr + o.rn) : 0.f;
    }
    __syncthreads();
    // dy -> t0 (read-out micro-steps only); k -> t5, b k -> t6, w v -> t7
    gather_rows<false>(t0, kLD, dv, dvp, p.dy, [&](int r, int j) -> int64_t { return s_rt[r] < 0 ? -1 : s_rt[r] * dv + j; },
                static_cast<const float *>(nullptr), [&](int, int) -> int64_t { return 0; });
    load_chunk_inputs<TI, TG>(f, s_rn, s_rt, dkp, dvp, nullptr, t5, t6, t7);

    // ---- phase 1: the products with S and dS_next, block by block of 32 value rows, on the tensor
    // cores: warp w holds the 16 x 32 tile (rows (w % 2) * 16, columns (w / 2) * 32) of dQ', dV' S^T, dK^ ----
    const int wi0 = ((tid >> 5) & 1) * 16, wj0 = (tid >> 6) * 32;
    const bool wown = wj0 < dkp;
    float aq[4][4] = {}, aw[4][4] = {}, ak[4][4] = {};
    float dgl_part = 0.f;
    const int nb = (dvp + kBL - 1) / kBL;
    for (int kb = 0; kb < nb; ++kb) {
        const int jb = kb * kBL, jn = dvp - jb < kBL ? dvp - jb : kBL;
        if (kb + 1 < nb) issue_block(kb + 1);
        ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // block kb (and, with it, everything issued before)
        __syncthreads();
        const float *bs = (kb & 1) ? t8 : t3, *bd = (kb & 1) ? t9 : t4;
        for (int idx = tid; idx < jn * (dkp >> 2); idx += kThreads) {  // <dS_next, S> over the block
            const int r = idx / (dkp >> 2), q = idx - r * (dkp >> 2);
            const float4 x = *reinterpret_cast<const float4 *>(bs + r * kLD + 4 * q);
            const float4 y = *reinterpret_cast<const float4 *>(bd + r * kLD + 4 * q);
            dgl_part += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
        }
        if (wown) {
            warp_mma3<4, kLD, 1, kLD, 1, 1>(aq, wi0, wj0, jn, t0 + jb, bs);  // dy S^T
            warp_mma3<4, kLD, 1, kLD, 1, 1>(aw, wi0, wj0, jn, t2 + jb, bs);  // dV' S^T
            warp_mma3<4, kLD, 1, kLD, 1, 1>(ak, wi0, wj0, jn, t1 + jb, bd);  // V' dS_next^T
        }
        __syncthreads();
    }
    // datt = lower(dy V'^T), on the tensor cores like the other products
    for_warp_tiles<1>(kBL, kBL, [&](int i0, int j0) {
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        warp_mma3<1, kLD, 1, 1, kLD, 1>(acc, i0, j0, dvp, t0, t1);
        frag_store(acc, i0, j0, kBL, kBL, [&](int i, int j, float a) { sdatt[i * kLS + j] = j <= i ? a : 0.f; });
    });
    {
        float v = dgl_part;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((tid & 31) == 0) sscal[tid >> 5] = v;
    }
    __syncthreads();
    // park dQ' -> t0, dW = -dV' S^T -> t1, dK^ -> t3; q -> t4
    if (wown) {
        frag_store(aq, wi0, wj0, kBL, dkp, [&](int i, int d, float a) { t0[i * kLD + d] = a; });
        frag_store(aw, wi0, wj0, kBL, dkp, [&](int i, int d, float a) { t1[i * kLD + d] = -a; });
        frag_store(ak, wi0, wj0, kBL, dkp, [&](int i, int d, float a) { t3[i * kLD + d] = a; });
    }
    {
        const TI *Q = static_cast<const TI *>(f.q);
        gather_rows<false>(t4, kLD, dk, dkp, Q, [&](int r, int d) -> int64_t { return s_rt[r] < 0 ? -1 : s_rt[r] * dk + d; },
                    static_cast<const float *>(nullptr), [&](int, int) -> int64_t { return 0; });
    }
    __syncthreads();

    // ---- phase 2, on the tensor cores; every [kBL][dkp] result in the phase-1 warp tiles ----
    const int lane = tid & 31, fg = lane >> 2, ft = lane & 3;
    // Row sums of a warp tile: lane (fg, ft) holds rows fg and fg + 8; the four lanes of a row add up and
    // lane ft == 0 files the tile's share under its 32-column group.
    auto file_rows = [&](float *red, int i0, int j0, float r0, float r1) {
        r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
        r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
        r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
        r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
        if (ft == 0) {
            red[(i0 + fg) * kRed + (j0 >> 5)] = r0;
            red[(i0 + fg + 8) * kRed + (j0 >> 5)] = r1;
        }
    };
    // dT = dV' (w v)^T + dW (b k)^T diag(gam)
    for_warp_tiles<1>(kBL, kBL, [&](int i0, int j0) {
        float a1[1][4] = {{0.f, 0.f, 0.f, 0.f}}, a2[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        warp_mma3<1, kLD, 1, 1, kLD, 1>(a1, i0, j0, dvp, t2, t7);
        warp_mma3<1, kLD, 1, 1, kLD, 1>(a2, i0, j0, dkp, t1, t6);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = i0 + fg + (q >> 1) * 8, j = j0 + 2 * ft + (q & 1);
            sdT[i * kLS + j] = fmaf(sgam[j], a2[0][q], a1[0][q]);
        }
    });
    // d(w v) = T^T dV'  ->  d_v = w d(wv), d_write = v d(wv)
    for_warp_tiles<4>(kBL, dvp, [&](int i0, int j0) {
        float acc[4][4] = {};
        warp_mma3<4, 1, kLS, kLD, 1, 1>(acc, i0, j0, kBL, sT, t2);
        float vv[4][4], wv[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // every load first, then the arithmetic
                const int i = i0 + fg + (q >> 1) * 8, d = j0 + 8 * n + 2 * ft + (q & 1);
                const int64_t rn = s_rn[i];
                const int64_t o = (rn >= 0 && d < dv) ? rn * dv + d : 0;
                vv[n][q] = ld(V + o);
                wv[n][q] = f.ww == 1 ? sw1[i] : ld(Wr + o);
            }
        float r0 = 0.f, r1 = 0.f;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = i0 + fg + (q >> 1) * 8, d = j0 + 8 * n + 2 * ft + (q & 1);
                const int64_t rn = s_rn[i];
                const bool in = rn >= 0 && d < dv;
                const float dwv = vv[n][q] * acc[n][q];
                if (in) {
                    p.dv[rn * dv + d] = wv[n][q] * acc[n][q];
                    if (f.ww != 1) p.dw[rn * dv + d] = dwv;
                }
                if (in) (q < 2 ? r0 : r1) += dwv;
            }
        if (f.ww == 1) file_rows(redW, i0, j0, r0, r1);
    });
    // d(b k gam) = T^T dW: its share of d(b k) (ake, kept in registers) and of dG (rows gp0 / gp1)
    float ake[4][4] = {}, gp0 = 0.f, gp1 = 0.f;
    if (wown) {
        warp_mma3<4, 1, kLS, kLD, 1, 1>(ake, wi0, wj0, kBL, sT, t1);
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = wi0 + fg + (q >> 1) * 8, d = wj0 + 8 * n + 2 * ft + (q & 1);
                const float gm = sgam[i];
                const float x = gm * ake[n][q] * t6[i * kLD + d];
                (q < 2 ? gp0 : gp1) += d < dkp ? x : 0.f;
                ake[n][q] *= gm;
            }
    }
    __syncthreads();
    // dA = strict_lower(-T^T dT T^T): X = T^T dT, then dA = -X T^T; Fa = dA D -> sdT, dA A -> sM
    for_warp_tiles<1>(kBL, kBL, [&](int i0, int j0) {
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        warp_mma3<1, 1, kLS, kLS, 1, 1>(acc, i0, j0, kBL, sT, sdT);
        frag_store(acc, i0, j0, kBL, kBL, [&](int i, int j, float a) { sX[i * kLS + j] = a; });
    });
    __syncthreads();
    for_warp_tiles<1>(kBL, kBL, [&](int i0, int j0) {
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        warp_mma3<1, kLS, 1, 1, kLS, 1>(acc, i0, j0, kBL, sX, sT);
        frag_store(acc, i0, j0, kBL, kBL, [&](int i, int j, float a) {
            const float da = j < i ? -a : 0.f;
            sdT[i * kLS + j] = j < i ? da * expf(sG[i] - sG[j]) : 0.f;
            sM[i * kLS + j] = da * sA[i * kLS + j];
        });
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
        float sacc = 0.f;
        for (int j = 0; j < kBL; ++j)
            sacc += (sM[tid * kLS + j] + satt[tid * kLS + j]) - (sM[j * kLS + tid] + satt[j * kLS + tid]);
        sdG[tid] = sacc;
    }
    // d_q, d_k, d_erase
    float khat_part = 0.f;
    if (wown) {
        float aqk[4][4] = {}, akk[4][4] = {};
        warp_mma3<4, kLS, 1, kLD, 1, 1>(aqk, wi0, wj0, kBL, sdatt, t5);  // F k
        warp_mma3<4, 1, kLS, kLD, 1, 1>(akk, wi0, wj0, kBL, sdatt, t4);  // F^T q
        warp_mma3<4, 1, kLS, kLD, 1, 1>(akk, wi0, wj0, kBL, sdT, t6);    // Fa^T (b k)
        warp_mma3<4, kLS, 1, kLD, 1, 1>(ake, wi0, wj0, kBL, sdT, t5);    // Fa k
        float ev[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = wi0 + fg + (q >> 1) * 8, d = wj0 + 8 * n + 2 * ft + (q & 1);
                const int64_t rn = s_rn[i];
                ev[n][q] = f.ew == 1 ? se1[i] : ld(E + ((rn >= 0 && d < dk) ? rn * dk + d : 0));
            }
        float e0 = 0.f, e1 = 0.f;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = wi0 + fg + (q >> 1) * 8, d = wj0 + 8 * n + 2 * ft + (q & 1);
                if (d >= dkp) continue;
                const int o = i * kLD + d;
                const float sg = f.scale * sgam[i], el = seL[i];
                const int64_t rn = s_rn[i], rt = s_rt[i];
                const float dqp = t0[o], dkh = t3[o], qv = t4[o], kv = t5[o];
                const float dq = fmaf(sg, dqp, aqk[n][q]);
                const float kh = el * dkh * kv;
                (q < 2 ? gp0 : gp1) += sg * dqp * qv - kh;
                khat_part += kh;
                const bool in = rn >= 0 && d < dk;
                const float e = in ? ev[n][q] : 0.f;
                const float dkv = fmaf(el, dkh, fmaf(e, ake[n][q], akk[n][q]));
                const float de = kv * ake[n][q];
                if (f.ew == 1) (q < 2 ? e0 : e1) += in ? de : 0.f;
                else if (in) p.de[rn * dk + d] = de;
                if (in) {
                    p.dk[rn * dk + d] = dkv;
                    if (rt >= 0) p.dq[rt * dk + d] = dq;
                }
            }
        file_rows(redG, wi0, wj0, gp0, gp1);
        if (f.ew == 1) file_rows(redE, wi0, wj0, e0, e1);
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
        const ChunkRows o = chunk_rows(f, b, h, c, i);
        float dG = sdG[i];
        for (int g = 0; g < ngk; ++g) dG += redG[i * kRed + g];
        if (i == kBL - 1) {
            float dgl = 0.f, kh = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) dgl += sscal[w], kh += sscal[8 + w];
            dG += kh + sgam[kBL - 1] * dgl;
        }
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const float x = __shfl_down_sync(0xffffffffu, dG, s);
            if (i + s < 32) dG += x;
        }
        if (o.rg >= 0) p.dg[o.rg] = dG;
        if (o.rn >= 0) {
            if (f.ew == 1) {
                float s = 0.f;
                for (int g = 0; g < ngk; ++g) s += redE[i * kRed + g];
                p.de[o.rn] = s;
            }
            if (f.ww == 1) {
                float s = 0.f;
                for (int g = 0; g < ngv; ++g) s += redW[i * kRed + g];
                p.dw[o.rn] = s;
            }
        }
    }
}

}  // namespace bwdc
}  // namespace dc
