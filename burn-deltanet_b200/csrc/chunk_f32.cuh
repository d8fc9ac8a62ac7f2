// chunk_f32.cuh — the chunked prefill at the reference's own precision: fp32 (or bf16) q/k/v, any
// dk, dv <= 128, a log-decay per head or none, any erase / write width and any n_householder.  It serves
// every call the bf16 tensor-core kernels (chunk_tc.cuh, chunk_split.cuh) do not take and that has a
// workspace, in place of the CUDA-core kernel (chunk_simt.cuh).
//
// The chunk algorithm of the reference (src/delta/chunk.rs:103-205, the forward of
// src/delta/chunk_recalculated/forward.rs:154-439) on the folded sequence, cut into chunks of kBL = 32
// micro-steps; chunking is exact, so the result does not depend on the caller's chunk_len.  Per chunk,
// with S the state at its start (G = cumsum(g), gam = e^G, D_ij = e^{G_i - G_j}):
//
//   T = (I + strict_lower((b (.) k) k^T (.) D))^-1,  W = T (b (.) k (.) gam),  U = T (w (.) v)
//   att = lower(s q k^T (.) D),  Q' = s q (.) gam,  K^ = k (.) e^{G_L - G}
//   V' = U - W S,  y = Q' S + att V',  S_next = gam_L S + K^^T V'
//
// Two kernels over a workspace:
//   bwdc::prep_kernel  one CTA per (batch x head, chunk), chunk-parallel: W, U, att, Q', K^, gam_L (the
//                      backward's own prep, without the two arrays only the backward reads);
//   fwd_scan_kernel    one CTA per (batch x head, 32 value columns): the chunks in order, the state's
//                      slice in shared memory; y of the slice's columns and the final state;
//   fwd_scan_wide_kernel  the same with one CTA per (batch x head) over every value column, for calls
//                      with more (head, slice) pairs than two per SM.
// Every product runs on the tensor cores as three mma.sync m16n8k8 tf32 products of split operands
// (big x big + big x small + small x big, about 2^-20 relative), which holds the reference's 1e-4 with
// fp32 inputs over hundreds of chunks.
#pragma once

#include "bwd_chunk.cuh"

namespace dc {
namespace f32c {

using bwdc::kBL;
using bwdc::kLD;
using bwdc::kLS;
using bwdc::kMaxD;
using bwdc::kSlice;
using bwdc::kThreads;
using bwdc::block_store;
using bwdc::warp_mma3_block;


// Whether the forward scan serves these shapes (the prep kernel has the same limits).
inline bool applies(const CoreParams &p, uint32_t flags) {
    if (flags & 0x3u) return false;  // DC_FLAG_FORCE_SIMT, DC_FLAG_RECURRENT
    if (p.gw > 1) return false;      // per-channel log-decays put D inside the key sums
    if (p.dk < 1 || p.dv < 1 || p.dk > kMaxD || p.dv > kMaxD) return false;
    const int64_t nc = (p.seq * p.u + kBL - 1) / kBL;
    return p.batch * p.heads <= 0x7fffffffLL && p.batch * p.heads * nc <= 0x7fffffffLL;
}

// Per-chunk arrays of the workspace, in floats (each a multiple of 4: 16-byte aligned regions).
struct Plan {
    int64_t nc, nch;
    int32_t dkp, dvp, nslice;
    uint64_t w, uv, sq, gl, total_bytes;
};
inline Plan plan(const CoreParams &p) {
    Plan pl{};
    pl.nc = (p.seq * p.u + kBL - 1) / kBL;
    pl.nch = p.batch * p.heads * pl.nc;
    pl.dkp = (int32_t)((p.dk + 7) / 8 * 8);
    pl.dvp = (int32_t)((p.dv + 7) / 8 * 8);
    pl.nslice = (pl.dvp + kSlice - 1) / kSlice;
    pl.w = (uint64_t)pl.nch * kBL * pl.dkp;
    pl.uv = (uint64_t)pl.nch * kBL * pl.dvp;
    pl.sq = (uint64_t)pl.nch * kBL * kBL;
    pl.gl = ((uint64_t)pl.nch + 3) / 4 * 4;
    pl.total_bytes = 4ull * (3 * pl.w + pl.uv + pl.sq + pl.gl);
    return pl;
}

using bwdc::kAS;
using bwdc::kWS;
constexpr int kWideSmemFloats = kMaxD * kWS + 2 * kBL * kLD + 3 * kBL * kWS + kBL * kAS;

// The sliced scan's shared memory: the state slice [kMaxD][kLS]; W, Q' [kBL][kLD]; K^ [kBL][kWS];
// att [kBL][kAS]; U, V' [kBL][kLS].
constexpr int kScanSmemFloats = kMaxD * kLS + 2 * kBL * kLD + kBL * kWS + kBL * kAS + 2 * kBL * kLS;

// fwd_scan_kernel: blockIdx.x = batch x head, blockIdx.y = value slice of kSlice columns.
//
// Per chunk, two barrier intervals:
//   1. V' = U - W S into shared memory and Q' S into the warp's registers (one 16 x 8 tile per warp);
//   2. y = Q' S + att V' to HBM (read-out rows only), and S = gam_L S + K^^T V' in place.
// Operands arrive by cp.async in two groups, each refilled for chunk c + 1 as soon as chunk c's last
// reader is past a barrier: [W, U, Q'] after interval 1, [att, K^] after interval 2.
template <typename TO>
__global__ void __launch_bounds__(kThreads) fwd_scan_kernel(const bwdc::Params p) {
    using namespace bwdc;
    extern __shared__ __align__(16) float sm[];
    __shared__ int64_t s_rt[kBL];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int warp = tid >> 5;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh - b * f.heads, nc = p.nc;
    const int c0 = blockIdx.y * kSlice, wsl = dvp - c0 < kSlice ? dvp - c0 : kSlice;  // a multiple of 4
    float *sX = sm;                                                                   // [kMaxD][kLS]
    float *sW = sX + kMaxD * kLS, *sQp = sW + kBL * kLD;                              // [kBL][kLD]
    float *sKh = sQp + kBL * kLD;                                                     // [kBL][kWS]
    float *satt = sKh + kBL * kWS;                                                    // [kBL][kAS]
    float *sU = satt + kBL * kAS, *sV = sU + kBL * kLS;                               // [kBL][kLS]
    const int64_t sbase = bh * (int64_t)dk * dv;
    TO *Y = static_cast<TO *>(f.y);

    // this slice of S0 (zero outside dk x dv)
    for (int idx = tid; idx < dkp * wsl; idx += kThreads) {
        const int d = idx / wsl, j = idx - d * wsl;
        sX[d * kLS + j] = (d < dk && c0 + j < dv) ? f.state_in[sbase + (int64_t)d * dv + c0 + j] : 0.f;
    }
    auto issue_wuq = [&](int64_t ch) {
        copy_rows_async(sW, kLD, p.W + ch * kBL * dkp, dkp, dkp);
        copy_rows_async(sU, kLS, p.U + ch * kBL * dvp + c0, dvp, wsl);
        copy_rows_async(sQp, kLD, p.Qp + ch * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    };
    auto issue_ak = [&](int64_t ch) {
        copy_rows_async(satt, kAS, p.att + ch * kBL * kBL, kBL, kBL);
        copy_rows_async(sKh, kWS, p.Kh + ch * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    };
    issue_wuq(bh * nc);
    issue_ak(bh * nc);

    // The warp's tile of the [kBL x wsl] chunk outputs (V', y): at most one per warp (2 x 4 tiles of
    // 16 x 8 for 8 warps).  State-update tiles: 16 key rows x 32 columns, dealt round robin.
    const int tn = (wsl + 7) >> 3;
    const bool has_tile = warp < 2 * tn;
    const int i0 = has_tile ? (warp / tn) * 16 : 0, j0 = has_tile ? (warp % tn) * 8 : 0;

    for (int64_t c = 0; c < nc; ++c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        ptx::cp_async_wait<1>();  // W, U, Q' of chunk c
        __syncthreads();
        if (tid < kBL) s_rt[tid] = chunk_rows(f, b, h, c, tid).rt;
        // ---- 1. [W; Q'] S (stacked in shared memory): V' = U - W S, Q' S kept in registers ----
        float ay[1][1][4] = {};
        if (has_tile) {
            float a1[2][1][4] = {};
            warp_mma3_block<2, kBL, 1, kLD, 1, kLS>(a1, i0, j0, dkp, sW, sX);
            block_store<1, 16, 1>(reinterpret_cast<const float(&)[1][1][4]>(a1[0]), i0, j0, kBL, wsl,
                                  [&](int i, int j, float a) { sV[i * kLS + j] = sU[i * kLS + j] - a; });
#pragma unroll
            for (int q = 0; q < 4; ++q) ay[0][0][q] = a1[1][0][q];
        }
        __syncthreads();
        if (c + 1 < nc) issue_wuq(ch + 1);
        else ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // att, K^ of chunk c
        __syncthreads();
        // ---- 2. y = Q' S + att V';  S = gam_L S + K^^T V' ----
        if (has_tile) {
            warp_mma3_block<1, 16, 1, kAS, 1, kLS>(ay, i0, j0, kBL, satt, sV);
            block_store<1, 16, 1>(ay, i0, j0, kBL, wsl, [&](int i, int j, float a) {
                const int64_t rt = s_rt[i];
                if (rt >= 0 && c0 + j < dv) st(Y + rt * dv + c0 + j, a);
            });
        }
        for_warp_tiles<4>(dkp, wsl, [&](int d0, int jj) {
            float acc[1][4][4] = {};
            warp_mma3_block<1, 16, 4, 1, kWS, kLS>(acc, d0, jj, kBL, sKh, sV);
            block_store<1, 16, 4>(acc, d0, jj, dkp, wsl,
                                  [&](int d, int j, float a) { sX[d * kLS + j] = fmaf(gl, sX[d * kLS + j], a); });
        });
        __syncthreads();
        if (c + 1 < nc) issue_ak(ch + 1);
        else ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    for (int idx = tid; idx < dk * wsl; idx += kThreads) {
        const int d = idx / wsl, j = idx - d * wsl;
        if (c0 + j < dv) f.state_out[sbase + (int64_t)d * dv + c0 + j] = sX[d * kLS + j];
    }
}

// ---------------------------------------------------------------------------------------------------
// The full-width scan: one CTA per (batch x head) holding the whole [dk x dv] state, for calls with more
// (head, slice) pairs than SMs.  Each chunk operand is read once per head instead of once per slice, and
// every warp tile is large enough that an operand fragment, once loaded and split, feeds 4 to 16 MMAs.
// ---------------------------------------------------------------------------------------------------
using bwdc::copy_rows;
using bwdc::kWideThreads;

// fwd_scan_wide_kernel: blockIdx.x = batch x head.  Per chunk, as fwd_scan_kernel over all dv columns:
//   1. [W; Q'] S: warp w takes rows (w & 1) * 16 of W and of Q' (stacked in shared memory) and 16 value
//      columns; V' = U - W S to shared memory, Q' S kept in registers;
//   2. y = Q' S + att V' (read-out rows) to HBM; S = gam_L S + K^^T V', warp w a 32 x 32 block of S.
template <typename TO>
__global__ void __launch_bounds__(kWideThreads, 1) fwd_scan_wide_kernel(const bwdc::Params p) {
    using namespace bwdc;
    extern __shared__ __align__(16) float sm[];
    __shared__ int64_t s_rt[kBL];
    const CoreParams &f = p.f;
    const int dk = (int)f.dk, dv = (int)f.dv, dkp = p.dkp, dvp = p.dvp, tid = threadIdx.x;
    const int warp = tid >> 5;
    const int64_t bh = blockIdx.x, b = bh / f.heads, h = bh - b * f.heads, nc = p.nc;
    float *sX = sm;                                        // [kMaxD][kWS]  the state
    float *sW = sX + kMaxD * kWS, *sQp = sW + kBL * kLD;   // [kBL][kLD]    W, then Q' (one stacked A)
    float *sKh = sQp + kBL * kLD;                          // [kBL][kWS]
    float *sU = sKh + kBL * kWS, *sV = sU + kBL * kWS;     // [kBL][kWS]
    float *satt = sV + kBL * kWS;                          // [kBL][kAS]
    const int64_t sbase = bh * (int64_t)dk * dv;
    TO *Y = static_cast<TO *>(f.y);

    for (int idx = tid; idx < dkp * dvp; idx += kWideThreads) {
        const int d = idx / dvp, j = idx - d * dvp;
        sX[d * kWS + j] = (d < dk && j < dv) ? f.state_in[sbase + (int64_t)d * dv + j] : 0.f;
    }
    auto issue_wuq = [&](int64_t ch) {
        copy_rows<kWideThreads>(sW, kLD, p.W + ch * kBL * dkp, dkp, dkp);
        copy_rows<kWideThreads>(sQp, kLD, p.Qp + ch * kBL * dkp, dkp, dkp);
        copy_rows<kWideThreads>(sU, kWS, p.U + ch * kBL * dvp, dvp, dvp);
        ptx::cp_async_commit();
    };
    auto issue_ak = [&](int64_t ch) {
        copy_rows<kWideThreads>(satt, kAS, p.att + ch * kBL * kBL, kBL, kBL);
        copy_rows<kWideThreads>(sKh, kWS, p.Kh + ch * kBL * dkp, dkp, dkp);
        ptx::cp_async_commit();
    };
    issue_wuq(bh * nc);
    issue_ak(bh * nc);

    // interval-1/2 tile: rows r0 (of W and of Q'), columns c1 .. c1 + 15
    const int ncb = (dvp + 15) >> 4;
    const bool t1 = warp < 2 * ncb;
    const int r0 = (warp & 1) * 16, c1 = (warp >> 1) * 16;
    // state-update tile: key rows d0 .. d0 + 31, value columns c3 .. c3 + 31
    const int nsb = (dvp + 31) >> 5;
    const bool t3 = warp < ((dkp + 31) >> 5) * nsb;
    const int d0 = (warp / nsb) * 32, c3 = (warp % nsb) * 32;

    for (int64_t c = 0; c < nc; ++c) {
        const int64_t ch = bh * nc + c;
        const float gl = p.gl[ch];
        ptx::cp_async_wait<1>();  // W, Q', U of chunk c
        __syncthreads();
        if (tid < kBL) s_rt[tid] = chunk_rows(f, b, h, c, tid).rt;
        float ay[1][2][4] = {};
        if (t1) {
            float a1[2][2][4] = {};
            warp_mma3_block<2, kBL, 2, kLD, 1, kWS>(a1, r0, c1, dkp, sW, sX);
            block_store<1, 16, 2>(reinterpret_cast<const float(&)[1][2][4]>(a1[0]), r0, c1, kBL, dvp,
                                  [&](int i, int j, float a) { sV[i * kWS + j] = sU[i * kWS + j] - a; });
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int q = 0; q < 4; ++q) ay[0][n][q] = a1[1][n][q];
        }
        __syncthreads();
        if (c + 1 < nc) issue_wuq(ch + 1);
        else ptx::cp_async_commit();
        ptx::cp_async_wait<1>();  // att, K^ of chunk c
        __syncthreads();
        if (t1) {
            warp_mma3_block<1, 16, 2, kAS, 1, kWS>(ay, r0, c1, kBL, satt, sV);
            block_store<1, 16, 2>(ay, r0, c1, kBL, dv, [&](int i, int j, float a) {
                const int64_t rt = s_rt[i];
                if (rt >= 0) st(Y + rt * dv + j, a);
            });
        }
        if (t3) {
            float a3[2][4][4] = {};
            warp_mma3_block<2, 16, 4, 1, kWS, kWS>(a3, d0, c3, kBL, sKh, sV);
            block_store<2, 16, 4>(a3, d0, c3, dkp, dvp,
                                  [&](int d, int j, float a) { sX[d * kWS + j] = fmaf(gl, sX[d * kWS + j], a); });
        }
        __syncthreads();
        if (c + 1 < nc) issue_ak(ch + 1);
        else ptx::cp_async_commit();
    }
    ptx::cp_async_wait<0>();
    for (int idx = tid; idx < dk * dv; idx += kWideThreads) {
        const int d = idx / dv, j = idx - d * dv;
        f.state_out[sbase + (int64_t)d * dv + j] = sX[d * kWS + j];
    }
}

}  // namespace f32c
}  // namespace dc
