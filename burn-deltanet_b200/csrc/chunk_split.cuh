// chunk_split.cuh — the tensor-core chunkwise prefill for per-channel gates
// (GDN-2: erase b in R^dk, write w in R^dv, log-decay g in R^dk), as two
// kernels over a caller-provided workspace.
//
// With per-channel decay, e^{G_id - G_jd} sits inside the key-channel sums of
// Akk and Aqk, and one chunk's gates alone are 96 KB in fp32: the
// S-independent half of a chunk no longer fits beside the state chain in one
// SM's shared memory.  The work splits where the chunk algorithm splits
// (src/delta/chunk.rs:103-157 is S-independent, 167-205 is the scan):
//
//   prep_kernel   one CTA per (chunk, batch x head), every chunk in parallel:
//                 gate scan, decay-aware Akk / Aqk, T = (I + Akk)^-1 and the
//                 S-independent products, written to the workspace per chunk:
//                   A6  = [-W; s (q e^G) - Aqk W]   bf16 128 x 128
//                   U   = T (v w)                   fp32  64 x 128
//                   Y0  = Aqk U                     bf16  64 x 128
//                   Kh  = k e^{G_63 - G}            bf16  64 x 128
//                   gam = e^{G_63}                  fp32  128
//                 with W = T (b k e^G), the per-channel form of chunk.rs:144-157.
//   scan_kernel   one CTA per (batch x head), chunks in order, S in TMEM:
//                   [V'; y] = [U; Y0] + A6 S        (V' = U - W S; y = Q' S + Aqk U)
//                   S      <- diag(gam) S + Kh^T V'
//
// Decay-aware Akk / Aqk without overflow.  G (the chunk-local cumulative log
// decay) does not increase along the chunk, so for j <= r <= i
//   e^{G_i - G_j} = e^{G_i - G_r} e^{G_r - G_j},   both factors in [0, 1].
// The 64 rows are bisected six times (blocks of 64, 32, ..., 2).  At each level
// a block's second-half rows i meet its first-half rows j through the
// reference r = the block's midpoint, and each pair i > j meets at exactly one
// level.  One level is one product of two packed 32-row operands
//   R[i] = (b k)_i e^{G_i - G_r}   (for Aqk: q_i e^{G_i - G_r}),
//   C[j] = k_j e^{G_r - G_j},
// whose block diagonal holds that level's pairs (warp MMAs, bf16).  The
// factors are running products of alpha = e^g inside each half-block: no
// exponent is taken of a difference that could overflow, and underflow goes
// to the exact limit 0.  The diagonal of Aqk (no decay) is a plain reduction.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "chunk_tc.cuh"
#include "common.cuh"
#include "ptx.cuh"

// Phase-timing hook of the prep kernel (defined by a timing build; a no-op here).
#ifndef DC_SPLIT_MARK
#define DC_SPLIT_MARK(id)
#endif

namespace dc {
namespace split {

using tc::kAP;
constexpr int kOP = 136;  // bf16 row pitch of the level operands (272 B: ldmatrix rows hit distinct banks)

// The workspace, structure of arrays, chunk-major inside each (batch, head).
struct SplitWs {
    __nv_bfloat16 *a6;  // [BH * nch * 128][128]
    float *u;           // [BH * nch * 64][128]
    __nv_bfloat16 *y0;  // [BH * nch * 64][128]
    __nv_bfloat16 *kh;  // [BH * nch * 64][128]
    float *gam;         // [BH * nch][128]
    int64_t nch;
};

constexpr uint64_t kWsBytesPerChunk = 32768ull + 32768ull + 16384ull + 16384ull + 512ull;

// ---------------------------------------------------------------- prep kernel
// Two CTAs per SM (the kernel is latency-bound per chunk; a second CTA hides it), so shared memory is
// shared between phases (P1 scan, P2 q.k diagonal, P3 bisection, P4 solve, P5 T hi/lo, P6 P = Aqk T,
// P7 P hi/lo, P8 [T; P] [v w | b k e^G], P9 workspace stores).  Two S-independent intermediates park in
// the chunk's own workspace slots until their shared memory frees up, and come back by TMA:
// [v w | b k e^G] in the A6 slot (rows 0-63 | 64-127) and s q e^G in the Y0 slot.
constexpr int kThreadsA = 256;
constexpr uint32_t A_QKT = 0;            // q, k tiles (TMA, SW128) [P1-P3]; then [T; P] hi | lo [P5-P8]
constexpr uint32_t A_TPH = 0, A_TPL = 16384;
constexpr uint32_t A_AF = 32768;         // scan staging ring [P1]; Akk fp32 [64][kAP] [P3-P4];
constexpr uint32_t A_TF = A_AF + 64 * kAP * 4;  //   T fp32 [64][kAP] [P4-P5];
constexpr uint32_t A_BOP = A_AF;         //   [v w | b k e^G], four MN-major SW128 blocks (TMA) [P6-P8]
constexpr uint32_t A_R = 67584;          // level operands Rkk, Rqk, C, bf16 [32][kOP] each [P3];
constexpr uint32_t A_RKK = A_R, A_RQK = A_R + 32 * kOP * 2, A_CC = A_R + 64 * kOP * 2;
constexpr uint32_t A_QT = A_R;           //   s q e^G, two SW128 64-column boxes (TMA) [P4-P9]
constexpr uint32_t A_STG = A_AF;         // erase / write / v rows staged by cp.async [P1]: three buffers of
constexpr uint32_t kStgBytes = 16 * 512 + 16 * 512 + 16 * 256;  // [16 rows] of e, w (up to fp32), v bf16
constexpr uint32_t A_AQK = 94208;        // Aqk bf16 64x64, K-major SW128 [P2-P6]
constexpr uint32_t A_X = A_AQK + 8192;   // exchange: fp32 [3][4][128] (per quarter: sum of g, first alpha,
                                         //   product of the other fifteen alphas), then [4][2][48] partial
                                         //   sums of the two finest levels
constexpr uint32_t A_BAR = A_X + 1920 * 4;  // five mbarriers, TMEM pointer, flag
constexpr uint32_t A_USED = A_BAR + 48;
constexpr uint32_t kSmemA = A_USED + 1024;
enum BarA { BA_P = 0, BA_BIG, BA_QK, BA_QT, BA_BOP };
static_assert(A_TF + 64 * kAP * 4 <= A_R, "Akk / T overlap the operands");
static_assert(A_BOP + 32768 <= A_R && A_BOP % 1024 == 0, "B operands misplaced");
static_assert(A_R + 96 * kOP * 2 <= A_AQK && A_QT + 16384 <= A_AQK && A_QT % 1024 == 0, "level operands misplaced");
static_assert(A_AQK % 1024 == 0, "SW128 tiles must be 1024-byte aligned");
static_assert(A_STG + 3 * kStgBytes <= A_AQK, "scan staging overflows into Aqk");
static_assert(kSmemA <= 115712, "prep kernel must fit two CTAs per SM");
constexpr uint32_t TMA_BIG = 0, TMA_P = 0;  // TMEM: P = Aqk T (N=64) first, then [U W; Y0 AqkW] (N=256)

__device__ __forceinline__ void st_bf16(uint8_t *p, float x) {
    *reinterpret_cast<__nv_bfloat16 *>(p) = __float2bfloat16_rn(x);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            ptx::smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(ptx::smem_u32(bar))
        : "memory");
}

// Generic-proxy global writes of this thread become visible to later TMA (async-proxy) reads.
__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Element (t, d) of the q (which = 0) or k (which = 1) tile.
__device__ __forceinline__ float qk_tile(const uint8_t *base, int which, int t, int d) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(
        base + A_QKT + 16384 * which + (uint32_t)(d >> 6) * 8192u + ptx::sw128(t, d & 63)));
}

// One bisection level (blocks of s = 2^LS rows), part 1: this thread's operand rows.  Thread (cp, q4) owns
// channels 2 cp, 2 cp + 1 of rows 16 q4 .. 16 q4 + 15 (one quarter).  Blocks of 16 rows or fewer lie inside a
// quarter; at the two coarser levels a quarter lies wholly on one side of its block, and the quarters'
// published first alphas (af) and products of the other fifteen (ar) give the starting products.  Each level
// is its own unrolled body (LS at compile time): which rows are on which side, where their packed index
// lands and where a running product starts are all constants, leaving a few multiplies, a pack and a store
// per row.
template <int LS>
__device__ __forceinline__ void level_build(uint8_t *base, const uint32_t (&bk2)[16], const float (&alpha)[32],
                                            const float *af, const float *ar, int cp, int q4) {
    constexpr int s = 1 << LS, half = s >> 1, lh = LS - 1;
    uint8_t *Rkk = base + A_RKK, *Rqk = base + A_RQK, *Cc = base + A_CC;
    const int ch = 2 * cp;
    auto tile2 = [&](int which, int i) -> uint32_t {  // q (0) or k (1) of row 16 q4 + i, channels ch, ch + 1
        return *reinterpret_cast<const uint32_t *>(base + A_QKT + 16384 * which + (uint32_t)(ch >> 6) * 8192u +
                                                   ptx::sw128(16 * q4 + i, ch & 63));
    };
    auto put = [&](uint8_t *buf, int row, float x0, float x1) {
        *reinterpret_cast<uint32_t *>(buf + 2 * (row * kOP + ch)) = ptx::pack_bf16(x0, x1);
    };
    auto row_side = [&](int i, int m, float (&P)[2], bool start, const float (&P0)[2]) {
#pragma unroll
        for (int c = 0; c < 2; ++c) P[c] = start ? P0[c] : P[c] * alpha[2 * i + c];
        const uint32_t b2 = bk2[i], q2 = tile2(0, i);
        put(Rkk, m, ptx::bf16lo(b2) * P[0], ptx::bf16hi(b2) * P[1]);
        put(Rqk, m, ptx::bf16lo(q2) * P[0], ptx::bf16hi(q2) * P[1]);
    };
    auto col_side = [&](int i, int n, float (&Pb)[2], bool start, const float (&Pb0)[2]) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float an = alpha[2 * (i + 1 < 16 ? i + 1 : 15) + c];  // alpha of the next row (in quarter)
            Pb[c] = start ? Pb0[c] : Pb[c] * an;
        }
        const uint32_t k2 = tile2(1, i);
        put(Cc, n, ptx::bf16lo(k2) * Pb[0], ptx::bf16hi(k2) * Pb[1]);
    };
    float P[2] = {1.f, 1.f}, Pb[2] = {1.f, 1.f};
    if constexpr (LS >= 5) {
        // The quarter is wholly a row side or a column side of its 2^LS block.
        const bool all_row = (LS == 6) ? (q4 >= 2) : ((q4 & 1) != 0);
        const int mbase = (LS == 6) ? 16 * (q4 & 1) : 16 * (q4 >> 1);
        if (all_row) {
            float P0[2] = {1.f, 1.f};
            if (LS == 6 && q4 == 3) {
#pragma unroll
                for (int c = 0; c < 2; ++c) P0[c] = ar[2 * 128 + ch + c] * alpha[c];  // product of alphas 33 .. 48
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) row_side(i, mbase + i, P, i == 0, P0);
        } else {
            float Pb0[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (LS == 6)
                    Pb0[c] = (q4 == 1) ? af[2 * 128 + ch + c]                                  // alpha 32
                                       : af[128 + ch + c] * ar[128 + ch + c] * af[2 * 128 + ch + c];  // alphas 16 .. 32
                else
                    Pb0[c] = af[(q4 + 1 < 4 ? q4 + 1 : 3) * 128 + ch + c];  // alpha of the next quarter's first row
            }
#pragma unroll
            for (int i = 15; i >= 0; --i) col_side(i, mbase + i, Pb, i == 15, Pb0);
        }
    } else {
        const int mbase = 8 * q4;
        const float one[2] = {1.f, 1.f};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int pos = i & (s - 1);
            if (pos >= half) row_side(i, mbase + ((i >> LS) << lh) + (pos - half), P, pos == half, one);
        }
#pragma unroll
        for (int i = 15; i >= 0; --i) {
            const int pos = i & (s - 1);
            if (pos < half) {
                float an[2];
#pragma unroll
                for (int c = 0; c < 2; ++c) an[c] = alpha[2 * (i + 1 < 16 ? i + 1 : 15) + c];
                col_side(i, mbase + ((i >> LS) << lh) + pos, Pb, pos == half - 1, an);
            }
        }
    }
}

// Part 2: the warps' MMAs of the packed 32 x 32 product, whose block-diagonal entries are scattered into Akk
// (fp32) and Aqk (bf16).  One copy serves every level (LS at run time).
__device__ __forceinline__ void level_mma(int LS, uint8_t *base, uint32_t sb, float *Af, float scale, int warp,
                                          int lane) {
    const int s = 1 << LS, half = s >> 1, lh = LS - 1;
    (void)s;
    // Tiles of the packed 32 x 32 product that meet its block diagonal: all eight at the top level,
    // (mt, 2 mt) and (mt, 2 mt + 1) below.  Job = (matrix, m tile, n tile); Akk and Aqk share C.
    const int njobs = (half == 32) ? 16 : 8;
#pragma unroll 1
    for (int job0 = 0; job0 < njobs; job0 += kThreadsA / 32) {
        const int job = job0 + warp;
        const int mat = job & 1;
        const int mt = (half == 32) ? ((job >> 1) & 1) : ((job >> 2) & 1);
        const int nt = (half == 32) ? (job >> 2) : (2 * mt + ((job >> 1) & 1));
        const uint32_t rb = sb + (mat ? A_RQK : A_RKK);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t a[4], bb[2];
            ptx::ldsm_x4(rb + 2u * ((16 * mt + (lane & 15)) * kOP + 16 * ks + 8 * (lane >> 4)), a);
            ptx::ldsm_x2(sb + A_CC + 2u * ((8 * nt + (lane & 7)) * kOP + 16 * ks + 8 * ((lane >> 3) & 1)), bb);
            ptx::mma_bf16_16x8x16(acc, a, bb);
        }
        const int gq = lane >> 2, t4 = lane & 3;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int m = 16 * mt + gq + 8 * (e >> 1), n = 8 * nt + 2 * t4 + (e & 1);
            const int blk = m >> lh;
            if (blk != (n >> lh)) continue;
            const int i = (blk << LS) + half + (m & (half - 1)), j = (blk << LS) + (n & (half - 1));
            if (mat == 0)
                Af[i * kAP + j] = acc[e];
            else
                st_bf16(base + A_AQK + ptx::sw128(i, j), scale * acc[e]);
        }
    }
}

// After the call, v[0] of lane l holds the sum over the warp's lanes of v[l] (32 values, 31 shuffles).
__device__ __forceinline__ void reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
            const float send = upper ? v[i] : v[i + w];
            const float keep = upper ? v[i + w] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
    }
}

// The two finest bisection levels (blocks of 2 and 4 rows) without the MMA machinery: each thread forms its
// quarter's 8 + 16 pairs per matrix for its two channels (at most three alpha factors each), the warp sums
// them over its 64 channels in registers, and the quarter's two warps add up through shared memory.
// Element e of the 48: Akk (e < 24) or Aqk, pair u = e mod 24: u < 8 the 2-block pair (2u+1, 2u), else the
// 4-block b = (u - 8) / 4 pair (4b + 2 + p/2, 4b + p mod 2), p = (u - 8) mod 4.
__device__ __forceinline__ void finest_levels(uint8_t *base, float *Af, float *Xr, const uint32_t (&bk2)[16],
                                              const float (&alpha)[32], float scale, int cp, int q4, int tid,
                                              int lane) {
    const int ch = 2 * cp;
    auto tile2 = [&](int which, int i) -> uint32_t {
        return *reinterpret_cast<const uint32_t *>(base + A_QKT + 16384 * which + (uint32_t)(ch >> 6) * 8192u +
                                                   ptx::sw128(16 * q4 + i, ch & 63));
    };
    float v[48];
#pragma unroll
    for (int e = 0; e < 48; ++e) v[e] = 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        auto a = [&](int i) { return alpha[2 * i + c]; };
        auto half_of = [&](uint32_t w) { return c ? ptx::bf16hi(w) : ptx::bf16lo(w); };
#pragma unroll
        for (int m = 0; m < 8; ++m) {  // 2-blocks: (2m + 1, 2m)
            const float kj = half_of(tile2(1, 2 * m)) * a(2 * m + 1);
            v[m] += half_of(bk2[2 * m + 1]) * kj;
            v[24 + m] += half_of(tile2(0, 2 * m + 1)) * kj;
        }
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {  // 4-blocks: rows 4bb + {2, 3} with 4bb + {0, 1}
            const int r0 = 4 * bb;
            const float a1 = a(r0 + 1), a2 = a(r0 + 2), a3 = a(r0 + 3);
            const float k0 = half_of(tile2(1, r0)), k1 = half_of(tile2(1, r0 + 1));
            const float dec[4] = {a1 * a2, a2, a1 * a2 * a3, a2 * a3};  // (2,0), (2,1), (3,0), (3,1)
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) {
                const int i = r0 + 2 + (pp >> 1);
                const float kd = ((pp & 1) ? k1 : k0) * dec[pp];
                v[8 + 4 * bb + pp] += half_of(bk2[i]) * kd;
                v[24 + 8 + 4 * bb + pp] += half_of(tile2(0, i)) * kd;
            }
        }
    }
    // Sum over the warp's lanes: elements 0-31 by a full reduce-scatter, 32-47 by a half one.
    float lo[32], hi[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) lo[e] = v[e];
#pragma unroll
    for (int e = 0; e < 32; ++e) hi[e] = (e < 16) ? v[32 + e] : 0.f;
    reduce_scatter32(lo, lane);
    reduce_scatter32(hi, lane);
    const int wh = cp >> 5;  // which of the quarter's two warps
    Xr[(q4 * 2 + wh) * 48 + lane] = lo[0];
    if (lane < 16) Xr[(q4 * 2 + wh) * 48 + 32 + lane] = hi[0];
    ptx::named_sync(tc::NB_PAR, kThreadsA);
    if (cp < 48) {
        const int e = cp, u = e % 24;
        const float sum = Xr[(q4 * 2) * 48 + e] + Xr[(q4 * 2 + 1) * 48 + e];
        int i, j;
        if (u < 8) {
            i = 2 * u + 1;
            j = 2 * u;
        } else {
            const int bb = (u - 8) >> 2, pp = (u - 8) & 3;
            i = 4 * bb + 2 + (pp >> 1);
            j = 4 * bb + (pp & 1);
        }
        i += 16 * q4;
        j += 16 * q4;
        if (e < 24)
            Af[i * kAP + j] = sum;
        else
            st_bf16(base + A_AQK + ptx::sw128(i, j), scale * sum);
    }
    (void)tid;
}

template <typename TG>
__global__ void __launch_bounds__(kThreadsA, 2)
    prep_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_bop, const __grid_constant__ CUtensorMap tm_qt,
                const CoreParams p, const SplitWs ws, int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    const uint32_t sb = ptx::smem_u32(base);
    float *Af = reinterpret_cast<float *>(base + A_AF);
    float *Tf = reinterpret_cast<float *>(base + A_TF);
    float *X = reinterpret_cast<float *>(base + A_X);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + A_BAR);
    uint32_t *tmem_ptr = reinterpret_cast<uint32_t *>(base + A_BAR + 40);
    volatile int *flag = reinterpret_cast<volatile int *>(base + A_BAR + 44);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t c = blockIdx.x, bh = blockIdx.y, nch = ws.nch;
    const int64_t b = bh / p.heads, h = bh % p.heads;
    const int64_t row0 = c * tc::kL;
    const int nvalid = (int)((p.seq - row0) < 64 ? (p.seq - row0) : 64);
    const int64_t bhc = bh * nch + c;
    const float scale = p.scale;

    if (tid == 0) {
        *flag = 0;
        for (int i = 0; i < 5; ++i) ptx::mbar_init(&bars[i], 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_bop);
        ptx::prefetch_tmap(&tm_qt);
        // The chunk's q and k rows (rows past the sequence read as zeros).
        ptx::mbar_arrive_expect_tx(&bars[BA_QK], 2 * 16384);
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            ptx::tma_load_4d(base + A_QKT + 8192 * x, &tm_q, &bars[BA_QK], 64 * x, (int)h, (int)row0, (int)b);
            ptx::tma_load_4d(base + A_QKT + 16384 + 8192 * x, &tm_k, &bars[BA_QK], 64 * x, (int)h, (int)row0, (int)b);
        }
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_ptr, 256);
        ptx::tmem_relinquish();
    }
    for (int i = tid; i < 512; i += kThreadsA) ptx::st_shared_v4(sb + A_AQK + 16 * i, 0u, 0u, 0u, 0u);

    // Two adjacent key / value channels per thread, a quarter of the chunk's rows each.
    const int cp = tid & 63, q4 = tid >> 6, ch = 2 * cp;
    const __nv_bfloat16 *vg = static_cast<const __nv_bfloat16 *>(p.v);
    auto rowidx = [&](int t) -> int64_t { return (b * p.seq + row0 + t) * p.heads + h; };
    auto gate2 = [&](const void *ptr, int w, int64_t r, float &x0, float &x1) {  // inputs are read-only here
        const TG *g = static_cast<const TG *>(ptr) + r * w + (w == 1 ? 0 : ch);
        if (w == 1) {
            x0 = x1 = (sizeof(TG) == 4) ? __ldg(reinterpret_cast<const float *>(g))
                                        : __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16 *>(g)));
        } else if constexpr (sizeof(TG) == 4) {
            const float2 v2 = __ldg(reinterpret_cast<const float2 *>(g));
            x0 = v2.x;
            x1 = v2.y;
        } else {
            const __nv_bfloat162 v2 = __ldg(reinterpret_cast<const __nv_bfloat162 *>(g));
            x0 = __low2float(v2);
            x1 = __high2float(v2);
        }
    };
    float *Xg = X, *Xaf = X + 512, *Xar = X + 1024;  // [quarter][channel]

    constexpr int kRowB = 128 * (int)sizeof(TG);  // bytes of one full-width gate row
    const bool e_full = p.ew != 1, w_full = p.ww != 1;
    const int64_t r_first = rowidx(16 * q4), r_step = p.heads;  // rows of this quarter: r_first + i * r_step
    uint32_t *park_v = reinterpret_cast<uint32_t *>(ws.a6 + bhc * 128 * 128 + (16 * q4) * 128 + ch);  // v w
    uint32_t *park_k = park_v + 64 * 64;                                                          // b k e^G
    uint32_t *park_q = reinterpret_cast<uint32_t *>(ws.y0 + bhc * 64 * 128 + (16 * q4) * 128 + ch);  // s q e^G
    uint32_t *kh_out = reinterpret_cast<uint32_t *>(ws.kh + (bhc * 64 + 16 * q4) * 128 + ch);
    auto stage = [&](int k) {  // batch k: rows 4k..4k+3 of each quarter -> slots 4 q + 0..3
        const uint32_t buf = sb + A_STG + (uint32_t)(k % 3) * kStgBytes;
        for (int q = tid; q < 16 * (kRowB / 16); q += kThreadsA) {
            const int slot = q / (kRowB / 16), piece = q % (kRowB / 16);
            const int t = 16 * (slot >> 2) + 4 * k + (slot & 3);
            const int64_t r = t < nvalid ? rowidx(t) : 0;
            const uint32_t n = t < nvalid ? 16u : 0u;
            if (e_full)
                ptx::cp_async16(buf + slot * kRowB + piece * 16,
                                static_cast<const uint8_t *>(p.erase) + r * kRowB + piece * 16, n);
            if (w_full)
                ptx::cp_async16(buf + 8192 + slot * kRowB + piece * 16,
                                static_cast<const uint8_t *>(p.write) + r * kRowB + piece * 16, n);
        }
        {
            const int slot = tid >> 4, piece = tid & 15;
            const int t = 16 * (slot >> 2) + 4 * k + (slot & 3);
            const int64_t r = t < nvalid ? rowidx(t) : 0;
            ptx::cp_async16(buf + 16384 + slot * 256 + piece * 16, vg + r * 128 + piece * 8, t < nvalid ? 16u : 0u);
        }
        ptx::cp_async_commit();
    };
    // The scan's first two batches of erase / write / v are in flight while g loads.
    stage(0);
    stage(1);
    DC_SPLIT_MARK(0);
    // ---- (0) this quarter's g (all loads in flight at once) and its sum: the chunk-local offsets of G ----
    float alpha[32];  // [row][channel]; g until the scan turns it into e^g
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int t = 16 * q4 + i;
        alpha[2 * i] = alpha[2 * i + 1] = 0.f;
        if (p.gw > 0 && t < nvalid) gate2(p.g, p.gw, rowidx(t), alpha[2 * i], alpha[2 * i + 1]);
    }
    {
        float gs0 = 0.f, gs1 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            gs0 += alpha[2 * i];
            gs1 += alpha[2 * i + 1];
        }
        Xg[q4 * 128 + ch] = gs0;
        Xg[q4 * 128 + ch + 1] = gs1;
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_ptr;
    float G[2], G63[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        float before = 0.f, all = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float x = Xg[q * 128 + ch + c];
            if (q < q4) before += x;
            all += x;
        }
        G[c] = before;
        G63[c] = all;
    }
    DC_SPLIT_MARK(1);

    // ---- (1) the scan: G, alpha = e^g, and per row v w, b k e^G, s q e^G (parked in the workspace),
    //      Kh (to the workspace) and b k (for the bisection).  erase, write (when per channel) and v
    //      stream through a three-buffer shared-memory ring by cp.async, 4 rows of each quarter per batch,
    //      two batches ahead; q and k come from the TMA tiles.  The batch loop is not unrolled (the
    //      kernel's code must fit the instruction cache), so alpha and bk2 are rotating windows whose
    //      first slots always hold the current batch. ----
    const bool tiles_ok = ptx::mbar_wait(&bars[BA_QK], 0);
    uint32_t bk2[16];  // per row, (b k) of the two channels as a bf16 pair; rotates with alpha
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
        if (k + 2 < 4)
            stage(k + 2);
        else
            ptx::cp_async_commit();  // an empty group keeps the count uniform
        ptx::cp_async_wait<2>();
        ptx::named_sync(tc::NB_PAR, kThreadsA);  // every thread's copies of batch k have landed
        const uint8_t *buf = base + A_STG + (k % 3) * kStgBytes;
        const TG *se = reinterpret_cast<const TG *>(buf) + (4 * q4) * 128 + ch;
        const TG *sw = reinterpret_cast<const TG *>(buf + 8192) + (4 * q4) * 128 + ch;
        const uint32_t *sv = reinterpret_cast<const uint32_t *>(buf + 16384 + (4 * q4) * 256 + 2 * ch);
        uint32_t bkw[4];
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const int i = 4 * k + o, t = 16 * q4 + i;
            const bool ok_row = t < nvalid;
            float ex[2], wx[2];
            if (e_full) {
                ex[0] = ld(se + o * 128);
                ex[1] = ld(se + o * 128 + 1);
            } else {
                ex[0] = ex[1] = 0.f;
                if (ok_row) gate2(p.erase, 1, r_first + i * r_step, ex[0], ex[1]);
            }
            if (w_full) {
                wx[0] = ld(sw + o * 128);
                wx[1] = ld(sw + o * 128 + 1);
            } else {
                wx[0] = wx[1] = 0.f;
                if (ok_row) gate2(p.write, 1, r_first + i * r_step, wx[0], wx[1]);
            }
            const uint32_t v2 = sv[o * 64];
            const uint32_t q2 = *reinterpret_cast<const uint32_t *>(base + A_QKT + (uint32_t)(ch >> 6) * 8192u +
                                                                    ptx::sw128(t, ch & 63));
            const uint32_t k2 = *reinterpret_cast<const uint32_t *>(base + A_QKT + 16384 + (uint32_t)(ch >> 6) * 8192u +
                                                                    ptx::sw128(t, ch & 63));
            const float vx[2] = {ptx::bf16lo(v2), ptx::bf16hi(v2)}, qx[2] = {ptx::bf16lo(q2), ptx::bf16hi(q2)};
            const float kx[2] = {ptx::bf16lo(k2), ptx::bf16hi(k2)};
            float vw[2], kg[2], qg[2], kh[2], bk[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                G[c] += alpha[2 * o + c];
                alpha[2 * o + c] = __expf(alpha[2 * o + c]);
                const float gam = __expf(G[c]);
                vw[c] = vx[c] * wx[c];
                kg[c] = ex[c] * kx[c] * gam;
                qg[c] = scale * qx[c] * gam;
                kh[c] = kx[c] * __expf(G63[c] - G[c]);
                bk[c] = ex[c] * kx[c];
            }
            park_v[i * 64] = ptx::pack_bf16(vw[0], vw[1]);
            park_k[i * 64] = ptx::pack_bf16(kg[0], kg[1]);
            park_q[i * 64] = ptx::pack_bf16(qg[0], qg[1]);
            kh_out[i * 64] = ptx::pack_bf16(kh[0], kh[1]);
            bkw[o] = ptx::pack_bf16(bk[0], bk[1]);
        }
        // rotate: the processed batch moves to the back of both windows
        float a8[8];
#pragma unroll
        for (int o = 0; o < 8; ++o) a8[o] = alpha[o];
#pragma unroll
        for (int j = 0; j < 24; ++j) alpha[j] = alpha[j + 8];
#pragma unroll
        for (int o = 0; o < 8; ++o) alpha[24 + o] = a8[o];
#pragma unroll
        for (int j = 0; j < 12; ++j) bk2[j] = bk2[j + 4];
#pragma unroll
        for (int o = 0; o < 4; ++o) bk2[12 + o] = bkw[o];
        ptx::named_sync(tc::NB_PAR, kThreadsA);  // batch k's buffer is free for batch k + 3
    }
    if (q4 == 0) {
        ws.gam[bhc * 128 + ch] = __expf(G63[0]);
        ws.gam[bhc * 128 + ch + 1] = __expf(G63[1]);
    }
    // Publish this quarter's first alpha and the product of its other fifteen (the coarse levels' starts).
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        float rest = 1.f;
#pragma unroll
        for (int i = 1; i < 16; ++i) rest *= alpha[2 * i + c];
        Xaf[q4 * 128 + ch + c] = alpha[c];
        Xar[q4 * 128 + ch + c] = rest;
    }
    fence_async_global();  // the parked rows are read back by TMA
    if (!tiles_ok) *flag = 1;
    // Aqk's diagonal: row t's q.k from the tiles, 32 channels per thread, four threads per row.
    {
        const int t = tid >> 2, part = tid & 3;
        float acc = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
            const int col = 32 * (part & 1) + 8 * c8;  // channels 64 (part >> 1) + col .. + 7
            const uint32_t off = (uint32_t)(part >> 1) * 8192u + ptx::sw128(t, col);
            const uint4 qv = ptx::ld_shared_v4(sb + A_QKT + off), kv = ptx::ld_shared_v4(sb + A_QKT + 16384 + off);
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w}, kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                acc += ptx::bf16lo(qw[e]) * ptx::bf16lo(kw[e]) + ptx::bf16hi(qw[e]) * ptx::bf16hi(kw[e]);
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (part == 0) st_bf16(base + A_AQK + ptx::sw128(t, t), scale * acc);
    }
    ptx::named_sync(tc::NB_PAR, kThreadsA);
    DC_SPLIT_MARK(2);

    // ---- (2) Akk (strictly lower) and Aqk (lower) by bisection levels, coarsest first ----
#pragma unroll 1
    for (int LS = 6; LS >= 3; --LS) {
        switch (LS) {
            case 6: level_build<6>(base, bk2, alpha, Xaf, Xar, cp, q4); break;
            case 5: level_build<5>(base, bk2, alpha, Xaf, Xar, cp, q4); break;
            case 4: level_build<4>(base, bk2, alpha, Xaf, Xar, cp, q4); break;
            default: level_build<3>(base, bk2, alpha, Xaf, Xar, cp, q4); break;
        }
        ptx::named_sync(tc::NB_PAR, kThreadsA);
        level_mma(LS, base, sb, Af, scale, warp, lane);
        ptx::named_sync(tc::NB_PAR, kThreadsA);
    }
    finest_levels(base, Af, X + 1536, bk2, alpha, scale, cp, q4, tid, lane);
    ptx::named_sync(tc::NB_PAR, kThreadsA);
    // The level operands are dead: bring s q e^G back into their place.
    if (tid == 0) {
        ptx::mbar_arrive_expect_tx(&bars[BA_QT], 16384);
        tma_load_2d(base + A_QT, &tm_qt, &bars[BA_QT], 0, (int)(bhc * 64));
        tma_load_2d(base + A_QT + 8192, &tm_qt, &bars[BA_QT], 64, (int)(bhc * 64));
    }
    DC_SPLIT_MARK(3);
    // ---- (3) T = (I + Akk)^-1 ----
    tc::solve_unit_lower(Af, Tf, warp, lane, [] {}, [] {});
    DC_SPLIT_MARK(4);

    // ---- (4) T hi + lo: rows 0-63 of the A operand (blocks above the diagonal zero), over the q / k tiles ----
    {
        const int i = tid & 63, j0 = (tid >> 6) * 16;
        float t[16];
#pragma unroll
        for (int m = 0; m < 16; m += 4) {
            const float4 tv = *reinterpret_cast<const float4 *>(Tf + i * kAP + j0 + m);
            t[m] = j0 + m <= i ? tv.x : 0.f;
            t[m + 1] = j0 + m + 1 <= i ? tv.y : 0.f;
            t[m + 2] = j0 + m + 2 <= i ? tv.z : 0.f;
            t[m + 3] = j0 + m + 3 <= i ? tv.w : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float x0 = t[8 * q + 2 * e], x1 = t[8 * q + 2 * e + 1];
                hi[e] = ptx::pack_bf16(x0, x1);
                lo[e] = ptx::pack_bf16(x0 - ptx::bf16lo(hi[e]), x1 - ptx::bf16hi(hi[e]));
            }
            const uint32_t off = ptx::sw128(i, j0 + 8 * q);
            ptx::st_shared_v4(sb + A_TPH + off, hi[0], hi[1], hi[2], hi[3]);
            ptx::st_shared_v4(sb + A_TPL + off, lo[0], lo[1], lo[2], lo[3]);
        }
    }
    ptx::fence_async_smem();
    ptx::tc_fence_before();
    ptx::named_sync(tc::NB_PAR, kThreadsA);

    auto role_wait = [&](int bar, uint32_t parity) {
        const bool bad = !ptx::mbar_wait(&bars[bar], parity) || *flag != 0;
        if (ptx::named_sync_or(tc::NB_PAR, kThreadsA, bad)) {
            *flag = 1;
            return false;
        }
        return true;
    };

    // ---- (5) P = Aqk T (hi); Akk and T are dead: bring [v w | b k e^G] back over them ----
    if (tid == 0) {
        ptx::tc_fence_after();
        const uint32_t id = ptx::idesc_bf16(64, 64, 0, 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            ptx::umma_bf16(tmem + TMA_P, ptx::sdesc(sb + A_AQK + kk * 32, 16, 1024),
                           ptx::sdesc(sb + A_TPH + kk * 2048, 16384, 1024), id, kk > 0);
        ptx::umma_commit(&bars[BA_P]);
        ptx::mbar_arrive_expect_tx(&bars[BA_BOP], 32768);
        const int prow = (int)(bhc * 128);
#pragma unroll
        for (int x = 0; x < 4; ++x)
            tma_load_2d(base + A_BOP + 8192 * x, &tm_bop, &bars[BA_BOP], 64 * (x & 1), prow + 64 * (x >> 1));
    }
    bool ok = role_wait(BA_P, 0);
    DC_SPLIT_MARK(5);

    // ---- (6) P hi + lo: rows 64-127 of the A operand (M=64 accumulator: rows in lanes 0-15) ----
    if (ok) {
        ptx::tc_fence_after();
        const int sp = warp & 3, ch = warp >> 2;
        uint32_t v[32];
        ptx::tmem_ld32(tmem + ((uint32_t)(32 * sp) << 16) + TMA_P + 32 * ch, v);
        ptx::tmem_wait_ld();
        if (lane < 16) {
            const int i = 16 * sp + lane;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float *f = reinterpret_cast<const float *>(v + 8 * q);
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hi[e] = ptx::pack_bf16(f[2 * e], f[2 * e + 1]);
                    lo[e] = ptx::pack_bf16(f[2 * e] - ptx::bf16lo(hi[e]), f[2 * e + 1] - ptx::bf16hi(hi[e]));
                }
                const uint32_t off = ptx::sw128(64 + i, 32 * ch + 8 * q);
                ptx::st_shared_v4(sb + A_TPH + off, hi[0], hi[1], hi[2], hi[3]);
                ptx::st_shared_v4(sb + A_TPL + off, lo[0], lo[1], lo[2], lo[3]);
            }
        }
        ptx::fence_async_smem();
        ptx::tc_fence_before();
        ok = role_wait(BA_BOP, 0);  // also: every thread's P reads are done before the big MMA overwrites them
    }

    // ---- (7) [U W; Y0 Aqk W] = [T; P] (hi + lo) [v w | b k e^G] ----
    if (ok) {
        if (tid == 0) {
            ptx::tc_fence_after();
            const uint32_t id = ptx::idesc_bf16(128, 256, 0, 1);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                ptx::umma_bf16(tmem + TMA_BIG, ptx::sdesc(sb + (kk < 4 ? A_TPH : A_TPL) + (kk & 3) * 32, 16, 1024),
                               ptx::sdesc(sb + A_BOP + (kk & 3) * 2048, 8192, 1024), id, kk > 0);
            ptx::umma_commit(&bars[BA_BIG]);
        }
        DC_SPLIT_MARK(6);
        ok = role_wait(BA_BIG, 0) && role_wait(BA_QT, 0);
    }
    DC_SPLIT_MARK(7);

    // ---- (8) the workspace: U, Y0 (warps 0-3), A6 = [-W; Q'] (warps 4-7) ----
    if (ok) {
        ptx::tc_fence_after();
        const int sp = warp & 3, ch = warp >> 2, r = 32 * sp + lane;
        auto store32 = [&](const float *f, int col0) {  // this row's 32 columns from col0
            if (ch == 0 && r < 64) {
                float4 *dst = reinterpret_cast<float4 *>(ws.u + (bhc * 64 + r) * 128 + col0);
#pragma unroll
                for (int e = 0; e < 8; ++e) dst[e] = make_float4(f[4 * e], f[4 * e + 1], f[4 * e + 2], f[4 * e + 3]);
            } else if (ch == 0) {
                uint4 *dst = reinterpret_cast<uint4 *>(ws.y0 + (bhc * 64 + r - 64) * 128 + col0);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    dst[e] = make_uint4(ptx::pack_bf16(f[8 * e], f[8 * e + 1]), ptx::pack_bf16(f[8 * e + 2], f[8 * e + 3]),
                                        ptx::pack_bf16(f[8 * e + 4], f[8 * e + 5]),
                                        ptx::pack_bf16(f[8 * e + 6], f[8 * e + 7]));
            } else {
                uint4 *dst = reinterpret_cast<uint4 *>(ws.a6 + (bhc * 128 + r) * 128 + col0);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float x[8];
                    if (r < 64) {
#pragma unroll
                        for (int o = 0; o < 8; ++o) x[o] = -f[8 * e + o];
                    } else {
                        const int cc = col0 + 8 * e;  // s q e^G, SW128 box (cc >> 6), row r - 64
                        const uint4 qv = ptx::ld_shared_v4(sb + A_QT + (uint32_t)(cc >> 6) * 8192u +
                                                           ptx::sw128(r - 64, cc & 63));
                        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                        for (int o = 0; o < 4; ++o) {
                            x[2 * o] = ptx::bf16lo(qw[o]) - f[8 * e + 2 * o];
                            x[2 * o + 1] = ptx::bf16hi(qw[o]) - f[8 * e + 2 * o + 1];
                        }
                    }
                    dst[e] = make_uint4(ptx::pack_bf16(x[0], x[1]), ptx::pack_bf16(x[2], x[3]), ptx::pack_bf16(x[4], x[5]),
                                        ptx::pack_bf16(x[6], x[7]));
                }
            }
        };
#pragma unroll 1
        for (int q2 = 0; q2 < 2; ++q2) {  // two 32-column TMEM loads per wait
            uint32_t vv[2][32];
            ptx::tmem_ld32(tmem + ((uint32_t)(32 * sp) << 16) + TMA_BIG + 128 * ch + 64 * q2, vv[0]);
            ptx::tmem_ld32(tmem + ((uint32_t)(32 * sp) << 16) + TMA_BIG + 128 * ch + 64 * q2 + 32, vv[1]);
            ptx::tmem_wait_ld();
            store32(reinterpret_cast<const float *>(vv[0]), 64 * q2);
            store32(reinterpret_cast<const float *>(vv[1]), 64 * q2 + 32);
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    DC_SPLIT_MARK(8);
    if (*flag && tid == 0) {
        atomicExch(status, kStatusTimeout);
        // Let this CTA's own TMA loads land before its shared memory goes away.
        ptx::mbar_wait(&bars[BA_QT], 0);
        ptx::mbar_wait(&bars[BA_BOP], 0);
    }
    __syncthreads();
    if (warp == 0) ptx::tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- scan kernel
// One CTA per (batch x head, slice of W = 64 NB value columns): V', y and S restricted to a set of value
// columns depend only on S's same columns, so the slices of one head run independently (each reads the
// head's full A6 and Kh, which its sibling slices find in L2).  Narrow slices shorten the per-chunk chain
// and fill the GPU when there are few heads.
constexpr int kThreadsB = 128;
template <int NB>
struct ScanLayout {
    static constexpr int W = 64 * NB;                           // value columns of the slice
    static constexpr uint32_t A6 = 0;                           // two K-major SW128 blocks, 128 rows
    static constexpr uint32_t KH = 32768;                       // two MN-major SW128 blocks, 64 rows
    static constexpr uint32_t U = KH + 16384;                   // fp32, 2 NB SW128 blocks of 32 columns, 64 rows
    static constexpr uint32_t Y0 = U + 16384 * NB;              // NB SW128 blocks of 64 columns, 64 rows
    static constexpr uint32_t VP = Y0 + 8192 * NB;              // V' hi (NB blocks), then lo
    static constexpr uint32_t S = VP + 16384 * NB;              // S bf16, MN-major, NB blocks of 128 rows
    static constexpr uint32_t Y = S;                            // y staging (NB SW128 boxes) over S: between
                                                                //   MMA6's read of S and the tail's rewrite
    static constexpr uint32_t BAR = S + 16384 * NB;
    static constexpr uint32_t TMEMPTR = BAR + 8 * 5, FLAG = TMEMPTR + 4, PEND = FLAG + 4;
    static constexpr uint32_t SMEM = PEND + 12 + 1024;
    static constexpr uint32_t TM_D = 0, TM_S = W, TM_COLS = 2 * W;  // TMEM: [V'; y] and S
    static_assert(SMEM <= 232448, "scan kernel over the shared-memory limit");
};
enum BarB { BB_A6 = 0, BB_KH, BB_UY, BB_M6, BB_M7, kBarsB };

// Byte offset of 16-byte chunk `chunk` of row `row` in a SW128 tile.
__device__ __forceinline__ uint32_t sw128c(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

template <typename TO, int NB>
__global__ void __launch_bounds__(kThreadsB, 1)
    scan_kernel(const __grid_constant__ CUtensorMap tm_a6, const __grid_constant__ CUtensorMap tm_u,
                const __grid_constant__ CUtensorMap tm_y0, const __grid_constant__ CUtensorMap tm_kh,
                const __grid_constant__ CUtensorMap tm_y, const CoreParams p, const SplitWs ws, int *status) {
    using Ly = ScanLayout<NB>;
    constexpr int W = Ly::W;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    const uint32_t sb = ptx::smem_u32(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + Ly::BAR);
    uint32_t *tmem_ptr = reinterpret_cast<uint32_t *>(base + Ly::TMEMPTR);
    volatile int *flag = reinterpret_cast<volatile int *>(base + Ly::FLAG);
    volatile int *pend = reinterpret_cast<volatile int *>(base + Ly::PEND);
    constexpr bool kYTma = sizeof(TO) == 2;

    const int tid = threadIdx.x, warp = tid >> 5, r = tid;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const int slices = 128 / W;
    const int64_t bh = blockIdx.x / slices, b = bh / p.heads, h = bh % p.heads, nch = ws.nch;
    const int col0 = (int)(blockIdx.x % slices) * W;  // first value column of this slice
    const bool leader = tid == 0;

    if (leader) {
        *flag = 0;
        pend[0] = pend[1] = pend[2] = -1;
        for (int i = 0; i < kBarsB; ++i) ptx::mbar_init(&bars[i], 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_a6);
        ptx::prefetch_tmap(&tm_u);
        ptx::prefetch_tmap(&tm_y0);
        ptx::prefetch_tmap(&tm_kh);
        if (kYTma) ptx::prefetch_tmap(&tm_y);
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_ptr, Ly::TM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_ptr;

    auto load_a6 = [&](int64_t c) {
        pend[0] = (int)(c & 1);
        ptx::mbar_arrive_expect_tx(&bars[BB_A6], 32768);
        const int row = (int)((bh * nch + c) * 128);
        tma_load_2d(base + Ly::A6, &tm_a6, &bars[BB_A6], 0, row);
        tma_load_2d(base + Ly::A6 + 16384, &tm_a6, &bars[BB_A6], 64, row);
    };
    auto load_kh = [&](int64_t c) {
        pend[1] = (int)(c & 1);
        ptx::mbar_arrive_expect_tx(&bars[BB_KH], 16384);
        const int row = (int)((bh * nch + c) * 64);
        tma_load_2d(base + Ly::KH, &tm_kh, &bars[BB_KH], 0, row);
        tma_load_2d(base + Ly::KH + 8192, &tm_kh, &bars[BB_KH], 64, row);
    };
    auto load_uy = [&](int64_t c) {
        pend[2] = (int)(c & 1);
        ptx::mbar_arrive_expect_tx(&bars[BB_UY], 24576 * NB);
        const int row = (int)((bh * nch + c) * 64);
#pragma unroll
        for (int j = 0; j < 2 * NB; ++j) tma_load_2d(base + Ly::U + 8192 * j, &tm_u, &bars[BB_UY], col0 + 32 * j, row);
#pragma unroll
        for (int j = 0; j < NB; ++j) tma_load_2d(base + Ly::Y0 + 8192 * j, &tm_y0, &bars[BB_UY], col0 + 64 * j, row);
    };
    auto role_wait = [&](int bar, uint32_t parity) {
        const bool bad = !ptx::mbar_wait(&bars[bar], parity) || *flag != 0;
        if (ptx::named_sync_or(1, kThreadsB, bad)) {
            *flag = 1;
            return false;
        }
        return true;
    };

    if (leader) {
        load_a6(0);
        load_kh(0);
        load_uy(0);
    }

    // S0 (this slice's columns) -> TMEM (pre-scaled by chunk 0's decay) and its bf16 copy.
    {
        const float g0 = ws.gam[(bh * nch) * 128 + r];
        const float *src = p.state_in + (bh * 128 + r) * 128 + col0;
#pragma unroll 1
        for (int hh = 0; hh < NB; ++hh) {
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
                uint32_t v[32];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 f = *reinterpret_cast<const float4 *>(src + 64 * hh + 32 * q2 + 4 * q);
                    v[4 * q] = __float_as_uint(f.x);
                    v[4 * q + 1] = __float_as_uint(f.y);
                    v[4 * q + 2] = __float_as_uint(f.z);
                    v[4 * q + 3] = __float_as_uint(f.w);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float *f = reinterpret_cast<const float *>(v + 8 * q);
                    ptx::st_shared_v4(sb + Ly::S + hh * 16384 + ptx::sw128(r, 32 * q2 + 8 * q), ptx::pack_bf16(f[0], f[1]),
                                      ptx::pack_bf16(f[2], f[3]), ptx::pack_bf16(f[4], f[5]), ptx::pack_bf16(f[6], f[7]));
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * g0);
                ptx::tmem_st32(tmem + lane_base + Ly::TM_S + 64 * hh + 32 * q2, v);
            }
        }
        ptx::tmem_wait_st();
        ptx::fence_async_smem();
        ptx::tc_fence_before();
        ptx::named_sync(1, kThreadsB);
    }

    float gnext = (nch > 1) ? ws.gam[(bh * nch + 1) * 128 + r] : 1.f;
    bool ok = true;
    for (int64_t c = 0; c < nch && ok; ++c) {
        const uint32_t par = (uint32_t)(c & 1);
        const float gam_next = gnext;
        if (c + 2 < nch) gnext = ws.gam[(bh * nch + c + 2) * 128 + r];

        // ---- D = A6 S[:, slice] ----
        if (leader) {
            if (!ptx::mbar_wait(&bars[BB_A6], par)) {
                *flag = 1;
            } else {
                pend[0] = -1;
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, W, 0, 1);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    ptx::umma_bf16(tmem + Ly::TM_D, ptx::sdesc(sb + Ly::A6 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                                   ptx::sdesc(sb + Ly::S + kk * 2048, 16384, 1024), id, kk > 0);
                ptx::umma_commit(&bars[BB_M6]);
            }
        }
        if (!(ok = role_wait(BB_M6, par))) break;
        if (leader && c + 1 < nch) load_a6(c + 1);

        // ---- [V'; y] = D + [U; Y0]: V' hi + lo -> smem (MMA7's B), y -> HBM ----
        if (!(ok = role_wait(BB_UY, par))) break;
        if (leader) pend[2] = -1;
        ptx::tc_fence_after();
        {
            const int64_t tok = c * tc::kL + (r - 64);
            const bool write_y = r >= 64 && tok < p.seq;
            TO *yrow = static_cast<TO *>(p.y) + ((b * p.seq + (write_y ? tok : 0)) * p.heads + h) * 128 + col0;
#pragma unroll 1
            for (int hh = 0; hh < NB; ++hh) {
                uint32_t vv[2][32];
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_D + 64 * hh, vv[0]);
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_D + 64 * hh + 32, vv[1]);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    const float *f = reinterpret_cast<const float *>(vv[q2]);
                    if (r < 64) {
                        const uint32_t ub = sb + Ly::U + 8192 * (2 * hh + q2);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 u0 = ptx::ld_shared_v4(ub + sw128c(r, 2 * q));
                            const uint4 u1 = ptx::ld_shared_v4(ub + sw128c(r, 2 * q + 1));
                            const float x[8] = {f[8 * q] + __uint_as_float(u0.x),     f[8 * q + 1] + __uint_as_float(u0.y),
                                                f[8 * q + 2] + __uint_as_float(u0.z), f[8 * q + 3] + __uint_as_float(u0.w),
                                                f[8 * q + 4] + __uint_as_float(u1.x), f[8 * q + 5] + __uint_as_float(u1.y),
                                                f[8 * q + 6] + __uint_as_float(u1.z), f[8 * q + 7] + __uint_as_float(u1.w)};
                            uint32_t hi[4], lo[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                hi[e] = ptx::pack_bf16(x[2 * e], x[2 * e + 1]);
                                lo[e] = ptx::pack_bf16(x[2 * e] - ptx::bf16lo(hi[e]), x[2 * e + 1] - ptx::bf16hi(hi[e]));
                            }
                            const uint32_t off = hh * 8192 + ptx::sw128(r, 32 * q2 + 8 * q);
                            ptx::st_shared_v4(sb + Ly::VP + off, hi[0], hi[1], hi[2], hi[3]);
                            ptx::st_shared_v4(sb + Ly::VP + 8192 * NB + off, lo[0], lo[1], lo[2], lo[3]);
                        }
                    } else {
                        float yv[32];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 y0 = ptx::ld_shared_v4(sb + Ly::Y0 + hh * 8192 + ptx::sw128(r - 64, 32 * q2 + 8 * q));
                            const uint32_t yw[4] = {y0.x, y0.y, y0.z, y0.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                yv[8 * q + 2 * e] = f[8 * q + 2 * e] + ptx::bf16lo(yw[e]);
                                yv[8 * q + 2 * e + 1] = f[8 * q + 2 * e + 1] + ptx::bf16hi(yw[e]);
                            }
                        }
                        if (kYTma) {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                ptx::st_shared_v4(sb + Ly::Y + hh * 8192 + ptx::sw128(r - 64, 32 * q2 + 8 * q),
                                                  ptx::pack_bf16(yv[8 * q], yv[8 * q + 1]),
                                                  ptx::pack_bf16(yv[8 * q + 2], yv[8 * q + 3]),
                                                  ptx::pack_bf16(yv[8 * q + 4], yv[8 * q + 5]),
                                                  ptx::pack_bf16(yv[8 * q + 6], yv[8 * q + 7]));
                        } else if (write_y) {
                            tc::store_row32(yrow + 64 * hh + 32 * q2, yv);
                        }
                    }
                }
            }
        }
        ptx::fence_async_smem();
        ptx::tc_fence_before();
        ptx::named_sync(1, kThreadsB);
        if (leader) {
            if (kYTma) {
#pragma unroll
                for (int j = 0; j < NB; ++j)
                    ptx::tma_store_4d(&tm_y, sb + Ly::Y + 8192 * j, col0 + 64 * j, (int)h, (int)(c * tc::kL), (int)b);
                ptx::bulk_commit();
            }
            if (c + 1 < nch) load_uy(c + 1);
        }

        // ---- S[:, slice] <- diag(gam) S + Kh^T (V'hi + V'lo); TMEM S already holds diag(gam) S ----
        if (leader) {
            if (!ptx::mbar_wait(&bars[BB_KH], par)) {
                *flag = 1;
            } else {
                pend[1] = -1;
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, W, 1, 1);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    ptx::umma_bf16(tmem + Ly::TM_S, ptx::sdesc(sb + Ly::KH + (kk & 3) * 2048, 8192, 1024),
                                   ptx::sdesc(sb + Ly::VP + (kk >= 4 ? 8192 * NB : 0) + (kk & 3) * 2048, 8192, 1024), id,
                                   1);
                ptx::umma_commit(&bars[BB_M7]);
            }
            if (kYTma) ptx::bulk_wait_all();  // the y tile (over S) has been read before the tail rewrites S
        }
        if (!(ok = role_wait(BB_M7, par))) break;
        if (leader && c + 1 < nch) load_kh(c + 1);

        // ---- S -> bf16 operand, and the accumulator pre-scaled by the next chunk's decay ----
        ptx::tc_fence_after();
        if (c + 1 < nch) {
#pragma unroll 1
            for (int hh = 0; hh < NB; ++hh) {
                uint32_t vv[2][32];
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_S + 64 * hh, vv[0]);
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_S + 64 * hh + 32, vv[1]);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    uint32_t(&v)[32] = vv[q2];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float *f = reinterpret_cast<const float *>(v + 8 * q);
                        ptx::st_shared_v4(sb + Ly::S + hh * 16384 + ptx::sw128(r, 32 * q2 + 8 * q), ptx::pack_bf16(f[0], f[1]),
                                          ptx::pack_bf16(f[2], f[3]), ptx::pack_bf16(f[4], f[5]),
                                          ptx::pack_bf16(f[6], f[7]));
                    }
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * gam_next);
                    ptx::tmem_st32(tmem + lane_base + Ly::TM_S + 64 * hh + 32 * q2, v);
                }
            }
            ptx::tmem_wait_st();
            ptx::fence_async_smem();
            ptx::tc_fence_before();
            ptx::named_sync(1, kThreadsB);
        } else {
            float *dst = p.state_out + (bh * 128 + r) * 128 + col0;
#pragma unroll 1
            for (int hh = 0; hh < NB; ++hh) {
                uint32_t vv[2][32];
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_S + 64 * hh, vv[0]);
                ptx::tmem_ld32(tmem + lane_base + Ly::TM_S + 64 * hh + 32, vv[1]);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2)
                    tc::store_row32(dst + 64 * hh + 32 * q2, reinterpret_cast<const float *>(vv[q2]));
            }
        }
    }

    if (kYTma && leader) ptx::bulk_wait_all();
    ptx::tc_fence_before();
    __syncthreads();
    if (*flag) {
        if (leader) {
            atomicExch(status, kStatusTimeout);
            // Let this CTA's own TMA loads land before its shared memory goes away.
            if (pend[0] >= 0) ptx::mbar_wait(&bars[BB_A6], (uint32_t)pend[0]);
            if (pend[1] >= 0) ptx::mbar_wait(&bars[BB_KH], (uint32_t)pend[1]);
            if (pend[2] >= 0) ptx::mbar_wait(&bars[BB_UY], (uint32_t)pend[2]);
        }
        __syncthreads();
    }
    if (warp == 0) ptx::tmem_dealloc(tmem, Ly::TM_COLS);
}

}  // namespace split

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Whether the split kernels serve this request (given enough workspace): bf16 q/k/v, d = 128, one
// micro-step per token, and a per-channel gate somewhere (or DC_FLAG_FORCE_SPLIT = 0x4).
inline bool split_applies(const CoreParams &p, int32_t in_dtype, uint32_t flags) {
    if (flags & 0x3u) return false;  // DC_FLAG_FORCE_SIMT, DC_FLAG_RECURRENT
    if (in_dtype != 1) return false;
    if (p.dk != 128 || p.dv != 128 || p.u != 1) return false;
    if (!((flags & 0x4u) || p.ew != 1 || p.ww != 1 || p.gw > 1)) return false;
    if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) || !aligned16(p.y) || !aligned16(p.state_in) ||
        !aligned16(p.state_out))
        return false;
    const int64_t bhn = p.batch * p.heads;
    const int64_t nch = (p.seq + tc::kL - 1) / tc::kL;
    if (bhn > 65535 || nch > 0x7fffffff || bhn * nch * 128 > 0x7fffffff) return false;
    return true;
}

inline uint64_t split_workspace_bytes(const CoreParams &p) {
    const int64_t nch = (p.seq + tc::kL - 1) / tc::kL;
    return (uint64_t)(p.batch * p.heads * nch) * split::kWsBytesPerChunk;
}

inline split::SplitWs split_carve(const CoreParams &p, void *ws) {
    const int64_t nch = (p.seq + tc::kL - 1) / tc::kL;
    const uint64_t n = (uint64_t)(p.batch * p.heads * nch);
    uint8_t *w = static_cast<uint8_t *>(ws);
    split::SplitWs s;
    s.a6 = reinterpret_cast<__nv_bfloat16 *>(w);
    s.u = reinterpret_cast<float *>(w + n * 32768);
    s.y0 = reinterpret_cast<__nv_bfloat16 *>(w + n * 65536);
    s.kh = reinterpret_cast<__nv_bfloat16 *>(w + n * 81920);
    s.gam = reinterpret_cast<float *>(w + n * 98304);
    s.nch = nch;
    return s;
}

// A 2-D [rows][inner] tensor map with a (box_inner, box_rows) SW128 box.
inline bool encode_2d(CUtensorMap *m, CUtensorMapDataType dt, uint32_t esize, const void *ptr, uint64_t inner,
                      uint64_t rows, uint32_t box_inner, uint32_t box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(inner * esize)};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename TG, typename TO>
int launch_split_typed(const CoreParams &p, void *workspace, cudaStream_t stream) {
    const split::SplitWs ws = split_carve(p, workspace);
    const int64_t bhn = p.batch * p.heads;
    const uint64_t n = (uint64_t)(bhn * ws.nch);
    CUtensorMap ma6, mu, my0, mkh, my, mq, mk, mbop, mqt;
    if (!encode_rows(&mq, p.q, p.heads, p.seq, p.batch) || !encode_rows(&mk, p.k, p.heads, p.seq, p.batch) ||
        !encode_2d(&mbop, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws.a6, 128, n * 128, 64, 64) ||
        !encode_2d(&mqt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws.y0, 128, n * 64, 64, 64) || !encode_2d(&ma6, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws.a6, 128, n * 128, 64, 128) ||
        !encode_2d(&mu, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws.u, 128, n * 64, 32, 64) ||
        !encode_2d(&my0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws.y0, 128, n * 64, 64, 64) ||
        !encode_2d(&mkh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws.kh, 128, n * 64, 64, 64) ||
        (sizeof(TO) == 2 ? !encode_rows(&my, p.y, p.heads, p.seq, p.batch) : (my = ma6, false))) {
        g_tc_error = (int)cudaErrorInvalidValue;
        return 6;  // DC_ECUDA
    }
    int *status = device_status_ptr();
    if (!status) {
        g_tc_error = (int)cudaErrorInvalidSymbol;
        return 6;
    }
    // The scan runs in 64-column value slices: two CTAs per SM and a shorter per-chunk chain than whole heads.
    constexpr int kNB = 1;
    using Ly = split::ScanLayout<kNB>;
    auto ka = split::prep_kernel<TG>;
    auto kb = split::scan_kernel<TO, kNB>;
    cudaError_t e = cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)split::kSmemA);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ly::SMEM);
    if (e == cudaSuccess) {
        ka<<<dim3((unsigned)ws.nch, (unsigned)bhn), split::kThreadsA, split::kSmemA, stream>>>(mq, mk, mbop, mqt, p,
                                                                                                 ws, status);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        kb<<<(unsigned)(bhn * (128 / Ly::W)), split::kThreadsB, Ly::SMEM, stream>>>(ma6, mu, my0, mkh, my, p, ws,
                                                                                       status);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        g_tc_error = (int)e;
        return 6;
    }
    return 0;
}

inline int launch_chunk_split(const CoreParams &p, int32_t gate_dtype, int32_t out_dtype, void *workspace,
                              cudaStream_t stream) {
    switch (gate_dtype * 2 + out_dtype) {
        case 0: return launch_split_typed<float, float>(p, workspace, stream);
        case 1: return launch_split_typed<float, __nv_bfloat16>(p, workspace, stream);
        case 2: return launch_split_typed<__nv_bfloat16, float>(p, workspace, stream);
        case 3: return launch_split_typed<__nv_bfloat16, __nv_bfloat16>(p, workspace, stream);
    }
    return 3;  // DC_EUNSUPPORTED_DTYPE
}

}  // namespace dc
