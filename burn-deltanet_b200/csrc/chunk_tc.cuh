// chunk_tc.cuh — the tensor-core (tcgen05 / TMEM / TMA) chunkwise WY prefill.
//
// Serves dc_chunk_fwd for bf16 q/k/v with dk = dv = 128 and per-head gates
// (DeltaNet, Gated DeltaNet and DeltaProduct with its micro-steps folded in).  One CTA owns one (batch, head)
// and walks its chunks of L = 64 steps; the fp32 state S lives in tensor
// memory for the whole sequence and never touches HBM in between.
//
// Per chunk (rows i, j in [0, 64); G = chunk cumsum of g, gam_i = e^{G_i}):
//
//   D1   = [K; Q] K^T                                   M=128 N=64  K=128   (tcgen05)
//   Akk  = tril(e_i (k_i.k_j) e^{G_i-G_j}, -1)           fp32, shared memory (CUDA cores)
//   Aqk  = tril(s (q_i.k_j) e^{G_i-G_j}, 0)              bf16 operand
//   T    = (I + Akk)^-1                                  16x16 blocks, forward substitution
//   Tb   = T diag(w),  Tw = T diag(e gam)                bf16 hi + lo operands
//   D_P  = Aqk [Tb | Tw]                                 M=64  N=128 K=64    (tcgen05)
//   D_UY = [Tb; Aqk Tb] V      = [U; Aqk U]              M=128 N=128 K=64    (tcgen05, hi + lo)
//   D_W  = [Tw; Aqk Tw] K      = [W; Aqk W]              M=128 N=128 K=64    (tcgen05, hi + lo)
//   A6   = [-W; s gam Q - Aqk W]                         bf16, written into TMEM over D_W
//   D_UY += A6 S               = [U - W S; y]            M=128 N=128 K=128   (tcgen05, A from TMEM)
//   D_S  = Gam S + K^T diag(e^{G_63 - G_j}) V'           M=128 N=128 K=64    (tcgen05, hi + lo, accumulate)
//
// The D_UY += A6 S line is the reference's scan step (src/delta/chunk.rs:
// 177-187) with its two S products stacked into one M=128 MMA: V' = U - W S
// comes out in the top 64 TMEM lanes and y = (s gam Q) S + Aqk V' =
// (s gam Q - Aqk W) S + Aqk U in the bottom 64, because Aqk U and Aqk W are
// S-independent and formed before S is needed.  The last line is chunk.rs:
// 191-202 with the per-row decay folded into V'.
//
// Warp specialisation.  Everything above D_UY += A6 S depends only on the
// chunk's own inputs; only the last three lines depend on S.  Warps 0-7
// (the "parallel" role) build chunk c+1's operands (masks, solve, Tb/Tw,
// Pb/Pw) while warps 8-11 (the "serial" role) run chunk c's S chain (A6,
// V'/y, the state update), so the two chains' latencies overlap.  Warp 12
// issues D1 and the D_UY/D_W products ("MMA4"): an MMA issue blocks its
// thread while the tensor pipe accepts the MMAs, so neither role waits on
// it.  It puts chunk c+1's D1 ahead of chunk c's MMA4 in the (in-order)
// tensor pipe once chunk c+1's tiles have landed, so that the next chunk's
// masks need not wait for MMA4.  The roles meet on mbarriers: the serial role
// waits for chunk c's D_W (A6) and D_UY (its MMA), the issue warp for the
// parallel role's operands and for the serial role to release chunk c-1's
// D_UY/D_W (after V'/y), and the parallel role for MMA4 to have read the
// buffers it rewrites (the T buffer, then the hi / lo operands).
//
// T (through Tb, Tw and their Aqk products) and V' enter their products as
// two bf16 terms each (hi + lo, the rounding residual of hi), i.e. at ~16
// significant bits instead of bf16's 8: T's long alternating tails (a chunk
// of near-parallel keys) and V''s rounding are otherwise the largest errors
// in the fp32 state.  The inputs q, k, v are exact in bf16.
//
// Operand layouts in shared memory are the 128-byte-swizzled canonical ones
// (8 rows x 128 B atoms): tiles written by TMA with CU_TENSOR_MAP_SWIZZLE_128B
// and tiles written by threads through ptx::sw128 share one pattern, so the
// same bytes serve as a K-major operand of one MMA and an MN-major operand of
// another.  V' (hi, lo) is written into the consumed stage's V and Q slots,
// and bf16 y is staged for its TMA store in the S operand buffer, which the
// state update rewrites only after MMA6 has read it and the store has left.
//
// Every mbarrier wait is bounded (ptx::kWaitLimitNs); a wait that runs out
// sets the library's device status word, the CTA waits (bounded) for its own
// TMA loads still in flight, frees its tensor memory and returns.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "ptx.cuh"

namespace dc {

// Device status word written by kernels whose bounded waits run out (0 = ok).
__device__ int g_device_status;
constexpr int kStatusTimeout = 1;

namespace tc {

constexpr int kParThreads = 256;  // warps 0-7: the S-independent ("parallel") role
constexpr int kSerThreads = 128;  // warps 8-11: the S chain ("serial") role
constexpr int kIssueWarp = 12;    // warp 12: issues D1 and MMA4 (an issue blocks its thread while the
                                  // tensor pipe accepts the MMAs, so no role waits on it)
constexpr int kThreads = kParThreads + kSerThreads + 32;
constexpr int kL = 64;    // chunk rows
constexpr int kD = 128;   // dk = dv
constexpr int kAP = 68;   // row pitch (floats) of the fp32 Akk and T tiles

// Shared-memory map (bytes from a 1024-aligned base).
constexpr uint32_t kStageBytes = 49152;                 // [K|Q d0-63][K|Q d64-127][V d0-63][V d64-127]
constexpr uint32_t OFF_STAGE = 0;                       // two stages
constexpr uint32_t OFF_AU = 2 * kStageBytes;            // [Tb; Pb] hi, 128x64 bf16 K-major
constexpr uint32_t OFF_AW = OFF_AU + 16384;             // [Tw; Pw] hi
constexpr uint32_t OFF_S = OFF_AW + 16384;              // S bf16, MN-major, two 64-column blocks of 16 KB; once
                                                        // MMA6 has read it, block h stages y columns 64h..
constexpr uint32_t OFF_AQK = OFF_S + 32768;             // Aqk bf16 64x64 K-major
constexpr uint32_t OFF_AF = OFF_AQK + 8192;             // [Tb; Pb] lo
constexpr uint32_t OFF_TF = OFF_AF + 64 * kAP * 4;      // T fp32 [64][68];   then [Tw; Pw] lo
constexpr uint32_t OFF_AK = OFF_TF + 64 * kAP * 4;      // Akk fp32 [64][68]; E blocks above its diagonal
// Gate slots: chunk c's gates live in slot c % 3.  Three, not two: the operand role writes chunk c+2's
// gates as soon as it finishes chunk c+1, which can be before the state role has read chunk c's (A6, V'/y);
// it can only start chunk c+3 after chunk c+1's MMA4, which waits for the state role to release chunk c.
constexpr int kGateSlots = 3;
constexpr uint32_t OFF_GATE = OFF_AK + 64 * kAP * 4;             // per slot: e[64], w[64], g[64]
constexpr uint32_t OFF_G = OFF_GATE + kGateSlots * 3 * 64 * 4;   // per slot: G[64], gam[64]
constexpr uint32_t OFF_BAR = OFF_G + kGateSlots * 2 * 64 * 4;    // mbarriers (below)
constexpr int kBars = 13;
constexpr uint32_t OFF_TMEMPTR = OFF_BAR + kBars * 8;
constexpr uint32_t OFF_FLAG = OFF_TMEMPTR + 4;
constexpr uint32_t OFF_PEND = OFF_FLAG + 4;             // int[2]: parity of a stage's TMA load in flight, or -1
constexpr uint32_t OFF_NORMW = (OFF_PEND + 8 + 15) & ~15u;  // the fused output norm's weight [128] fp32
constexpr uint32_t kSmemUsed = OFF_NORMW + 512;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;       // alignment slack
static_assert(OFF_AF % 1024 == 0 && OFF_TF % 1024 == 0 && OFF_AQK % 1024 == 0 && OFF_S % 1024 == 0,
              "operand tiles need 1 KB alignment");
static_assert(kSmemBytes <= 232448, "over the 227 KB per-CTA shared-memory limit");

// mbarrier slots.  MMA4 commits twice: B_MMA4W once its D_W half (reading [Tw; Pw] and the T buffer) is
// done, B_MMA4 once all of it is.  B_OPS: the operand role has finished a chunk (TM_A free, MMA4's
// operands written).
enum Bar { B_TMA0 = 0, B_TMA1, B_MMA1, B_MMAP, B_MMA4W, B_MMA4, B_MMA6, B_MMA7, B_UY_FREE, B_OPS, B_GATE0 };
static_assert(B_GATE0 + kGateSlots == kBars, "barrier count");

// TMEM columns (512 allocated): A = D1 / D_P, W = D_W (then A6), UY = D_UY, S = D_S.
constexpr uint32_t TM_A = 0, TM_W = 128, TM_UY = 256, TM_S = 384;

// Named barriers of the two roles (id 0 is __syncthreads).
constexpr uint32_t NB_PAR = 1, NB_SER = 2;

__device__ __forceinline__ float gate_at(const float *p) { return *p; }
__device__ __forceinline__ float gate_at(const __nv_bfloat16 *p) { return __bfloat162float(*p); }

// e, w (per folded row) and g (per token, on micro-step 0) of one chunk row;
// thread `t` in [0, 192) loads e (t < 64), w (t < 128) or g of row t % 64.
template <typename TG>
__device__ __forceinline__ float load_gate(const CoreParams &p, int64_t b, int64_t h, int64_t c, int t) {
    const int which = t >> 6, l = t & 63;
    const int64_t P = p.seq * p.u;
    const int64_t pos = c * kL + l;
    if (pos >= P) return 0.f;
    const TG *e = static_cast<const TG *>(p.erase), *w = static_cast<const TG *>(p.write);
    const TG *g = static_cast<const TG *>(p.g);
    if (which == 0) return gate_at(e + (b * P + pos) * p.heads + h);
    if (which == 1) return gate_at(w + (b * P + pos) * p.heads + h);
    if (p.gw == 0) return 0.f;
    if (p.u == 1) return gate_at(g + (b * p.seq + pos) * p.heads + h);
    if ((pos % p.u) != 0) return 0.f;
    return gate_at(g + (b * p.seq + pos / p.u) * p.heads + h);
}

// The micro-step fold (DeltaProduct / GDN-2, u = n_householder): chunk c
// covers folded rows 64c .. 64c + 63, and token t reads out at folded row
// t*u + u - 1 (src/delta_product/delta_product.rs:178-228).  The chunk's Q
// tile holds the 64 token rows from q_first(c) = floor(64c / u), the first
// token whose readout falls in the chunk; row i of the tile reads out at
// chunk row q_pos(c, i), or nowhere (-1).  For u = 1 both are the identity.
__device__ __forceinline__ int64_t q_first(int64_t c, int u) { return (c * kL) / u; }
__device__ __forceinline__ int q_pos(int64_t c, int i, const CoreParams &p) {
    const int64_t t = q_first(c, p.u) + i;
    const int64_t pos = t * p.u + p.u - 1 - c * kL;
    return (t < p.seq && pos < kL) ? (int)pos : -1;
}

// 32 consecutive outputs of one row, as 16-byte stores.
__device__ __forceinline__ void store_row32(float *dst, const float *f) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4 *>(dst)[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
}
__device__ __forceinline__ void store_row32(__nv_bfloat16 *dst, const float *f) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
        reinterpret_cast<uint4 *>(dst)[q] =
            make_uint4(ptx::pack_bf16(f[8 * q], f[8 * q + 1]), ptx::pack_bf16(f[8 * q + 2], f[8 * q + 3]),
                       ptx::pack_bf16(f[8 * q + 4], f[8 * q + 5]), ptx::pack_bf16(f[8 * q + 6], f[8 * q + 7]));
}

// Phase timestamps for performance work: compiled out unless a build defines
// DC_TC_MARK(id) (the chunk index `c` is in scope at every mark).
#ifndef DC_TC_MARK
#define DC_TC_MARK(id)
#endif

// E_pq (p > q) is kept in the mirrored block (q, p) of the Akk buffer: the blocks above the diagonal
// hold values that nothing reads once the solve has started.
__device__ __forceinline__ float *eblock(float *Af, int p, int q) { return Af + (16 * q) * kAP + 16 * p; }

// D(16x8) += A(16 x K) B(K x 8) for fp32 operands in shared memory (row
// pitches lda, ldb), on the warp's tensor cores in three tf32 passes
// (big*big + big*small + small*big: ~2^-20 relative, fp32-class), each pass
// in its own accumulator so the three dependency chains overlap.
__device__ __forceinline__ void mma_rows16(float (&d)[4], const float *A, int lda, const float *B, int ldb, int K) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    float ds[4] = {0.f, 0.f, 0.f, 0.f}, dt[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 8) {
        const float av[4] = {A[g * lda + k0 + t], A[(g + 8) * lda + k0 + t], A[g * lda + k0 + t + 4],
                             A[(g + 8) * lda + k0 + t + 4]};
        const float bv[2] = {B[(k0 + t) * ldb + g], B[(k0 + t + 4) * ldb + g]};
        uint32_t ab[4], as[4], bb[2], bs[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) ptx::split_tf32(av[e], ab[e], as[e]);
#pragma unroll
        for (int e = 0; e < 2; ++e) ptx::split_tf32(bv[e], bb[e], bs[e]);
        ptx::mma_tf32_16x8x8(ds, as, bb);
        ptx::mma_tf32_16x8x8(dt, ab, bs);
        ptx::mma_tf32_16x8x8(d, ab, bb);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] += ds[e] + dt[e];
}

// Store a D fragment (16x8) to shared memory, scaled.
__device__ __forceinline__ void store_frag(float *D, int ld, const float (&d)[4], float scale) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    *reinterpret_cast<float2 *>(D + g * ld + 2 * t) = make_float2(scale * d[0], scale * d[1]);
    *reinterpret_cast<float2 *>(D + (g + 8) * ld + 2 * t) = make_float2(scale * d[2], scale * d[3]);
}

// T = (I + A)^-1 for the 64x64 strictly lower A in Af (row pitch kAP), into Tf
// (same pitch; blocks above the diagonal are left untouched, the upper
// triangles of the diagonal blocks are written as zeros).  Run by the 256
// threads of the operand role; only Af's strictly lower part is read, and the
// E blocks overwrite its upper blocks.
//  (1) diagonal blocks T_pp = (I + A_pp)^-1, one per warp, a lane substituting
//      down one column;
//  (2) E_pq = T_pp A_pq for the six blocks below the diagonal;
//  (3) T_pq = -sum_{r=q}^{p-1} E_pr T_rq by distance p - q = 1, 2, 3.
// (2) and (3) run on the warps' tensor cores in three tf32 passes (fp32-class).
// mark_diag / mark_e are called after (1) and (2) (phase-timing hooks).
template <typename M1, typename M2>
__device__ __forceinline__ void solve_unit_lower(float *Af, float *Tf, int warp, int lane,
                                                 M1 &&mark_diag, M2 &&mark_e) {
    if (warp < 4 && lane < 16) {
        const int pb = warp, j = lane;
        const float *A = Af + (16 * pb) * kAP + 16 * pb;
        float tcol[16];
#pragma unroll
        for (int a = 0; a < 16; ++a) {
            float acc0 = (a == j) ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
            for (int m = 0; m < a; m += 4) {
                const float4 av = *reinterpret_cast<const float4 *>(A + a * kAP + m);
                acc0 = fmaf(-av.x, tcol[m], acc0);
                if (m + 1 < a) acc1 = fmaf(-av.y, tcol[m + 1], acc1);
                if (m + 2 < a) acc0 = fmaf(-av.z, tcol[m + 2], acc0);
                if (m + 3 < a) acc1 = fmaf(-av.w, tcol[m + 3], acc1);
            }
            tcol[a] = acc0 + acc1;
        }
#pragma unroll
        for (int a = 0; a < 16; ++a) Tf[(16 * pb + a) * kAP + 16 * pb + j] = tcol[a];
    }
    ptx::named_sync(NB_PAR, kParThreads);
    mark_diag();
    if (warp < 6) {  // six independent blocks, one per warp
        const int pr = warp < 1 ? 1 : (warp < 3 ? 2 : 3), q = warp - pr * (pr - 1) / 2;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            mma_rows16(d, Tf + (16 * pr) * kAP + 16 * pr, kAP, Af + (16 * pr) * kAP + 16 * q + 8 * nt, kAP, 16);
            store_frag(eblock(Af, pr, q) + 8 * nt, kAP, d, 1.f);
        }
    }
    ptx::named_sync(NB_PAR, kParThreads);
    mark_e();
#pragma unroll
    for (int dist = 1; dist < 4; ++dist) {
        if (warp < 2 * (4 - dist)) {  // (4 - dist) blocks x 2 column halves, one per warp
            const int q = warp >> 1, nt = warp & 1, pr = q + dist;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int rr = q; rr < pr; ++rr)
                mma_rows16(d, eblock(Af, pr, rr), kAP, Tf + (16 * rr) * kAP + 16 * q + 8 * nt, kAP, 16);
            store_frag(Tf + (16 * pr) * kAP + 16 * q + 8 * nt, kAP, d, -1.f);
        }
        ptx::named_sync(NB_PAR, kParThreads);
    }
}

// NORM: the plain output norm in the read-out (a separate instantiation, so the plain prefill carries
// none of its code).
template <typename TG, typename TO, bool NORM>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_y,
                    const CoreParams p, int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    const uint32_t sb = ptx::smem_u32(base);
    float *Ak = reinterpret_cast<float *>(base + OFF_AK);
    float *Tf = reinterpret_cast<float *>(base + OFF_TF);
    float *gates = reinterpret_cast<float *>(base + OFF_GATE);  // [slot][e | w | g][64]
    float *Gs = reinterpret_cast<float *>(base + OFF_G);        // [slot][G | gam][64]
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + OFF_BAR);
    uint32_t *tmem_ptr = reinterpret_cast<uint32_t *>(base + OFF_TMEMPTR);
    volatile int *flag = reinterpret_cast<volatile int *>(base + OFF_FLAG);
    volatile int *pend = reinterpret_cast<volatile int *>(base + OFF_PEND);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t bh = blockIdx.x, b = bh / p.heads, h = bh % p.heads;
    const int64_t P = p.seq * p.u;
    const int64_t nchunks = (P + kL - 1) / kL;
    const bool gated = p.gw > 0;
    const float scale = p.scale;
    // bf16 y leaves through staged TMA stores (keeps the load/store pipe free for the operand role);
    // fp32 y is stored row by row.
    constexpr bool kYTma = sizeof(TO) == 2;

    if (tid == 0) {
        *flag = 0;
        pend[0] = pend[1] = -1;
        for (int i = 0; i < kBars; ++i) ptx::mbar_init(&bars[i], 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_k);
        ptx::prefetch_tmap(&tm_q);
        ptx::prefetch_tmap(&tm_v);
        if (kYTma) ptx::prefetch_tmap(&tm_y);
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_ptr, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_ptr;

    // One chunk's q/k/v tiles pulled into L2 ahead of their load into a stage.
    auto prefetch_tiles = [&](int64_t c) {
        const int row = (int)(c * kL), qrow = (int)q_first(c, p.u);
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            ptx::tma_prefetch_4d(&tm_k, 64 * x, (int)h, row, (int)b);
            ptx::tma_prefetch_4d(&tm_q, 64 * x, (int)h, qrow, (int)b);
            ptx::tma_prefetch_4d(&tm_v, 64 * x, (int)h, row, (int)b);
        }
    };
    // One chunk's q/k/v tiles into stage `st`, completing on its mbarrier.
    auto issue_tma = [&](int64_t c, int st) {
        uint64_t *bar = &bars[B_TMA0 + st];
        uint8_t *stg = base + OFF_STAGE + st * kStageBytes;
        const int row = (int)(c * kL);
        pend[st] = (int)((c >> 1) & 1);
        ptx::mbar_arrive_expect_tx(bar, kStageBytes);
        ptx::tma_load_4d(stg + 0, &tm_k, bar, 0, (int)h, row, (int)b);
        ptx::tma_load_4d(stg + 16384, &tm_k, bar, 64, (int)h, row, (int)b);
        const int qrow = (int)q_first(c, p.u);
        ptx::tma_load_4d(stg + 8192, &tm_q, bar, 0, (int)h, qrow, (int)b);
        ptx::tma_load_4d(stg + 24576, &tm_q, bar, 64, (int)h, qrow, (int)b);
        ptx::tma_load_4d(stg + 32768, &tm_v, bar, 0, (int)h, row, (int)b);
        ptx::tma_load_4d(stg + 40960, &tm_v, bar, 64, (int)h, row, (int)b);
    };

    if (warp < 8) {
        // =============================== parallel role: chunk c's operands ===============================
        const int sp = warp & 3, ch = warp >> 2;  // TMEM subpartition, column half
        const int r = 32 * sp + lane;
        const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
        const bool leader = (tid == 0);
        auto par_wait = [&](int bar, uint32_t parity) {
            // A wait that ran out anywhere (here, or already flagged by either role) stops every operand
            // thread at the same point.
            const bool bad = !ptx::mbar_wait(&bars[bar], parity) || *flag != 0;
            if (ptx::named_sync_or(NB_PAR, kParThreads, bad)) {
                *flag = 1;
                return false;
            }
            return true;
        };
        if (leader && !p.stall) {  // (the stall test hook withholds the loads: every wait on them runs out)
            issue_tma(0, 0);
            if (nchunks > 1) issue_tma(1, 1);
        }
        float gnext = (tid < 192) ? load_gate<TG>(p, b, h, 0, tid) : 0.f;

        for (int64_t c = 0; c < nchunks; ++c) {
            const int gsl = (int)(c % kGateSlots);
            const float *ge = gates + (gsl * 3 + 0) * 64;
            const float *gw = gates + (gsl * 3 + 1) * 64;
            float *Gc = Gs + gsl * 128;
            float *gam = Gc + 64;
            DC_TC_MARK(0);

            // ---- chunk c's gates -> G = cumsum(g), gam = e^G; published to the serial role ----
            if (tid < 192) gates[gsl * 192 + tid] = gnext;
            ptx::named_sync(NB_PAR, kParThreads);
            if (c + 1 < nchunks && tid < 192) gnext = load_gate<TG>(p, b, h, c + 1, tid);
            if (warp == 0) {
                const float *g = gates + (gsl * 3 + 2) * 64;
                const float x0 = g[2 * lane], x1 = g[2 * lane + 1];
                float s = x0 + x1;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float t = __shfl_up_sync(0xffffffffu, s, off);
                    if (lane >= off) s += t;
                }
                Gc[2 * lane + 1] = s;
                Gc[2 * lane] = s - x1;
                gam[2 * lane + 1] = __expf(s);
                gam[2 * lane] = __expf(s - x1);
            }
            ptx::named_sync(NB_PAR, kParThreads);
            if (leader) ptx::mbar_arrive(&bars[B_GATE0 + gsl]);
            DC_TC_MARK(1);

            // ---- D1 = [K; Q] K^T, issued by the issue warp once chunk c's tiles landed ----
            if (!par_wait(B_MMA1, (uint32_t)(c & 1))) break;
            DC_TC_MARK(2);

            // ---- masks: Akk (fp32, rows 0-63 of D1) and Aqk (bf16 operand, rows 64-127) ----
            ptx::tc_fence_after();
            {
                uint32_t v[32];
                ptx::tmem_ld32(tmem + lane_base + TM_A + 32 * ch, v);
                ptx::tmem_wait_ld();
                // Akk row i = r; Aqk row r - 64 reads out at chunk row pq (causal up to pq).
                const int i = (r < 64) ? r : q_pos(c, r - 64, p);
                const float coef = (r < 64) ? ge[r] : (i >= 0 ? scale : 0.f);
                float a[32];
                if (gated) {
                    const float Gi = Gc[i & 63];
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        a[jj] = coef * __uint_as_float(v[jj]) * __expf(Gi - Gc[32 * ch + jj]);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) a[jj] = coef * __uint_as_float(v[jj]);
                }
                if (r < 64) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int j = 32 * ch + 4 * q;
                        *reinterpret_cast<float4 *>(Ak + i * kAP + j) =
                            make_float4(j < i ? a[4 * q] : 0.f, j + 1 < i ? a[4 * q + 1] : 0.f,
                                        j + 2 < i ? a[4 * q + 2] : 0.f, j + 3 < i ? a[4 * q + 3] : 0.f);
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float m[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) m[e] = (32 * ch + 8 * q + e <= i) ? a[8 * q + e] : 0.f;
                        ptx::st_shared_v4(sb + OFF_AQK + ptx::sw128(r - 64, 32 * ch + 8 * q), ptx::pack_bf16(m[0], m[1]),
                                          ptx::pack_bf16(m[2], m[3]), ptx::pack_bf16(m[4], m[5]),
                                          ptx::pack_bf16(m[6], m[7]));
                    }
                }
            }
            ptx::fence_async_smem();
            ptx::tc_fence_before();
            ptx::named_sync(NB_PAR, kParThreads);
            DC_TC_MARK(3);

            // ---- T = (I + Akk)^-1 in 16x16 blocks, into the buffer chunk c-1's [Tw; Pw] lo occupied ----
            if (c > 0 && !par_wait(B_MMA4W, (uint32_t)((c - 1) & 1))) break;
            solve_unit_lower(Ak, Tf, warp, lane, [&] { DC_TC_MARK(14); }, [&] { DC_TC_MARK(15); });
            DC_TC_MARK(4);

            // ---- Tb = T diag(w), Tw = T diag(e gam) as bf16 hi + lo (blocks above the diagonal masked) ----
            // Every A operand buffer of chunk c-1's MMA4 is rewritten from here on.
            if (c > 0 && !par_wait(B_MMA4, (uint32_t)((c - 1) & 1))) break;
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
                ptx::named_sync(NB_PAR, kParThreads);  // every T read is done before the T buffer is overwritten
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int j = j0 + 8 * q;
                    uint32_t bhi[4], blo[4], whi[4], wlo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j1 = j + 2 * e;
                        const float b0 = t[8 * q + 2 * e] * gw[j1], b1 = t[8 * q + 2 * e + 1] * gw[j1 + 1];
                        const float w0 = t[8 * q + 2 * e] * ge[j1] * gam[j1];
                        const float w1 = t[8 * q + 2 * e + 1] * ge[j1 + 1] * gam[j1 + 1];
                        bhi[e] = ptx::pack_bf16(b0, b1);
                        blo[e] = ptx::pack_bf16(b0 - ptx::bf16lo(bhi[e]), b1 - ptx::bf16hi(bhi[e]));
                        whi[e] = ptx::pack_bf16(w0, w1);
                        wlo[e] = ptx::pack_bf16(w0 - ptx::bf16lo(whi[e]), w1 - ptx::bf16hi(whi[e]));
                    }
                    const uint32_t off = ptx::sw128(i, j);
                    ptx::st_shared_v4(sb + OFF_AU + off, bhi[0], bhi[1], bhi[2], bhi[3]);
                    ptx::st_shared_v4(sb + OFF_AF + off, blo[0], blo[1], blo[2], blo[3]);
                    ptx::st_shared_v4(sb + OFF_AW + off, whi[0], whi[1], whi[2], whi[3]);
                    ptx::st_shared_v4(sb + OFF_TF + off, wlo[0], wlo[1], wlo[2], wlo[3]);
                }
            }
            ptx::fence_async_smem();
            ptx::named_sync(NB_PAR, kParThreads);
            DC_TC_MARK(5);

            // ---- D_P = Aqk [Tb | Tw] ----
            if (leader) {
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(64, 128, 0, 1);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t a = ptx::sdesc(sb + OFF_AQK + kk * 32, 16, 1024);
                    const uint64_t bd = ptx::sdesc(sb + OFF_AU + kk * 2048, 16384, 1024);
                    ptx::umma_bf16(tmem + TM_A, a, bd, id, kk > 0);
                }
                ptx::umma_commit(&bars[B_MMAP]);
            }
            if (!par_wait(B_MMAP, (uint32_t)(c & 1))) break;
            DC_TC_MARK(6);

            // ---- Pb, Pw (hi + lo): the bottoms of the four A operands (M=64 accumulator: rows in lanes 0-15) ----
            ptx::tc_fence_after();
            {
                const uint32_t dst_hi = sb + (ch ? OFF_AW : OFF_AU), dst_lo = sb + (ch ? OFF_TF : OFF_AF);
                const int i = 16 * sp + lane;
                uint32_t vv[2][32];
                ptx::tmem_ld32(tmem + lane_base + TM_A + 64 * ch, vv[0]);
                ptx::tmem_ld32(tmem + lane_base + TM_A + 64 * ch + 32, vv[1]);
                ptx::tmem_wait_ld();
                if (lane < 16) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float *f = reinterpret_cast<const float *>(vv[hh] + 8 * q);
                            uint32_t hi[4], lo[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                hi[e] = ptx::pack_bf16(f[2 * e], f[2 * e + 1]);
                                lo[e] = ptx::pack_bf16(f[2 * e] - ptx::bf16lo(hi[e]), f[2 * e + 1] - ptx::bf16hi(hi[e]));
                            }
                            const uint32_t off = ptx::sw128(64 + i, 32 * hh + 8 * q);
                            ptx::st_shared_v4(dst_hi + off, hi[0], hi[1], hi[2], hi[3]);
                            ptx::st_shared_v4(dst_lo + off, lo[0], lo[1], lo[2], lo[3]);
                        }
                    }
                }
            }
            ptx::fence_async_smem();
            ptx::tc_fence_before();
            ptx::named_sync(NB_PAR, kParThreads);
            DC_TC_MARK(7);

            // ---- chunk c's MMA4 operands are written and TM_A is free: over to the issue warp ----
            if (leader) ptx::mbar_arrive(&bars[B_OPS]);
        }
    } else if (warp == kIssueWarp) {
        // ================ issue warp: chunk c's D1, then chunk c-1's MMA4 ================
        // D1 goes first so that chunk c's masks do not queue behind MMA4 in the tensor pipe (unless chunk
        // c's tiles are still in flight, in which case MMA4 goes first).  MMA4 waits until the serial role
        // has released chunk c-2's D_UY / D_W.  A wait that runs out sets the flag and ends the warp; the
        // roles then run into their own bounded waits.
        if (lane == 0) {
            auto issue_d1 = [&](int64_t c) {
                const int st = (int)(c & 1);
                const uint32_t stg = sb + OFF_STAGE + st * kStageBytes;
                pend[st] = -1;
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, 64, 0, 0);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t d = ptx::sdesc(stg + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
                    ptx::umma_bf16(tmem + TM_A, d, d, id, kk > 0);
                }
                ptx::umma_commit(&bars[B_MMA1]);
            };
            // MMA4 of chunk c in two parts: D_W = [Tw; Pw] K (commit B_MMA4W), D_UY = [Tb; Pb] V (B_MMA4).
            auto issue_mma4 = [&](int64_t c, bool w_part) {
                const uint32_t stg = sb + OFF_STAGE + (int)(c & 1) * kStageBytes;
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, 128, 0, 1);
                const uint32_t hi = w_part ? OFF_AW : OFF_AU, lo = w_part ? OFF_TF : OFF_AF;
                const uint32_t bop = w_part ? stg : stg + 32768, lbo = w_part ? 16384 : 8192;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    ptx::umma_bf16(tmem + (w_part ? TM_W : TM_UY), ptx::sdesc(sb + (kk < 4 ? hi : lo) + (kk & 3) * 32, 16, 1024),
                                   ptx::sdesc(bop + (kk & 3) * 2048, lbo, 1024), id, kk > 0);
                ptx::umma_commit(&bars[w_part ? B_MMA4W : B_MMA4]);
            };
            bool ok = true;
            for (int64_t c = 0; c <= nchunks && ok; ++c) {
                const int st = (int)(c & 1);
                const uint32_t tpar = (uint32_t)((c >> 1) & 1);
                // chunk c-1's operands are written, and D1's TM_A has been read
                if (c > 0 && !(ok = ptx::mbar_wait(&bars[B_OPS], (uint32_t)((c - 1) & 1)))) break;
                // D1 goes ahead of whichever MMA4 part has not been issued when chunk c's tiles land.
                bool d1 = !(c < nchunks);
                auto try_d1 = [&] {
                    if (!d1 && ptx::mbar_test(&bars[B_TMA0 + st], tpar)) {
                        issue_d1(c);
                        d1 = true;
                    }
                };
                try_d1();
                if (c > 0) {
                    if (c > 1 && !(ok = ptx::mbar_wait(&bars[B_UY_FREE], (uint32_t)((c - 2) & 1)))) break;
                    issue_mma4(c - 1, true);
                    try_d1();
                    issue_mma4(c - 1, false);
                }
                if (!d1) {
                    if (!(ok = ptx::mbar_wait(&bars[B_TMA0 + st], tpar))) break;
                    issue_d1(c);
                }
                // Chunk c+2 loads into chunk c's stage once chunk c's MMA7 is done, more than a chunk from
                // now: pull its tiles into L2 already, so that its load (and D1) does not wait on HBM.
                if (c + 2 < nchunks && !p.stall) prefetch_tiles(c + 2);
            }
            if (!ok) *flag = 1;
        }
        __syncwarp();
    } else {
        // =============================== serial role: the S chain of chunk c ===============================
        const int sp = warp - 8;  // TMEM subpartition
        const int r = 32 * sp + lane;
        const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
        const bool leader = (tid == kParThreads);
        auto ser_wait = [&](int bar, uint32_t parity) {
            const bool bad = !ptx::mbar_wait(&bars[bar], parity) || *flag != 0;
            if (ptx::named_sync_or(NB_SER, kSerThreads, bad)) {
                *flag = 1;
                return false;
            }
            return true;
        };
        float *normw = reinterpret_cast<float *>(base + OFF_NORMW);
        if constexpr (NORM) normw[r] = p.norm_weight[r];  // read only by this role, after the barrier below
        bool ok = ser_wait(B_GATE0, 0);
        if (ok) {
            // S0 -> TMEM (scaled by chunk 0's total decay) and its bf16 copy.
            const float Gam = Gs[64 + 63];
            const float *src = p.state_in + (bh * kD + r) * kD;
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
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
                        ptx::st_shared_v4(sb + OFF_S + hh * 16384 + ptx::sw128(r, 32 * q2 + 8 * q),
                                          ptx::pack_bf16(f[0], f[1]), ptx::pack_bf16(f[2], f[3]),
                                          ptx::pack_bf16(f[4], f[5]), ptx::pack_bf16(f[6], f[7]));
                    }
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * Gam);
                    ptx::tmem_st32(tmem + lane_base + TM_S + 64 * hh + 32 * q2, v);
                }
            }
            ptx::tmem_wait_st();
            ptx::fence_async_smem();
            ptx::tc_fence_before();
            ptx::named_sync(NB_SER, kSerThreads);
        }

        for (int64_t c = 0; c < nchunks && ok; ++c) {
            const int st = (int)(c & 1);
            const uint32_t stg = sb + OFF_STAGE + st * kStageBytes;
            const float *Gc = Gs + (int)(c % kGateSlots) * 128;
            const float *gam = Gc + 64;
            DC_TC_MARK(8);

            // ---- A6 = [-W; s gam Q - Aqk W] into TMEM, over D_W (bf16 pairs, two per column) ----
            if (!(ok = ser_wait(B_MMA4W, (uint32_t)(c & 1)))) break;
            DC_TC_MARK(9);
            ptx::tc_fence_after();
            {
                const int pq = (r >= 64) ? q_pos(c, r - 64, p) : -1;
                const float qs = (pq >= 0) ? scale * gam[pq] : 0.f;
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t vv[2][32];
                    ptx::tmem_ld32(tmem + lane_base + TM_W + 64 * hh, vv[0]);
                    ptx::tmem_ld32(tmem + lane_base + TM_W + 64 * hh + 32, vv[1]);
                    ptx::tmem_wait_ld();
                    uint32_t packed[32];
                    const uint32_t qblk = stg + hh * 16384 + 8192;
#pragma unroll
                    for (int q2 = 0; q2 < 2; ++q2) {
                        const float *f = reinterpret_cast<const float *>(vv[q2]);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float a[8];
                            if (r < 64) {
#pragma unroll
                                for (int e = 0; e < 8; ++e) a[e] = -f[8 * q + e];
                            } else {
                                const uint4 qv = ptx::ld_shared_v4(qblk + ptx::sw128(r - 64, 32 * q2 + 8 * q));
                                const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    a[2 * e] = qs * ptx::bf16lo(qw[e]) - f[8 * q + 2 * e];
                                    a[2 * e + 1] = qs * ptx::bf16hi(qw[e]) - f[8 * q + 2 * e + 1];
                                }
                            }
#pragma unroll
                            for (int e = 0; e < 4; ++e) packed[16 * q2 + 4 * q + e] = ptx::pack_bf16(a[2 * e], a[2 * e + 1]);
                        }
                    }
                    ptx::tmem_st32(tmem + lane_base + TM_W + 32 * hh, packed);
                }
                ptx::tmem_wait_st();
            }
            ptx::tc_fence_before();
            // A6 is in TMEM, and MMA4's D_UY half (accumulated below) is done
            if (!(ok = ser_wait(B_MMA4, (uint32_t)(c & 1)))) break;
            DC_TC_MARK(10);

            // ---- D_UY += A6 S  ->  [V'; y] ----
            if (leader) {
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, 128, 0, 1);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    ptx::umma_bf16_ts(tmem + TM_UY, tmem + TM_W + 8 * kk, ptx::sdesc(sb + OFF_S + kk * 2048, 16384, 1024),
                                      id, 1);
                ptx::umma_commit(&bars[B_MMA6]);
                // The previous chunk's y store has landed: its tile may be rewritten, and rows it wrote
                // past its own readouts (u > 1) are rewritten below in order by their own chunk.
                if (kYTma) ptx::bulk_wait_all();
            }
            if (!(ok = ser_wait(B_MMA6, (uint32_t)(c & 1)))) break;
            DC_TC_MARK(11);

            // ---- V' (decayed to the chunk end, hi + lo) -> the stage's V and Q slots; y -> HBM ----
            ptx::tc_fence_after();
            {
                const float vs = (r < 64 && gated) ? __expf(Gc[63] - Gc[r]) : 1.f;
                const bool write_y = (r >= 64) && q_pos(c, r - 64, p) >= 0;
                const int64_t tok = write_y ? q_first(c, p.u) + (r - 64) : 0;
                TO *yrow = static_cast<TO *>(p.y) + ((b * p.seq + tok) * p.heads + h) * kD;
                // The fused plain output norm (OutNorm::Plain, src/common/norm.rs:129-135): each y-row thread
                // holds its whole row of dv = 128 values, so mean(y^2) is a sum in registers over a first
                // pass; the y warps have the time while the V' warps split their rows into hi + lo.
                float inv = 1.f;
                if (NORM && r >= 64) {  // warp-uniform: warps 10 and 11
                    float ss = 0.f;
#pragma unroll 1
                    for (int hh = 0; hh < 2; ++hh) {
                        uint32_t vv[2][32];
                        ptx::tmem_ld32(tmem + lane_base + TM_UY + 64 * hh, vv[0]);
                        ptx::tmem_ld32(tmem + lane_base + TM_UY + 64 * hh + 32, vv[1]);
                        ptx::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const float a0 = __uint_as_float(vv[0][e]), a1 = __uint_as_float(vv[1][e]);
                            ss = fmaf(a0, a0, fmaf(a1, a1, ss));
                        }
                    }
                    inv = rsqrtf(ss * (1.f / kD) + p.norm_eps);
                }
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t vv[2][32];
                    ptx::tmem_ld32(tmem + lane_base + TM_UY + 64 * hh, vv[0]);
                    ptx::tmem_ld32(tmem + lane_base + TM_UY + 64 * hh + 32, vv[1]);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int q2 = 0; q2 < 2; ++q2) {
                        float *f = reinterpret_cast<float *>(vv[q2]);
                        if (NORM && r >= 64) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) f[e] *= inv * normw[64 * hh + 32 * q2 + e];
                        }
                        if (r < 64) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                uint32_t hi[4], lo[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float x0 = vs * f[8 * q + 2 * e], x1 = vs * f[8 * q + 2 * e + 1];
                                    hi[e] = ptx::pack_bf16(x0, x1);
                                    lo[e] = ptx::pack_bf16(x0 - ptx::bf16lo(hi[e]), x1 - ptx::bf16hi(hi[e]));
                                }
                                const uint32_t off = ptx::sw128(r, 32 * q2 + 8 * q);
                                ptx::st_shared_v4(stg + 32768 + hh * 8192 + off, hi[0], hi[1], hi[2], hi[3]);
                                ptx::st_shared_v4(stg + hh * 16384 + 8192 + off, lo[0], lo[1], lo[2], lo[3]);
                            }
                        } else if (kYTma) {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                ptx::st_shared_v4(sb + OFF_S + hh * 16384 + ptx::sw128(r - 64, 32 * q2 + 8 * q),
                                                  ptx::pack_bf16(f[8 * q], f[8 * q + 1]),
                                                  ptx::pack_bf16(f[8 * q + 2], f[8 * q + 3]),
                                                  ptx::pack_bf16(f[8 * q + 4], f[8 * q + 5]),
                                                  ptx::pack_bf16(f[8 * q + 6], f[8 * q + 7]));
                        } else if (write_y) {
                            store_row32(yrow + 64 * hh + 32 * q2, f);
                        }
                    }
                }
            }
            ptx::fence_async_smem();
            ptx::tc_fence_before();
            ptx::named_sync(NB_SER, kSerThreads);
            if (leader) {
                ptx::mbar_arrive(&bars[B_UY_FREE]);  // D_UY and D_W (A6) may be overwritten now
                if (kYTma) {
                    // The Q tile's 64 token rows; rows past the sequence are clipped by the tensor map.
                    const int tok0 = (int)q_first(c, p.u);
                    ptx::tma_store_4d(&tm_y, sb + OFF_S, 0, (int)h, tok0, (int)b);
                    ptx::tma_store_4d(&tm_y, sb + OFF_S + 16384, 64, (int)h, tok0, (int)b);
                    ptx::bulk_commit();
                }
            }
            DC_TC_MARK(12);

            // ---- D_S = Gam S + K^T (V'hi + V'lo) ----
            if (leader) {
                ptx::tc_fence_after();
                const uint32_t id = ptx::idesc_bf16(128, 128, 1, 1);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t bdesc = (kk < 4) ? ptx::sdesc(stg + 32768 + (kk & 3) * 2048, 8192, 1024)
                                                    : ptx::sdesc(stg + 8192 + (kk & 3) * 2048, 16384, 1024);
                    ptx::umma_bf16(tmem + TM_S, ptx::sdesc(stg + (kk & 3) * 2048, 16384, 1024), bdesc, id, 1);
                }
                ptx::umma_commit(&bars[B_MMA7]);
                if (kYTma) ptx::bulk_wait_read_all();  // the y tiles have left the S buffer the tail rewrites
            }
            if (!(ok = ser_wait(B_MMA7, (uint32_t)(c & 1)))) break;
            DC_TC_MARK(13);
            if (leader && c + 2 < nchunks) issue_tma(c + 2, st);  // the stage is fully consumed

            // ---- S -> bf16 operand and the accumulator pre-scaled by the next chunk's decay ----
            if (c + 1 < nchunks) {
                const int gnx = (int)((c + 1) % kGateSlots);
                if (!(ok = ser_wait(B_GATE0 + gnx, (uint32_t)(((c + 1) / kGateSlots) & 1)))) break;
                const float Gam = Gs[gnx * 128 + 64 + 63];
                ptx::tc_fence_after();
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t vv[2][32];
                    ptx::tmem_ld32(tmem + lane_base + TM_S + 64 * hh, vv[0]);
                    ptx::tmem_ld32(tmem + lane_base + TM_S + 64 * hh + 32, vv[1]);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int q2 = 0; q2 < 2; ++q2) {
                        uint32_t(&v)[32] = vv[q2];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float *f = reinterpret_cast<const float *>(v + 8 * q);
                            ptx::st_shared_v4(sb + OFF_S + hh * 16384 + ptx::sw128(r, 32 * q2 + 8 * q),
                                              ptx::pack_bf16(f[0], f[1]), ptx::pack_bf16(f[2], f[3]),
                                              ptx::pack_bf16(f[4], f[5]), ptx::pack_bf16(f[6], f[7]));
                        }
                        if (gated) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * Gam);
                            ptx::tmem_st32(tmem + lane_base + TM_S + 64 * hh + 32 * q2, v);
                        }
                    }
                }
                ptx::tmem_wait_st();
                ptx::fence_async_smem();
                ptx::tc_fence_before();
                ptx::named_sync(NB_SER, kSerThreads);
            } else {
                ptx::tc_fence_after();
                float *dst = p.state_out + (bh * kD + r) * kD;
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t vv[2][32];
                    ptx::tmem_ld32(tmem + lane_base + TM_S + 64 * hh, vv[0]);
                    ptx::tmem_ld32(tmem + lane_base + TM_S + 64 * hh + 32, vv[1]);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int q2 = 0; q2 < 2; ++q2)
                        store_row32(dst + 64 * hh + 32 * q2, reinterpret_cast<const float *>(vv[q2]));
                }
            }
        }
    }

    if (kYTma && tid == kParThreads) ptx::bulk_wait_all();  // the staged y tile is read before smem goes away

    // Both roles meet here exactly once.
    ptx::tc_fence_before();
    __syncthreads();
    if (*flag) {
        // A wait ran out: report it and let this CTA's own TMA loads land before the smem goes away.
        if (tid == 0) {
            atomicExch(status, kStatusTimeout);
            for (int s = 0; s < 2; ++s)
                if (pend[s] >= 0) ptx::mbar_wait(&bars[B_TMA0 + s], (uint32_t)pend[s]);
        }
        __syncthreads();
    }
    if (warp == 0) ptx::tmem_dealloc(tmem, 512);
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Whether the tensor-core kernel serves this request.
inline bool tc_applies(const CoreParams &p, int32_t in_dtype, uint32_t flags) {
    if (flags & 0x3u) return false;  // DC_FLAG_FORCE_SIMT, DC_FLAG_RECURRENT
    if (in_dtype != 1) return false; // bf16 q, k, v
    if (p.dk != 128 || p.dv != 128) return false;
    if (p.ew != 1 || p.ww != 1 || p.gw > 1) return false;
    if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) || !aligned16(p.y) || !aligned16(p.state_in) ||
        !aligned16(p.state_out))
        return false;
    if (p.seq * p.u > 0x7fffffff || p.batch * p.heads > 0x7fffffff) return false;
    return true;
}

inline thread_local int g_tc_error = 0;
inline int tc_last_error() { return g_tc_error; }

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// [batch, rows, heads, 128] bf16 viewed as a 4-D tensor (128, heads, rows, batch),
// read in 64 x 1 x 64 x 1 boxes (64 rows of 128 bytes, 128-byte swizzle).
inline bool encode_rows(CUtensorMap *m, const void *ptr, int64_t heads, int64_t rows, int64_t batch) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[4] = {128, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
    const cuuint64_t strides[3] = {256, (cuuint64_t)(256 * heads), (cuuint64_t)(256 * heads * rows)};
    const cuuint32_t box[4] = {64, 1, 64, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The current thread's CUDA context (the driver's cuCtxGetCurrent), or null.  A device address looked up
// once is valid for the context it was looked up in: after cudaDeviceReset the device gets a new primary
// context, and an address cached under the old one would name memory the library no longer owns.
inline void *current_context() {
    using Fn = CUresult (*)(CUcontext *);
    static Fn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(ptr);
    }
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

// The device address of a __device__ symbol in the current device's current context, looked up with that
// device current and cached per (device, context); null when the lookup fails.
struct SymbolCache {
    std::mutex mu;
    void *ctx[64] = {};
    void *addr[64] = {};
    void *get(const void *symbol, int *err) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess || dev < 0 || dev >= 64) {
            *err = (int)(e != cudaSuccess ? e : cudaErrorInvalidDevice);
            return nullptr;
        }
        std::lock_guard<std::mutex> lock(mu);
        void *c = current_context();  // null before the runtime first touched the device
        if (c && addr[dev] && ctx[dev] == c) return addr[dev];
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, symbol);  // (creates the device's primary context if needed)
        if (e != cudaSuccess || !p) {
            *err = (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
            return nullptr;
        }
        ctx[dev] = current_context();
        addr[dev] = p;
        return p;
    }
};

inline int *device_status_ptr() {
    static SymbolCache cache;
    int err = 0;
    return static_cast<int *>(cache.get(reinterpret_cast<const void *>(&g_device_status), &err));
}

template <typename TG, typename TO, bool NORM>
int launch_tc_typed(const CoreParams &p, cudaStream_t stream) {
    CUtensorMap mk, mq, mv, my;
    const int64_t P = p.seq * p.u;
    if (!encode_rows(&mk, p.k, p.heads, P, p.batch) || !encode_rows(&mq, p.q, p.heads, p.seq, p.batch) ||
        !encode_rows(&mv, p.v, p.heads, P, p.batch) ||
        (sizeof(TO) == 2 ? !encode_rows(&my, p.y, p.heads, p.seq, p.batch) : (my = mq, false))) {
        g_tc_error = (int)cudaErrorInvalidValue;
        return 6;  // DC_ECUDA
    }
    int *status = device_status_ptr();
    if (!status) {
        g_tc_error = (int)cudaErrorInvalidSymbol;
        return 6;
    }
    auto kern = tc::chunk_tc_kernel<TG, TO, NORM>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes);
    if (e == cudaSuccess) {
        kern<<<(unsigned)(p.batch * p.heads), tc::kThreads, tc::kSmemBytes, stream>>>(mk, mq, mv, my, p, status);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        g_tc_error = (int)e;
        return 6;
    }
    return 0;
}

inline int launch_chunk_tc(const CoreParams &p, int32_t gate_dtype, int32_t out_dtype, cudaStream_t stream) {
    const int key = (p.norm ? 4 : 0) + gate_dtype * 2 + out_dtype;
    switch (key) {
        case 0: return launch_tc_typed<float, float, false>(p, stream);
        case 1: return launch_tc_typed<float, __nv_bfloat16, false>(p, stream);
        case 2: return launch_tc_typed<__nv_bfloat16, float, false>(p, stream);
        case 3: return launch_tc_typed<__nv_bfloat16, __nv_bfloat16, false>(p, stream);
        case 4: return launch_tc_typed<float, float, true>(p, stream);
        case 5: return launch_tc_typed<float, __nv_bfloat16, true>(p, stream);
        case 6: return launch_tc_typed<__nv_bfloat16, float, true>(p, stream);
        case 7: return launch_tc_typed<__nv_bfloat16, __nv_bfloat16, true>(p, stream);
    }
    return 3;  // DC_EUNSUPPORTED_DTYPE
}

}  // namespace dc
