// prologue.cuh — the front-end between the fused input projection and the delta-rule core, on the
// [q | u k | u v] channel segment of the projection (src/common/qkv.rs:373-440 forward, 447-500 step):
//
//   * the causal depthwise short convolution over the channels with its rolling window
//     (src/common/conv.rs:81-118, 124-160): x left-padded with the window's newest K - 1 columns,
//     y[c, t] = bias[c] + sum_j w[c, j] x_pad[c, t + j], the next window the padded input's last K
//     columns; then the convolution's SiLU (or none);
//   * the split into q [B, S, H, dk], k [B, S u, H, dk], v [B, S u, H, dv] (micro-step m of token t is
//     row t u + m: a reshape);
//   * without the convolution's SiLU: q, k through SiLU or identity, v through SiLU (qkv.rs:405-413);
//   * q, k over the head axis: x / sqrt(sum x^2 + 1e-6) (src/common/norm.rs:83-90), or none.
//
// One CTA (128 threads, one per channel of a head segment) per (segment, 32-token tile, batch), the
// segments being the H q heads, the u H k heads and the u H v heads.  The tile's inputs (32 + K - 1
// tokens; the window supplies the ones before the sequence) are staged in shared memory by 16-byte
// asynchronous copies, each thread slides its channel's K taps down them, and the q / k norms reduce
// over the segment (a warp-level transpose reduction, then the four warps).  HBM-bound: each input read
// once (plus the K - 1 halo rows), each output written once.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace dc {
namespace pro {

constexpr int kThreads = 128;  // channels of one head segment (dk, dv <= 128)
constexpr int kTile = 32;      // tokens per CTA (one warp's width: the transpose reduction)
constexpr int kMaxK = 8;       // short-convolution width

struct Params {
    int64_t batch, seq, heads, dk, dv, channels, x_stride;
    int32_t u, K, conv_silu, qk_silu, l2;
    int32_t vec_rows;          // x rows 16-byte aligned (x and x_stride): tiles staged by cp.async
    const void *x;             // [B, S, x_stride]: channel c of token t at (b S + t) x_stride + c
    const float *weight;       // [channels, K]
    const float *bias;         // [channels] or null
    const float *window_in;    // [B, channels, K] or null (zeros)
    float *window_out;         // [B, channels, K] or null
    void *q, *k, *v;
};

// x sigma(x) with the fast exponential and division intrinsics (a few ulp; x -> -inf gives 0)
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// KT: the taps compiled in (4, the reference's width, or kMaxK with the unused taps zero)
template <typename TI, typename TO, int KT>
__global__ void __launch_bounds__(kThreads) prologue_kernel(const Params p) {
    constexpr int kRows = kTile + KT - 1;           // the tile's inputs: tokens t0 - K + 1 .. t0 + kTile - 1
    __shared__ __align__(16) TI tile[kRows][kThreads];
    __shared__ float head[KT][kThreads];  // rows before the sequence (the window, float32)
    __shared__ float red[kThreads / 32][kTile];
    __shared__ float inv[kTile];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t seg = blockIdx.x, b = blockIdx.z, t0 = (int64_t)blockIdx.y * kTile;
    const int64_t H = p.heads, kd = H * p.dk;
    // this segment: its output tensor, head, micro-step, width and first channel
    int kind, width;  // 0 q, 1 k, 2 v
    int64_t h, m, base;
    if (seg < H) {
        kind = 0, width = (int)p.dk, h = seg, m = 0, base = seg * p.dk;
    } else if (seg < H + p.u * H) {
        const int64_t s = seg - H;
        kind = 1, width = (int)p.dk, m = s / H, h = s - m * H, base = kd + m * kd + h * p.dk;
    } else {
        const int64_t s = seg - H - p.u * H;
        kind = 2, width = (int)p.dv, m = s / H, h = s - m * H, base = kd * (1 + p.u) + m * H * p.dv + h * p.dv;
    }
    const int K = p.K;
    const TI *X = static_cast<const TI *>(p.x);
    const int64_t tfirst = t0 - (KT - 1);  // token of tile row 0 (rows before KT - K hold zero taps)

    // ---- stage the inputs: 16-byte copies of the in-sequence rows (or scalar loads when the rows are not
    // 16-byte aligned), the window's float32 values for the rows before the sequence, zeros after it ----
    constexpr int kVec = 16 / sizeof(TI);
    const bool vec = p.vec_rows && (base % kVec) == 0 && (width % kVec) == 0;
    const int r_lo = tfirst < 0 ? (int)(-tfirst) : 0;                                   // rows before the sequence
    const int r_hi = p.seq - tfirst < kRows ? (int)(p.seq - tfirst) : kRows;            // rows from r_hi: past it
    const TI *xrow = X + (b * p.seq + tfirst) * p.x_stride + base;                       // row r at r * x_stride
    if (vec) {
        const int per_row = width / kVec, rstep = kThreads / per_row;
        const int q = tid % per_row;
        for (int r = r_lo + tid / per_row; r < r_hi; r += rstep)
            ptx::cp_async16(ptx::smem_u32(&tile[r][q * kVec]), xrow + r * p.x_stride + q * kVec, 16u);
        ptx::cp_async_commit();
    } else if (tid < width) {
        for (int r = r_lo; r < r_hi; ++r) tile[r][tid] = xrow[r * p.x_stride + tid];
    }
    if (tid < width) {
        const float *win = p.window_in ? p.window_in + (b * p.channels + base + tid) * K : nullptr;
        for (int r = 0; r < r_lo; ++r) {  // token tfirst + r < 0: window column K + t (zero before it)
            const int64_t t = tfirst + r;
            if (r < KT) head[r][tid] = (t >= -(int64_t)(K - 1) && win) ? win[K + t] : 0.f;
        }
        for (int r = r_hi; r < kRows; ++r) st(&tile[r][tid], 0.f);
    }
    if (vec) ptx::cp_async_wait<0>();
    __syncthreads();

    // ---- convolve (taps j < K; the first KT - K rows are never read), activation ----
    const bool on = tid < width;
    const int cch = on ? tid : 0;
    const int64_t c = base + cch;
    // taps shifted to the tile rows they read: ws[j] = w[j - (KT - K)] (zero below)
    float ws[KT];
#pragma unroll
    for (int j = 0; j < KT; ++j) ws[j] = j >= KT - K ? p.weight[c * K + j - (KT - K)] : 0.f;
    const float bias = p.bias ? p.bias[c] : 0.f;
    const bool act = p.conv_silu || kind == 2 || p.qk_silu;  // the conv's SiLU, or v's, or q / k's
    // output token t0 + i reads tokens t0 + i - K + 1 + j (j < K): tile rows i + (KT - K) + j; the rows
    // before the sequence come from `head` (they only enter the first KT - 1 history values)
    float hist[KT];
#pragma unroll
    for (int j = 0; j < KT - 1; ++j) hist[j + 1] = tfirst + j < 0 ? head[j][cch] : ld(&tile[j][cch]);
    float y[kTile];
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
#pragma unroll
        for (int j = 0; j < KT - 1; ++j) hist[j] = hist[j + 1];
        hist[KT - 1] = ld(&tile[i + KT - 1][cch]);
        float a = bias;
#pragma unroll
        for (int j = 0; j < KT; ++j) a = fmaf(ws[j], hist[j], a);
        if (act) a = silu(a);
        y[i] = on ? a : 0.f;
    }
    if (p.l2 && kind < 2) {
        // sum over the segment of y^2 per token: a transpose reduction leaves token `lane`'s warp sum in
        // s[0] (31 shuffles for 32 tokens), then the warps add up
        float s[kTile];
#pragma unroll
        for (int i = 0; i < kTile; ++i) s[i] = y[i] * y[i];
#pragma unroll
        for (int wd = kTile / 2; wd >= 1; wd >>= 1) {
            const bool upper = (lane & wd) != 0;
#pragma unroll
            for (int i = 0; i < wd; ++i) {
                const float send = upper ? s[i] : s[i + wd];
                const float keep = upper ? s[i + wd] : s[i];
                s[i] = keep + __shfl_xor_sync(0xffffffffu, send, wd);
            }
        }
        red[warp][lane] = s[0];
        __syncthreads();
        if (tid < kTile) {
            float tot = 0.f;
#pragma unroll
            for (int q = 0; q < kThreads / 32; ++q) tot += red[q][tid];
            inv[tid] = rsqrtf(tot + 1e-6f);
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kTile; ++i) y[i] *= inv[i];
    }
    // ---- outputs: row (b, t) of q, row (b, t u + m) of k / v ----
    TO *out = static_cast<TO *>(kind == 0 ? p.q : kind == 1 ? p.k : p.v);
    const int64_t rows_per_b = kind == 0 ? p.seq : p.seq * p.u, step = kind == 0 ? 1 : p.u;
    const int64_t pitch = step * H * width;  // elements between consecutive tokens' rows
    const int n = p.seq - t0 < kTile ? (int)(p.seq - t0) : kTile;
    if (on) {
        TO *o = out + ((b * rows_per_b + t0 * step + m) * H + h) * width + tid;
#pragma unroll
        for (int i = 0; i < kTile; ++i, o += pitch)
            if (i < n) st(o, y[i]);
    }
    // ---- the next window: the padded input's last K columns, from the CTA holding the last token ----
    if (p.window_out && on && t0 <= p.seq - 1 && p.seq - 1 < t0 + kTile) {
        float *wo = p.window_out + (b * p.channels + c) * K;
        for (int j = 0; j < K; ++j) {
            const int r = (int)(p.seq - K + j - tfirst);
            wo[j] = p.seq - K + j < 0 ? head[r][cch] : ld(&tile[r][cch]);
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// The same computation two channels per thread (even dk and dv): a CTA of 128 threads serves two head
// segments, 64 threads each, so shared-memory reads and output stores move channel pairs (bf16x2 or
// float2) and each thread's share of the norm's reduction halves.  Both halves reach every barrier (the
// second half of the last CTA may have no segment, and a q / k half may sit beside a v half).
// ---------------------------------------------------------------------------------------------------
constexpr int kHalf = kThreads / 2;  // threads per segment

__device__ __forceinline__ float2 to_f2(float2 v) { return v; }
__device__ __forceinline__ float2 to_f2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
__device__ __forceinline__ void st2(float *o, float a, float b) { *reinterpret_cast<float2 *>(o) = make_float2(a, b); }
__device__ __forceinline__ void st2(__nv_bfloat16 *o, float a, float b) {
    *reinterpret_cast<__nv_bfloat162 *>(o) = __floats2bfloat162_rn(a, b);
}
template <typename T> struct PairOf;
template <> struct PairOf<float> { using type = float2; };
template <> struct PairOf<__nv_bfloat16> { using type = __nv_bfloat162; };

template <typename TI, typename TO, int KT>
__global__ void __launch_bounds__(kThreads) prologue_pair_kernel(const Params p) {
    using TI2 = typename PairOf<TI>::type;
    constexpr int kRows = kTile + KT - 1;
    __shared__ __align__(16) TI tile[2][kRows][kThreads];
    __shared__ float2 head[2][KT][kHalf];  // rows before the sequence (the window, float32)
    __shared__ float red[kThreads / 32][kTile];
    __shared__ float inv[2][kTile];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, half = tid / kHalf, lt = tid % kHalf;
    const int64_t H = p.heads, kd = H * p.dk, nseg = H * (1 + 2 * (int64_t)p.u);
    const int64_t seg = 2 * (int64_t)blockIdx.x + half, b = blockIdx.z, t0 = (int64_t)blockIdx.y * kTile;
    const bool live = seg < nseg;
    int kind, width;  // 0 q, 1 k, 2 v
    int64_t h, m, base;
    if (seg < H) {
        kind = 0, width = (int)p.dk, h = seg, m = 0, base = seg * p.dk;
    } else if (seg < H + p.u * H) {
        const int64_t sq = seg - H;
        kind = 1, width = (int)p.dk, m = sq / H, h = sq - m * H, base = kd + m * kd + h * p.dk;
    } else {
        const int64_t sq = live ? seg - H - p.u * H : 0;
        kind = 2, width = live ? (int)p.dv : 0, m = sq / H, h = sq - m * H,
        base = kd * (1 + p.u) + m * H * p.dv + h * p.dv;
    }
    const int K = p.K;
    const TI *X = static_cast<const TI *>(p.x);
    const int64_t tfirst = t0 - (KT - 1);
    TI(*tl)[kThreads] = tile[half];

    // ---- stage this half's segment ----
    constexpr int kVec = 16 / sizeof(TI);
    const bool vec = p.vec_rows && (base % kVec) == 0 && (width % kVec) == 0;
    const int r_lo = tfirst < 0 ? (int)(-tfirst) : 0;
    const int r_hi = p.seq - tfirst < kRows ? (int)(p.seq - tfirst) : kRows;
    const TI *xrow = X + (b * p.seq + tfirst) * p.x_stride + base;
    const bool on = 2 * lt < width;  // this thread's channel pair 2 lt, 2 lt + 1
    if (live && vec) {
        const int per_row = width / kVec, rstep = kHalf / per_row;
        const int q = lt % per_row;
        for (int r = r_lo + lt / per_row; r < r_hi; r += rstep)
            ptx::cp_async16(ptx::smem_u32(&tl[r][q * kVec]), xrow + r * p.x_stride + q * kVec, 16u);
    } else if (live && on) {
        for (int r = r_lo; r < r_hi; ++r) {
            tl[r][2 * lt] = xrow[r * p.x_stride + 2 * lt];
            tl[r][2 * lt + 1] = xrow[r * p.x_stride + 2 * lt + 1];
        }
    }
    ptx::cp_async_commit();
    if (live && on) {
        const float *win = p.window_in ? p.window_in + (b * p.channels + base + 2 * lt) * K : nullptr;
        for (int r = 0; r < r_lo; ++r) {  // token tfirst + r < 0: window column K + t (zero before it)
            const int64_t t = tfirst + r;
            const bool w_ok = t >= -(int64_t)(K - 1) && win;
            if (r < KT) head[half][r][lt] = w_ok ? make_float2(win[K + t], win[K + K + t]) : make_float2(0.f, 0.f);
        }
        for (int r = r_hi; r < kRows; ++r) {
            st(&tl[r][2 * lt], 0.f);
            st(&tl[r][2 * lt + 1], 0.f);
        }
    }
    ptx::cp_async_wait<0>();
    __syncthreads();

    // ---- convolve both channels, activation ----
    const int cch = on ? 2 * lt : 0;
    const int64_t c = base + cch;
    float w0[KT], w1[KT];
#pragma unroll
    for (int j = 0; j < KT; ++j) {
        w0[j] = (live && j >= KT - K) ? p.weight[c * K + j - (KT - K)] : 0.f;
        w1[j] = (live && j >= KT - K) ? p.weight[(c + 1) * K + j - (KT - K)] : 0.f;
    }
    const float b0 = (live && p.bias) ? p.bias[c] : 0.f, b1 = (live && p.bias) ? p.bias[c + 1] : 0.f;
    const bool act = p.conv_silu || kind == 2 || p.qk_silu;
    float2 hist[KT];
#pragma unroll
    for (int j = 0; j < KT - 1; ++j)
        hist[j + 1] = tfirst + j < 0 ? head[half][j][lt] : to_f2(*reinterpret_cast<const TI2 *>(&tl[j][cch]));
    float y0[kTile], y1[kTile];
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
#pragma unroll
        for (int j = 0; j < KT - 1; ++j) hist[j] = hist[j + 1];
        hist[KT - 1] = to_f2(*reinterpret_cast<const TI2 *>(&tl[i + KT - 1][cch]));
        float a0 = b0, a1 = b1;
#pragma unroll
        for (int j = 0; j < KT; ++j) {
            a0 = fmaf(w0[j], hist[j].x, a0);
            a1 = fmaf(w1[j], hist[j].y, a1);
        }
        if (act) a0 = silu(a0), a1 = silu(a1);
        y0[i] = (live && on) ? a0 : 0.f;
        y1[i] = (live && on) ? a1 : 0.f;
    }
    if (p.l2) {  // uniform over the CTA: every thread reaches the barriers, q / k halves apply the result
        float sm[kTile];
#pragma unroll
        for (int i = 0; i < kTile; ++i) sm[i] = fmaf(y0[i], y0[i], y1[i] * y1[i]);
#pragma unroll
        for (int wd = kTile / 2; wd >= 1; wd >>= 1) {
            const bool upper = (lane & wd) != 0;
#pragma unroll
            for (int i = 0; i < wd; ++i) {
                const float send = upper ? sm[i] : sm[i + wd];
                const float keep = upper ? sm[i + wd] : sm[i];
                sm[i] = keep + __shfl_xor_sync(0xffffffffu, send, wd);
            }
        }
        red[warp][lane] = sm[0];
        __syncthreads();
        if (tid < 2 * kTile) {
            const int hf = tid / kTile, i = tid % kTile;
            inv[hf][i] = rsqrtf(red[2 * hf][i] + red[2 * hf + 1][i] + 1e-6f);
        }
        __syncthreads();
        if (kind < 2) {
#pragma unroll
            for (int i = 0; i < kTile; ++i) y0[i] *= inv[half][i], y1[i] *= inv[half][i];
        }
    }
    // ---- outputs ----
    if (live && on) {
        TO *out = static_cast<TO *>(kind == 0 ? p.q : kind == 1 ? p.k : p.v);
        const int64_t rows_per_b = kind == 0 ? p.seq : p.seq * p.u, step = kind == 0 ? 1 : p.u;
        const int64_t pitch = step * H * width;
        const int n = p.seq - t0 < kTile ? (int)(p.seq - t0) : kTile;
        TO *o = out + ((b * rows_per_b + t0 * step + m) * H + h) * width + 2 * lt;
#pragma unroll
        for (int i = 0; i < kTile; ++i, o += pitch)
            if (i < n) st2(o, y0[i], y1[i]);
        if (p.window_out && t0 <= p.seq - 1 && p.seq - 1 < t0 + kTile) {
            float *wo = p.window_out + (b * p.channels + c) * K;
            for (int j = 0; j < K; ++j) {
                const int r = (int)(p.seq - K + j - tfirst);
                float2 v;
                if (p.seq - K + j < 0) v = head[half][r][lt];
                else v = to_f2(*reinterpret_cast<const TI2 *>(&tl[r][cch]));
                wo[j] = v.x;
                wo[K + j] = v.y;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// The front-end's gate producers, one elementwise map over a [rows, cols] column slice of the projection
// (row stride x_stride) into a contiguous float32 [rows, cols]:
//   kind 0  scale sigma(x)                                          the write gates (qkv.rs:333-368)
//   kind 1  -e^{a[c]} clamp(softplus(x + bias[c]), lo, hi)          ForgetGate::log_decay (gate.rs:51-59)
//   kind 2  scale sigma((x + bias[c]) e^{a[c / group]})             ChannelForgetGate::log_decay
//                                                                  (gate.rs:178-196), scale = lower bound
// softplus(x) = max(x, 0) + log1p(e^-|x|) at full precision; the sigmoids use the fast exponential and
// division intrinsics (a few ulp).
// ---------------------------------------------------------------------------------------------------
struct GateParams {
    int64_t rows, cols, x_stride;
    int32_t kind, group;
    float scale, lo, hi;
    const void *x;
    const float *bias, *a_log;
    float *out;
};

// sigma(z) * scale with the fast exponential and division intrinsics (a few ulp; z -> -inf gives 0)
__device__ __forceinline__ float scaled_sigmoid(float scale, float z) { return __fdividef(scale, 1.f + __expf(-z)); }

// kind 0 / 1 at column c; kind 2 with the column's per-head slope e^{a[c / group]} given
__device__ __forceinline__ float gate_map(const GateParams &p, float x, int c, float slope) {
    if (p.kind == 0) return scaled_sigmoid(p.scale, x);
    if (p.kind == 1) {
        const float z = x + p.bias[c];
        const float sp = fmaxf(z, 0.f) + log1pf(expf(-fabsf(z)));
        return -expf(p.a_log[c]) * fminf(fmaxf(sp, p.lo), p.hi);
    }
    return scaled_sigmoid(p.scale, (x + p.bias[c]) * slope);
}
__device__ __forceinline__ float gate_slope(const GateParams &p, int c) {
    return p.kind == 2 ? expf(p.a_log[c / p.group]) : 0.f;
}

// One CTA per row at a time (rows blockIdx.x, + gridDim.x, ...), its threads along the columns: four
// consecutive columns per thread (8- or 16-byte loads, 16-byte stores) when `vec4`, else one.
template <typename TI>
__global__ void __launch_bounds__(256) gates_kernel(const GateParams p, int vec4) {
    const TI *X = static_cast<const TI *>(p.x);
    const int cols = (int)p.cols;
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const TI *xr = X + r * p.x_stride;
        float *o = p.out + r * p.cols;
        if (vec4) {
            for (int c = 4 * threadIdx.x; c < cols; c += 4 * blockDim.x) {
                float x4[4];
                if constexpr (sizeof(TI) == 2) {
                    const uint2 t = *reinterpret_cast<const uint2 *>(xr + c);
                    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.x));
                    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.y));
                    x4[0] = lo.x, x4[1] = lo.y, x4[2] = hi.x, x4[3] = hi.y;
                } else {
                    const float4 t = *reinterpret_cast<const float4 *>(xr + c);
                    x4[0] = t.x, x4[1] = t.y, x4[2] = t.z, x4[3] = t.w;
                }
                // the four columns share a head when the group is a multiple of 4 (one slope)
                const bool one = p.group % 4 == 0;
                const float s0 = gate_slope(p, c);
                const float s1 = one ? s0 : gate_slope(p, c + 1), s2 = one ? s0 : gate_slope(p, c + 2),
                            s3 = one ? s0 : gate_slope(p, c + 3);
                *reinterpret_cast<float4 *>(o + c) = make_float4(gate_map(p, x4[0], c, s0), gate_map(p, x4[1], c + 1, s1),
                                                                 gate_map(p, x4[2], c + 2, s2), gate_map(p, x4[3], c + 3, s3));
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += blockDim.x) o[c] = gate_map(p, ld(xr + c), c, gate_slope(p, c));
        }
    }
}

}  // namespace pro
}  // namespace dc
