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
// segments being the H q heads, the u H k heads and the u H v heads.  Each thread loads its channel's
// 32 + K - 1 inputs at once (the window supplies the ones before the sequence), convolves, and the
// q / k norms reduce over the segment (a warp-level transpose reduction, then the four warps).  HBM-bound:
// each input read once, each output written once.
#pragma once

#include "common.cuh"

namespace dc {
namespace pro {

constexpr int kThreads = 128;  // channels of one head segment (dk, dv <= 128)
constexpr int kTile = 32;      // tokens per CTA (one warp's width: the transpose reduction)
constexpr int kMaxK = 8;       // short-convolution width

struct Params {
    int64_t batch, seq, heads, dk, dv, channels, x_stride;
    int32_t u, K, conv_silu, qk_silu, l2;
    const void *x;             // [B, S, x_stride]: channel c of token t at (b S + t) x_stride + c
    const float *weight;       // [channels, K]
    const float *bias;         // [channels] or null
    const float *window_in;    // [B, channels, K] or null (zeros)
    float *window_out;         // [B, channels, K] or null
    void *q, *k, *v;
};

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads) prologue_kernel(const Params p) {
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
    const bool on = tid < width;
    const int64_t c = base + (on ? tid : 0);
    const int K = p.K;
    const TI *X = static_cast<const TI *>(p.x);

    // inputs of tokens t0 - K + 1 .. t0 + kTile - 1 (the window before the sequence, zero past its end),
    // every load issued before the first use
    constexpr int kHalo = kTile + kMaxK - 1;
    float xs[kHalo];
    const float *win = p.window_in ? p.window_in + (b * p.channels + c) * K : nullptr;
#pragma unroll
    for (int i = 0; i < kHalo; ++i) {
        const int64_t t = t0 - K + 1 + i;
        const bool in_seq = i < kTile + K - 1 && t >= 0 && t < p.seq;
        const bool in_win = i < kTile + K - 1 && t < 0 && win != nullptr;
        const float xv = ld(X + (in_seq ? (b * p.seq + t) * p.x_stride + c : 0));
        const float wv = in_win ? win[K + t] : 0.f;
        xs[i] = in_seq ? xv : wv;
    }
    float w[kMaxK];
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) w[j] = j < K ? p.weight[c * K + j] : 0.f;
    const float bias = p.bias ? p.bias[c] : 0.f;
    // output token t0 + i reads the inputs of tokens t0 + i - K + 1 + j (j < K), i.e. xs[i + j]; the taps
    // j >= K have w = 0 and read zeros inside xs
    const bool act = p.conv_silu || kind == 2 || p.qk_silu;  // the conv's SiLU, or v's, or q / k's
    float y[kTile];
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        float a = bias;
#pragma unroll
        for (int j = 0; j < kMaxK; ++j) a = fmaf(w[j], xs[i + j], a);
        if (act) a = silu(a);
        y[i] = on ? a : 0.f;
    }
    const bool norm = p.l2 && kind < 2;
    if (norm) {
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
    // outputs: row (b, t) of q, row (b, t u + m) of k / v
    TO *out = static_cast<TO *>(kind == 0 ? p.q : kind == 1 ? p.k : p.v);
    const int64_t rows_per_b = kind == 0 ? p.seq : p.seq * p.u, step = kind == 0 ? 1 : p.u;
    if (on) {
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
            const int64_t t = t0 + i;
            if (t < p.seq) st(out + ((b * rows_per_b + t * step + m) * H + h) * width + tid, y[i]);
        }
    }
    // the next window: the padded input's last K columns, from the CTA holding the last token
    if (p.window_out && on && t0 <= p.seq - 1 && p.seq - 1 < t0 + kTile) {
        float *wo = p.window_out + (b * p.channels + c) * K;
        for (int j = 0; j < K; ++j) {
            const int64_t t = p.seq - K + j;  // token of padded column S - 1 + j
            wo[j] = t >= 0 ? ld(X + (b * p.seq + t) * p.x_stride + c) : (win ? win[K + t] : 0.f);
        }
    }
}

}  // namespace pro
}  // namespace dc
