// chunk_simt.cuh — chunkwise WY prefill on CUDA cores, fp32 throughout.
//
// The exact-arithmetic path of dc_chunk_fwd: it serves float32 inputs (the
// reference's own precision, held to 1e-4 relative) and every shape the
// tensor-core kernel does not take (dk != 128, dv != 128, tiny test shapes).
// It evaluates the reference's chunk algorithm (src/delta/chunk.rs:41-221)
// chunk by chunk with the state tile resident in shared memory:
//
//   per chunk of LC folded steps (zero-padded past the end, chunk.rs:16-24):
//     G      = cumsum(g) within the chunk                       (chunk.rs:101)
//     Akk_ij = sum_d (b k)_id k_jd e^{G_id - G_jd},  j < i      (chunk.rs:109-137)
//     Aqk_ij = sum_d (s q)_id k_jd e^{G_id - G_jd},  j <= i
//     T      = (I + Akk)^-1   by forward substitution, one warp lane per column
//     U      = T (w v),   W = T ((b k) e^G)                     (chunk.rs:144-153)
//     V'     = U - W S                                          (chunk.rs:179)
//     y      = (q e^G) S + Aqk V'                               (chunk.rs:182-187)
//     S      = e^{G_last} S + (k e^{G_last - G})^T V'           (chunk.rs:191-202)
//
// The per-channel decay is evaluated term by term as e^{G_id - G_jd} with
// j <= i, whose exponent is never positive, so no gate magnitude can overflow
// it (the reference's 16-row reference-point split clamps instead,
// src/delta/decay.rs:41-49).  The micro-step fold runs in the loader: folded
// step p is micro-step p % u of token p / u; q is read on the last micro-step
// and g on the first (src/delta_product/delta_product.rs:178-205).
//
// Grid: x = batch * heads, y = column tiles of CW value columns.  Each CTA
// recomputes the chunk-local matrices for its tile; the state tile [dk x CW]
// never leaves shared memory between chunks.
#pragma once

#include "common.cuh"

namespace dc {

constexpr int kSimtThreads = 256;

// Shared-memory layout of the CUDA-core chunk kernel, in floats.
struct SimtLayout {
    int dk, cw, lc, ks, gs;
    int off_S, off_K, off_Q, off_KE, off_W, off_G, off_V, off_U, off_A, off_Aq, off_T, off_dec, off_row;
    int total;
    __host__ __device__ SimtLayout(int dk_, int cw_, int lc_, int gw) : dk(dk_), cw(cw_), lc(lc_) {
        ks = dk + 1;                      // padded row stride of the [lc][dk] arrays
        gs = (gw > 1) ? ks : 1;
        int o = 0;
        off_S = o;  o += dk * cw;         // state tile
        off_K = o;  o += lc * ks;         // k (later k e^{G_last - G})
        off_Q = o;  o += lc * ks;         // scale q on output rows (later q e^G)
        off_KE = o; o += lc * ks;         // erase k (later erase k e^G)
        off_W = o;  o += lc * ks;         // W
        off_G = o;  o += lc * gs;         // cumulative gate
        off_V = o;  o += lc * cw;         // write v, then V'
        off_U = o;  o += lc * cw;         // U
        off_A = o;  o += lc * (lc + 1);   // Akk
        off_Aq = o; o += lc * (lc + 1);   // Aqk
        off_T = o;  o += lc * (lc + 1);   // T
        off_dec = o; o += dk;             // e^{G_last}
        off_row = o; o += lc;             // output token of each row, or -1
        total = o;
    }
};

template <typename TI, typename TG, typename TO, int LC>
__global__ void __launch_bounds__(kSimtThreads) chunk_simt_kernel(CoreParams p, int cw) {
    extern __shared__ float smem[];
    const int dk = (int)p.dk, dv = (int)p.dv, u = p.u;
    const SimtLayout Ly(dk, cw, LC, p.gw);
    const int ks = Ly.ks, gs = Ly.gs, ls = LC + 1;
    float *Sm = smem + Ly.off_S, *Kc = smem + Ly.off_K, *Qc = smem + Ly.off_Q, *KE = smem + Ly.off_KE;
    float *Wm = smem + Ly.off_W, *Gc = smem + Ly.off_G, *Vn = smem + Ly.off_V, *Um = smem + Ly.off_U;
    float *Akk = smem + Ly.off_A, *Aqk = smem + Ly.off_Aq, *Tm = smem + Ly.off_T, *dec = smem + Ly.off_dec;
    int *row_tok = reinterpret_cast<int *>(smem + Ly.off_row);

    const int64_t bh = blockIdx.x;
    const int64_t b = bh / p.heads, h = bh % p.heads, H = p.heads;
    const int c0 = blockIdx.y * cw;
    const int tid = threadIdx.x;
    const int64_t P = p.seq * u;  // folded length
    const bool gated = p.gw > 0, channel = p.gw > 1;
    const int gwid = channel ? dk : 1;

    const TI *q = static_cast<const TI *>(p.q);
    const TI *k = static_cast<const TI *>(p.k);
    const TI *v = static_cast<const TI *>(p.v);
    const TG *erase = static_cast<const TG *>(p.erase);
    const TG *write = static_cast<const TG *>(p.write);
    const TG *g = static_cast<const TG *>(p.g);
    TO *y = static_cast<TO *>(p.y);

    const float *S_in = p.state_in + bh * (int64_t)dk * dv;
    for (int idx = tid; idx < dk * cw; idx += kSimtThreads) {
        const int i = idx / cw, j = idx % cw;
        Sm[idx] = (c0 + j < dv) ? S_in[(int64_t)i * dv + c0 + j] : 0.f;
    }

    const int64_t nchunks = (P + LC - 1) / LC;
    for (int64_t c = 0; c < nchunks; ++c) {
        // ---- load the chunk (folded rows; zero pad past the end) ----
        for (int idx = tid; idx < LC * dk; idx += kSimtThreads) {
            const int l = idx / dk, d = idx % dk;
            const int64_t pos = c * LC + l;
            const bool valid = pos < P;
            const int64_t t = pos / u;
            const int m = (int)(pos % u);
            float kv = 0.f, ev = 0.f, qv = 0.f;
            if (valid) {
                const int64_t row = (b * P + pos) * H + h;
                kv = ld(k + row * dk + d);
                ev = ld(erase + row * p.ew + (p.ew == 1 ? 0 : d));
                if (m == u - 1) qv = p.scale * ld(q + ((b * p.seq + t) * H + h) * dk + d);
            }
            Kc[l * ks + d] = kv;
            KE[l * ks + d] = kv * ev;
            Qc[l * ks + d] = qv;
            if (d < gwid) {
                float gv = 0.f;
                if (gated && valid && m == 0) gv = ld(g + ((b * p.seq + t) * H + h) * p.gw + d);
                Gc[l * gs + d] = gv;
            }
        }
        for (int idx = tid; idx < LC * cw; idx += kSimtThreads) {
            const int l = idx / cw, j = idx % cw;
            const int64_t pos = c * LC + l;
            float val = 0.f;
            if (pos < P && c0 + j < dv) {
                const int64_t row = (b * P + pos) * H + h;
                val = ld(v + row * dv + c0 + j) * ld(write + row * p.ww + (p.ww == 1 ? 0 : c0 + j));
            }
            Vn[idx] = val;
        }
        for (int l = tid; l < LC; l += kSimtThreads) {
            const int64_t pos = c * LC + l;
            row_tok[l] = (pos < P && (int)(pos % u) == u - 1) ? (int)(pos / u) : -1;
        }
        __syncthreads();

        // ---- G = cumsum(g) within the chunk ----
        if (gated) {
            for (int d = tid; d < gwid; d += kSimtThreads) {
                float acc = 0.f;
                for (int l = 0; l < LC; ++l) {
                    acc += Gc[l * gs + d];
                    Gc[l * gs + d] = acc;
                }
            }
            __syncthreads();
        }

        // ---- the two score matrices ----
        for (int pr = tid; pr < LC * LC; pr += kSimtThreads) {
            const int a = pr / LC, j = pr % LC;
            float akk = 0.f, aqk = 0.f;
            if (j <= a) {
                if (channel) {
                    for (int d = 0; d < dk; ++d) {
                        const float kd = Kc[j * ks + d] * expf(Gc[a * gs + d] - Gc[j * gs + d]);
                        akk = fmaf(KE[a * ks + d], kd, akk);
                        aqk = fmaf(Qc[a * ks + d], kd, aqk);
                    }
                } else {
                    for (int d = 0; d < dk; ++d) {
                        akk = fmaf(KE[a * ks + d], Kc[j * ks + d], akk);
                        aqk = fmaf(Qc[a * ks + d], Kc[j * ks + d], aqk);
                    }
                    if (gated) {
                        const float mask = expf(Gc[a * gs] - Gc[j * gs]);
                        akk *= mask;
                        aqk *= mask;
                    }
                }
            }
            Akk[a * ls + j] = (j < a) ? akk : 0.f;
            Aqk[a * ls + j] = aqk;
        }
        __syncthreads();

        // ---- T = (I + Akk)^-1: lane j substitutes down column j ----
        if (tid < LC) {
            const int j = tid;
            float tc[LC];
#pragma unroll
            for (int a = 0; a < LC; ++a) {
                float acc = (a == j) ? 1.f : 0.f;
#pragma unroll
                for (int m = 0; m < a; ++m) acc = fmaf(-Akk[a * ls + m], tc[m], acc);
                tc[a] = acc;
                Tm[a * ls + j] = acc;
            }
        }
        // ---- gate factors (scores are done with the raw rows) ----
        if (gated) {
            for (int idx = tid; idx < LC * dk; idx += kSimtThreads) {
                const int l = idx / dk, d = idx % dk;
                const int gi = channel ? d : 0;
                const float gl = Gc[l * gs + gi], glast = Gc[(LC - 1) * gs + gi];
                KE[l * ks + d] *= expf(gl);
                Qc[l * ks + d] *= expf(gl);
                Kc[l * ks + d] *= expf(glast - gl);
            }
        }
        for (int d = tid; d < dk; d += kSimtThreads) dec[d] = gated ? expf(Gc[(LC - 1) * gs + (channel ? d : 0)]) : 1.f;
        __syncthreads();

        // ---- U = T (w v), W = T (b k e^G) ----
        for (int idx = tid; idx < LC * cw; idx += kSimtThreads) {
            const int a = idx / cw, j = idx % cw;
            float acc = 0.f;
            for (int m = 0; m <= a; ++m) acc = fmaf(Tm[a * ls + m], Vn[m * cw + j], acc);
            Um[idx] = acc;
        }
        for (int idx = tid; idx < LC * dk; idx += kSimtThreads) {
            const int a = idx / dk, d = idx % dk;
            float acc = 0.f;
            for (int m = 0; m <= a; ++m) acc = fmaf(Tm[a * ls + m], KE[m * ks + d], acc);
            Wm[a * ks + d] = acc;
        }
        __syncthreads();

        // ---- V' = U - W S ----
        for (int idx = tid; idx < LC * cw; idx += kSimtThreads) {
            const int a = idx / cw, j = idx % cw;
            float acc = Um[idx];
            for (int d = 0; d < dk; ++d) acc = fmaf(-Wm[a * ks + d], Sm[d * cw + j], acc);
            Vn[idx] = acc;
        }
        __syncthreads();

        // ---- y = (q e^G) S + Aqk V' on the output rows ----
        for (int idx = tid; idx < LC * cw; idx += kSimtThreads) {
            const int a = idx / cw, j = idx % cw;
            const int t = row_tok[a];
            if (t < 0 || c0 + j >= dv) continue;
            float acc = 0.f;
            for (int d = 0; d < dk; ++d) acc = fmaf(Qc[a * ks + d], Sm[d * cw + j], acc);
            for (int m = 0; m <= a; ++m) acc = fmaf(Aqk[a * ls + m], Vn[m * cw + j], acc);
            st(y + ((b * p.seq + t) * H + h) * dv + c0 + j, acc);
        }
        __syncthreads();

        // ---- S = e^{G_last} S + (k e^{G_last - G})^T V' ----
        for (int idx = tid; idx < dk * cw; idx += kSimtThreads) {
            const int d = idx / cw, j = idx % cw;
            float acc = dec[d] * Sm[idx];
            for (int l = 0; l < LC; ++l) acc = fmaf(Kc[l * ks + d], Vn[l * cw + j], acc);
            Sm[idx] = acc;
        }
        __syncthreads();
    }

    float *S_out = p.state_out + bh * (int64_t)dk * dv;
    for (int idx = tid; idx < dk * cw; idx += kSimtThreads) {
        const int i = idx / cw, j = idx % cw;
        if (c0 + j < dv) S_out[(int64_t)i * dv + c0 + j] = Sm[idx];
    }
}

}  // namespace dc
