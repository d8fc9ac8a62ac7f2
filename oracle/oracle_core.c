/*
 * oracle_core.c — CPU restatement of burn-deltanet's delta-rule core.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled twice by oracle/Makefile:
 * once with REAL=double (the parity oracle) and once with REAL=float (the
 * timed CPU baseline).  Every function names the reference lines it follows.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#include "oracle.h"

#ifndef REAL
#define REAL double
#define SFX _f64
#endif
#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)
#define FN(name) CAT(name, SFX)

#if defined(REAL_IS_FLOAT)
#define EXP expf
#else
#define EXP exp
#endif

/* Clamp on either factor's exponent in the per-channel score split:
 * src/delta/decay.rs:49 (MAX_EXPONENT). */
#define MAX_EXPONENT 48.0
/* Rows sharing one reference point: src/delta/decay.rs:39 (DECAY_BLOCK_LEN). */
#define DECAY_BLOCK_LEN 16

static int nthreads(const orc_dims *d) { return d->threads > 0 ? d->threads : omp_get_max_threads(); }

/* Offset of element [b, t, h, 0] of a [batch, seq, heads, width] tensor. */
static long tok(const orc_dims *d, long b, long t, long h, long width) {
    return ((b * d->seq + t) * d->heads + h) * width;
}

/* ------------------------------------------------------------------------- */
/* Recurrent: src/delta/recurrent.rs:41-99 (one tick), :107-142 (unrolled).   */
/* ------------------------------------------------------------------------- */
void FN(orc_recurrent)(const orc_dims *d, const REAL *q, const REAL *k, const REAL *v,
                       const REAL *erase, const REAL *write, const REAL *g,
                       const REAL *s0, REAL *y, REAL *s_out) {
    const long B = d->batch, T = d->seq, H = d->heads, K = d->dk, V = d->dv;
    const REAL scale = (REAL)d->scale;
#pragma omp parallel for collapse(2) schedule(dynamic) num_threads(nthreads(d))
    for (long b = 0; b < B; b++) {
        for (long h = 0; h < H; h++) {
            REAL *S = s_out + (b * H + h) * K * V;
            if (S != s0 + (b * H + h) * K * V) memcpy(S, s0 + (b * H + h) * K * V, sizeof(REAL) * K * V);
            REAL *u = (REAL *)malloc(sizeof(REAL) * V);
            for (long t = 0; t < T; t++) {
                const REAL *qt = q + tok(d, b, t, h, K), *kt = k + tok(d, b, t, h, K);
                const REAL *vt = v + tok(d, b, t, h, V);
                const REAL *et = erase + tok(d, b, t, h, d->erase_w);
                const REAL *wt = write + tok(d, b, t, h, d->write_w);
                /* S- = exp(g) (.) S on the key axis (recurrent.rs:57-64) */
                if (d->g_w > 0) {
                    const REAL *gt = g + tok(d, b, t, h, d->g_w);
                    for (long i = 0; i < K; i++) {
                        REAL a = EXP(gt[d->g_w == 1 ? 0 : i]);
                        for (long j = 0; j < V; j++) S[i * V + j] *= a;
                    }
                }
                /* u = write (.) v - (erase (.) k)^T S-   (recurrent.rs:69-76) */
                for (long j = 0; j < V; j++) {
                    REAL acc = 0;
                    for (long i = 0; i < K; i++) acc += (kt[i] * et[d->erase_w == 1 ? 0 : i]) * S[i * V + j];
                    u[j] = vt[j] * wt[d->write_w == 1 ? 0 : j] - acc;
                }
                /* S = S- + k u^T   (recurrent.rs:80-83) */
                for (long i = 0; i < K; i++)
                    for (long j = 0; j < V; j++) S[i * V + j] += kt[i] * u[j];
                /* y = S^T (scale q), read after the write (recurrent.rs:90-93) */
                REAL *yt = y + tok(d, b, t, h, V);
                for (long j = 0; j < V; j++) {
                    REAL acc = 0;
                    for (long i = 0; i < K; i++) acc += (qt[i] * scale) * S[i * V + j];
                    yt[j] = acc;
                }
            }
            free(u);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Blocked unit-lower inverse: src/delta/tri.rs:72-114 and :122-136.          */
/* ------------------------------------------------------------------------- */

/* 1 where floor(i/block) > floor(j/block); all zero once block >= size. */
static int block_strict_lower(long size, long block, long i, long j) {
    if (block >= size) return 0;
    return (i / block) > (j / block);
}

/* t = (I - n)^-1 for one strictly-lower [L, L] n, by the doubling ladder
 * P <- P + P X P with X = n masked to the blocks the level absorbs. */
static void FN(unit_lower_inverse_one)(long L, const REAL *n, REAL *p, REAL *x, REAL *px, REAL *tmp) {
    for (long i = 0; i < L; i++)
        for (long j = 0; j < L; j++) p[i * L + j] = (i == j) ? (REAL)1 : (REAL)0;
    long block = 1;
    while (block < L) {
        for (long i = 0; i < L; i++)
            for (long j = 0; j < L; j++) {
                int sel = block_strict_lower(L, block, i, j) - block_strict_lower(L, 2 * block, i, j);
                x[i * L + j] = sel ? n[i * L + j] : (REAL)0;
            }
        /* px = P X ; tmp = (P X) P ; P += tmp */
        for (long i = 0; i < L; i++)
            for (long j = 0; j < L; j++) {
                REAL acc = 0;
                for (long m = 0; m < L; m++) acc += p[i * L + m] * x[m * L + j];
                px[i * L + j] = acc;
            }
        for (long i = 0; i < L; i++)
            for (long j = 0; j < L; j++) {
                REAL acc = 0;
                for (long m = 0; m < L; m++) acc += px[i * L + m] * p[m * L + j];
                tmp[i * L + j] = acc;
            }
        for (long i = 0; i < L * L; i++) p[i] += tmp[i];
        block *= 2;
    }
}

#if !defined(REAL_IS_FLOAT)
void orc_unit_lower_inverse_f64(long count, long size, const double *n_strict, double *t) {
    double *x = malloc(sizeof(double) * size * size), *px = malloc(sizeof(double) * size * size);
    double *tmp = malloc(sizeof(double) * size * size);
    for (long c = 0; c < count; c++)
        unit_lower_inverse_one_f64(size, n_strict + c * size * size, t + c * size * size, x, px, tmp);
    free(x); free(px); free(tmp);
}
#endif

/* Largest block length dividing chunk_len, at most DECAY_BLOCK_LEN
 * (src/delta/decay.rs:55-60). */
static long decay_block_len(long chunk_len) {
    long lim = chunk_len < DECAY_BLOCK_LEN ? chunk_len : DECAY_BLOCK_LEN;
    for (long m = lim; m >= 1; m--)
        if (chunk_len % m == 0) return m;
    return 1;
}

/* ------------------------------------------------------------------------- */
/* Chunkwise WY: src/delta/chunk.rs:41-221.                                   */
/* ------------------------------------------------------------------------- */
void FN(orc_chunk)(const orc_dims *d, long L, const REAL *q, const REAL *k, const REAL *v,
                   const REAL *erase, const REAL *write, const REAL *g, const REAL *s0,
                   REAL *y, REAL *s_out) {
    const long B = d->batch, T = d->seq, H = d->heads, K = d->dk, V = d->dv;
    const long EW = d->erase_w, WW = d->write_w, GW = d->g_w;
    const REAL scale = (REAL)d->scale;
    const int channel = GW > 1;                     /* path.rs:170-172 */
    const long nchunks = (T + L - 1) / L;           /* chunk.rs:61 (pad to a multiple of L) */
    const long m = decay_block_len(L), nblocks = L / m;

#pragma omp parallel num_threads(nthreads(d))
    {
        REAL *Q = malloc(sizeof(REAL) * L * K), *Kc = malloc(sizeof(REAL) * L * K);
        REAL *Ke = malloc(sizeof(REAL) * L * K), *Vw = malloc(sizeof(REAL) * L * V);
        REAL *GC = malloc(sizeof(REAL) * L * (GW > 0 ? GW : 1));
        REAL *Akk = malloc(sizeof(REAL) * L * L), *Aqk = malloc(sizeof(REAL) * L * L);
        REAL *N = malloc(sizeof(REAL) * L * L), *Tm = malloc(sizeof(REAL) * L * L);
        REAL *X = malloc(sizeof(REAL) * L * L), *PX = malloc(sizeof(REAL) * L * L);
        REAL *TMP = malloc(sizeof(REAL) * L * L);
        REAL *U = malloc(sizeof(REAL) * L * V), *W = malloc(sizeof(REAL) * L * K);
        REAL *Vn = malloc(sizeof(REAL) * L * V);
        REAL *ROW = channel ? malloc(sizeof(REAL) * L * K) : NULL;
        REAL *COL = channel ? malloc(sizeof(REAL) * nblocks * L * K) : NULL;
        REAL *Snew = malloc(sizeof(REAL) * K * V);

#pragma omp for collapse(2) schedule(dynamic)
        for (long b = 0; b < B; b++) {
            for (long h = 0; h < H; h++) {
                REAL *S = s_out + (b * H + h) * K * V;
                if (S != s0 + (b * H + h) * K * V) memcpy(S, s0 + (b * H + h) * K * V, sizeof(REAL) * K * V);
                for (long c = 0; c < nchunks; c++) {
                    /* ---- chunk layout, zero pad, q.scale (chunk.rs:61-94) ---- */
                    for (long l = 0; l < L; l++) {
                        long t = c * L + l;
                        int valid = t < T;
                        for (long i = 0; i < K; i++) {
                            Q[l * K + i] = valid ? q[tok(d, b, t, h, K) + i] * scale : 0;
                            Kc[l * K + i] = valid ? k[tok(d, b, t, h, K) + i] : 0;
                            REAL e = valid ? erase[tok(d, b, t, h, EW) + (EW == 1 ? 0 : i)] : 0;
                            Ke[l * K + i] = Kc[l * K + i] * e;               /* chunk.rs:103 */
                        }
                        for (long j = 0; j < V; j++) {
                            REAL vv = valid ? v[tok(d, b, t, h, V) + j] : 0;
                            REAL w = valid ? write[tok(d, b, t, h, WW) + (WW == 1 ? 0 : j)] : 0;
                            Vw[l * V + j] = vv * w;                          /* chunk.rs:104 */
                        }
                        /* gc = cumsum(g) within the chunk (chunk.rs:101) */
                        for (long x = 0; x < GW; x++) {
                            REAL gv = valid ? g[tok(d, b, t, h, GW) + x] : 0;
                            GC[l * GW + x] = (l == 0 ? 0 : GC[(l - 1) * GW + x]) + gv;
                        }
                    }
                    /* ---- the two score matrices (chunk.rs:109-137) ---- */
                    if (channel) {
                        /* BlockDecay::new (decay.rs:82-122): reference at each
                         * block's middle row, exponents clamped at 48, -inf
                         * for column blocks after the row block. */
                        for (long l = 0; l < L; l++) {
                            long ref = (l / m) * m + m / 2;
                            for (long i = 0; i < K; i++) {
                                REAL e = GC[l * K + i] - GC[ref * K + i];
                                if (e > MAX_EXPONENT) e = MAX_EXPONENT;
                                ROW[l * K + i] = EXP(e);
                            }
                        }
                        for (long p = 0; p < nblocks; p++) {
                            long ref = p * m + m / 2;
                            for (long j = 0; j < L; j++)
                                for (long i = 0; i < K; i++) {
                                    REAL e = GC[ref * K + i] - GC[j * K + i];
                                    if (e > MAX_EXPONENT) e = MAX_EXPONENT;
                                    COL[(p * L + j) * K + i] = (j / m > p) ? 0 : Kc[j * K + i] * EXP(e);
                                }
                        }
                        /* BlockDecay::scores (decay.rs:130-143) */
                        for (long a = 0; a < L; a++) {
                            long p = a / m;
                            for (long bb = 0; bb < L; bb++) {
                                REAL akk = 0, aqk = 0;
                                for (long i = 0; i < K; i++) {
                                    REAL col = COL[(p * L + bb) * K + i];
                                    akk += (Ke[a * K + i] * ROW[a * K + i]) * col;
                                    aqk += (Q[a * K + i] * ROW[a * K + i]) * col;
                                }
                                Akk[a * L + bb] = akk;
                                Aqk[a * L + bb] = aqk;
                            }
                        }
                    } else {
                        for (long a = 0; a < L; a++)
                            for (long bb = 0; bb < L; bb++) {
                                REAL akk = 0, aqk = 0;
                                for (long i = 0; i < K; i++) {
                                    akk += Ke[a * K + i] * Kc[bb * K + i];
                                    aqk += Q[a * K + i] * Kc[bb * K + i];
                                }
                                if (GW == 1) {
                                    /* mask = exp(gc_a - gc_b), 0 above the diagonal */
                                    REAL mask = bb <= a ? EXP(GC[a] - GC[bb]) : 0;
                                    akk *= mask;
                                    aqk *= mask;
                                }
                                Akk[a * L + bb] = akk;
                                Aqk[a * L + bb] = aqk;
                            }
                    }
                    /* ---- WY transform (chunk.rs:144-157) ---- */
                    for (long a = 0; a < L; a++)
                        for (long bb = 0; bb < L; bb++) N[a * L + bb] = bb < a ? -Akk[a * L + bb] : 0;
                    FN(unit_lower_inverse_one)(L, N, Tm, X, PX, TMP);
                    for (long a = 0; a < L; a++) {
                        for (long j = 0; j < V; j++) {
                            REAL acc = 0;
                            for (long bb = 0; bb < L; bb++) acc += Tm[a * L + bb] * Vw[bb * V + j];
                            U[a * V + j] = acc;
                        }
                        for (long i = 0; i < K; i++) {
                            REAL acc = 0;
                            for (long bb = 0; bb < L; bb++) {
                                REAL kg = Ke[bb * K + i];
                                if (GW > 0) kg *= EXP(GC[bb * GW + (GW == 1 ? 0 : i)]);
                                acc += Tm[a * L + bb] * kg;
                            }
                            W[a * K + i] = acc;
                        }
                    }
                    /* ---- one scan step (chunk.rs:169-205) ---- */
                    /* V' = U - W S */
                    for (long a = 0; a < L; a++)
                        for (long j = 0; j < V; j++) {
                            REAL acc = 0;
                            for (long i = 0; i < K; i++) acc += W[a * K + i] * S[i * V + j];
                            Vn[a * V + j] = U[a * V + j] - acc;
                        }
                    /* y = (q (.) e^G) S + tril(Aqk) V' */
                    for (long a = 0; a < L; a++) {
                        long t = c * L + a;
                        if (t >= T) continue;
                        REAL *yt = y + tok(d, b, t, h, V);
                        for (long j = 0; j < V; j++) {
                            REAL acc = 0;
                            for (long i = 0; i < K; i++) {
                                REAL qr = Q[a * K + i];
                                if (GW > 0) qr *= EXP(GC[a * GW + (GW == 1 ? 0 : i)]);
                                acc += qr * S[i * V + j];
                            }
                            REAL acc2 = 0;
                            for (long bb = 0; bb <= a; bb++) acc2 += Aqk[a * L + bb] * Vn[bb * V + j];
                            yt[j] = acc + acc2;
                        }
                    }
                    /* S <- S (.) e^{G_last} + (K (.) e^{G_last - G})^T V' */
                    for (long i = 0; i < K; i++)
                        for (long j = 0; j < V; j++) {
                            REAL dec = 1;
                            if (GW > 0) dec = EXP(GC[(L - 1) * GW + (GW == 1 ? 0 : i)]);
                            REAL acc = 0;
                            for (long bb = 0; bb < L; bb++) {
                                REAL kc = Kc[bb * K + i];
                                if (GW > 0) {
                                    long x = GW == 1 ? 0 : i;
                                    kc *= EXP(GC[(L - 1) * GW + x] - GC[bb * GW + x]);
                                }
                                acc += kc * Vn[bb * V + j];
                            }
                            Snew[i * V + j] = S[i * V + j] * dec + acc;
                        }
                    memcpy(S, Snew, sizeof(REAL) * K * V);
                }
            }
        }
        free(Q); free(Kc); free(Ke); free(Vw); free(GC); free(Akk); free(Aqk); free(N); free(Tm);
        free(X); free(PX); free(TMP); free(U); free(W); free(Vn); free(ROW); free(COL); free(Snew);
    }
}
