/*
 * oracle.h — CPU restatement of burn-deltanet's delta-rule core.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels in burn-deltanet_b200/csrc and the timed CPU baseline of bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py (its CPU-baseline leg and
 * its `--impl reference` arm) may load it.  The product path never calls it.
 *
 * Parity pin: the float64 build reproduces the reference's own golden vectors
 * (src/delta/tests/reference.rs:17-59, generated from flash-linear-attention's
 * naive recurrences by scripts/gen_fixture.py) to <1e-12 on the recurrent path
 * and <1e-4 on the chunked path, mirroring the reference's own
 * tests (src/delta/tests.rs:533-568, 760-812).
 *
 * Layouts are the reference's (src/delta/path.rs:120-141):
 *   per-token tensors  [batch, seq, heads, width]   (row-major, contiguous)
 *   state              [batch, heads, dk, dv]
 * Gate widths: erase_w in {1, dk}, write_w in {1, dv}, g_w in {0 (no gate), 1, dk}.
 */
#ifndef DELTACORE_ORACLE_H
#define DELTACORE_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    long batch, seq, heads, dk, dv;
    long erase_w, write_w, g_w;  /* g_w == 0: no forget gate (alpha == 1) */
    double scale;                /* readout scale, already resolved (1/sqrt(dk) by default) */
    int threads;                 /* OpenMP threads; <= 0 means the runtime default */
} orc_dims;

/* Token-by-token recurrence: src/delta/recurrent.rs:41-99 (delta_step) unrolled
 * as in recurrent.rs:107-142 (delta_recurrent).  s_out may alias s0. */
void orc_recurrent_f64(const orc_dims *d, const double *q, const double *k, const double *v,
                       const double *erase, const double *write, const double *g,
                       const double *s0, double *y, double *s_out);
void orc_recurrent_f32(const orc_dims *d, const float *q, const float *k, const float *v,
                       const float *erase, const float *write, const float *g,
                       const float *s0, float *y, float *s_out);

/* Chunkwise WY forward: src/delta/chunk.rs:41-221 with the per-channel score
 * split of src/delta/decay.rs:82-143 and the blocked (I-N)^-1 ladder of
 * src/delta/tri.rs:72-136.  s_out may alias s0. */
void orc_chunk_f64(const orc_dims *d, long chunk_len, const double *q, const double *k,
                   const double *v, const double *erase, const double *write, const double *g,
                   const double *s0, double *y, double *s_out);
void orc_chunk_f32(const orc_dims *d, long chunk_len, const float *q, const float *k,
                   const float *v, const float *erase, const float *write, const float *g,
                   const float *s0, float *y, float *s_out);

/* Blocked unit-lower inverse (I - N)^-1 of `count` strictly-lower [size,size]
 * matrices: src/delta/tri.rs:72-114 (TriSolve::Blocked).  Exposed for the
 * reference's tri-solve known-answer tests (src/delta/tri/tests.rs). */
void orc_unit_lower_inverse_f64(long count, long size, const double *n_strict, double *t);

#ifdef __cplusplus
}
#endif
#endif
