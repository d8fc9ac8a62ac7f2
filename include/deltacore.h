/*
 * deltacore.h — C ABI of the B200 (sm_100a) delta-rule core.
 *
 * A drop-in for the two device entry points of burn-deltanet's shared
 * delta-rule core (src/delta):
 *
 *   dc_chunk_fwd  replaces  DeltaChunkBackendExt::delta_chunk_recalculated
 *                           (src/delta/chunk_recalculated/chunk_recalculated.rs:105-151),
 *                           the chunkwise WY prefill forward every family's
 *                           `forward` reaches through DeltaInput::run
 *                           (src/delta/path.rs:215-231).
 *   dc_step       replaces  delta_step (src/delta/recurrent.rs:41-99), the
 *                           decode tick every family's `step` calls, and the
 *                           u-micro-step recurrence of DeltaProduct / GDN-2
 *                           decode (src/delta/recurrent.rs:107-142 on the
 *                           sequence built at src/delta_product/delta_product.rs:270-305).
 *
 * Layouts are the reference's (src/delta/path.rs:120-141), row-major and
 * contiguous, on the CUDA device that is current when the call is made:
 *   q            [batch, seq, heads, dk]
 *   k            [batch, seq*u, heads, dk]       u = n_householder
 *   v            [batch, seq*u, heads, dv]
 *   erase        [batch, seq*u, heads, erase_w]  erase_w in {1, dk}
 *   write        [batch, seq*u, heads, write_w]  write_w in {1, dv}
 *   g            [batch, seq, heads, g_w]        g_w in {0 (no gate), 1, dk}
 *   state_in/out [batch, heads, dk, dv]          float32 always
 *   y            [batch, seq, heads, dv]
 * With u > 1 the micro-step fold of DeltaProduct / GDN-2 runs inside the
 * kernel: token t's u micro-steps use rows t*u .. t*u+u-1 of k, v, erase and
 * write; q is read on the last micro-step and g applied on the first, and y
 * holds the last micro-step's readout (src/delta_product/delta_product.rs:178-228).
 * With u == 1 this is exactly the reference op's argument list.
 *
 * Ownership and threading: the caller owns every buffer, the workspace
 * included (see dc_chunk_workspace_size); nothing is allocated, nothing is
 * freed.  The call validates on the host, enqueues the
 * kernel(s) on `stream` and returns; it is asynchronous like every Burn
 * device op.  state_out may alias state_in (in-place update); no other
 * output may alias an input.  Calls on different streams are independent.
 *
 * Errors: the reference panics (assert!) on shape and width violations
 * (src/delta/path.rs:177-208, chunk_recalculated.rs:74-78,
 * recurrent.rs:51-54).  Here the same checks return a status code before
 * anything is enqueued.
 */
#ifndef DELTACORE_H
#define DELTACORE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DC_API __attribute__((visibility("default")))
#else
#define DC_API
#endif

/* Binary-compatible with cudaStream_t / CUstream (NULL = the legacy default stream). */
typedef struct CUstream_st *dc_stream_t;

enum dc_status {
    DC_OK = 0,
    DC_EINVAL_SHAPE = 1,       /* a dimension is inconsistent (e.g. seq == 0, path.rs:179) */
    DC_EINVAL_WIDTH = 2,       /* a gate's last axis is not 1 / full (path.rs:187-195) */
    DC_EUNSUPPORTED_DTYPE = 3, /* dtype code not in dc_dtype */
    DC_EINVAL_ARG = 4,         /* null pointer, chunk_len < 1 (path.rs:219), n_householder < 1,
                                  non-finite scale, misaligned pointer, aliasing outputs */
    DC_EUNSUPPORTED = 5,       /* beyond this build's limits: dk > 256 or n_householder > 8 */
    DC_ECUDA = 6,              /* a CUDA runtime call failed: see dc_last_cuda_error() */
    DC_EDEVICE = 7,            /* the current device is not an sm_100 (B200-class) GPU */
    DC_EWORKSPACE = 8,         /* a workspace was passed but is smaller than dc_chunk_workspace_size */
    DC_ESCRATCH = 9            /* dc_chunk_fwd_noalloc: the request needs more than DC_NOALLOC_SCRATCH_BYTES */
};

enum dc_dtype {
    DC_F32 = 0,
    DC_BF16 = 1
};

/* dc_chunk_args.flags */
#define DC_FLAG_FORCE_SIMT 0x1u /* dc_chunk_fwd: the CUDA-core chunk kernel even where a tensor-core one applies;
                                   dc_step: the per-tile kernel even where the streaming one applies */
#define DC_FLAG_RECURRENT 0x2u  /* DeltaPath::Recurrent: walk the sequence token by token with the fused
                                   decode tick (one launch per token, state updated in state_out) */
#define DC_FLAG_FORCE_SPLIT 0x4u /* take the two-kernel (workspace) tensor-core path even for per-head gates */
/* Test hook for the failure path, no counterpart in the reference: the launched kernel issues none of
 * its tile loads, so every bounded wait on them runs out (about 2 s) and the kernel returns early with
 * the device status word set to 1 (dc_device_status); y and the final state are not written.  Nothing
 * faults and the context stays usable.  Accepted by dc_chunk_fwd when it takes the tensor-core kernel
 * (dc_chunk_kernel_choice 1) and by dc_step when it takes the streaming decode kernel; any other call
 * with it returns DC_EINVAL_ARG. */
#define DC_FLAG_TEST_STALL 0x100u

/*
 * Chunkwise prefill.  Mirrors
 *   fn delta_chunk_recalculated(q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV, g_bshK,
 *                               state_bhkv, has_gate: bool, chunk_len: usize, scale: f64)
 *       -> (y_bshv, final_state_bhkv)
 * (src/delta/chunk_recalculated/chunk_recalculated.rs:115-126); has_gate is g_w != 0.
 * `scale` is already resolved (1/sqrt(dk) is the reference default, path.rs:161-165).
 * `chunk_len` is validated (>= 1) and, as in the reference, does not change the
 * result (src/delta/tests.rs:340-363): the kernels pick their own tile length.
 *
 * Two paths pass per-chunk operands through a caller-owned device workspace of
 * dc_chunk_workspace_size(args) bytes (16-byte aligned):
 *   - per-channel gates (erase_w == dk, write_w == dv or g_w == dk, i.e. GDN-2) with
 *     bf16 q/k/v and d = 128: two tcgen05 kernels;
 *   - every other call with dk, dv <= 128 and a per-head log-decay (or none) that the
 *     fused bf16 kernel does not take, fp32 inputs (the reference's precision) first:
 *     a chunk-parallel prep kernel and a scan, every product an fp32-accurate
 *     three-part tf32 product on the tensor cores.
 * With workspace == NULL such a call runs the CUDA-core kernel instead; a non-NULL
 * workspace smaller than required is DC_EWORKSPACE.
 */
typedef struct dc_chunk_args {
    int64_t batch, seq, heads, dk, dv;
    int32_t n_householder;
    int32_t erase_w, write_w, g_w;
    int32_t chunk_len;
    int32_t in_dtype;   /* q, k, v: DC_F32 or DC_BF16 */
    int32_t gate_dtype; /* erase, write, g */
    int32_t out_dtype;  /* y */
    uint32_t flags;
    double scale;
    const void *q, *k, *v, *erase, *write, *g;
    const float *state_in;
    void *y;
    float *state_out;
    void *workspace;          /* device scratch for the two workspace paths, or NULL */
    uint64_t workspace_bytes; /* its size */
} dc_chunk_args;

DC_API int dc_chunk_fwd(const dc_chunk_args *args, dc_stream_t stream);

/*
 * One decode token for every (batch, head).  Mirrors
 *   fn delta_step(q_bhk, k_bhk, v_bhv, erase_bhK, write_bhV, g_bhK: Option<_>,
 *                 state_bhkv, scale: f64) -> (y_bhv, next_state_bhkv)
 * (src/delta/recurrent.rs:41-50), with n_householder micro-steps folded in:
 *   q [batch, heads, dk]; k, v, erase, write [batch, u, heads, .]; g [batch, heads, g_w].
 * The state is read once and written once per call however large u is.
 */
typedef struct dc_step_args {
    int64_t batch, heads, dk, dv;
    int32_t n_householder;
    int32_t erase_w, write_w, g_w;
    int32_t in_dtype, gate_dtype, out_dtype;
    uint32_t flags;
    double scale;
    const void *q, *k, *v, *erase, *write, *g;
    const float *state_in;
    void *y;
    float *state_out;
} dc_step_args;

DC_API int dc_step(const dc_step_args *args, dc_stream_t stream);

/*
 * dc_chunk_fwd without any allocation: the two-kernel tensor-core path with its
 * per-chunk workspace in a fixed device array inside this library.  It has no
 * counterpart in the reference.
 *
 * For callers that cannot allocate device memory: an engine whose device
 * memory belongs to its own pool allocator and that hands an FFI call tensors
 * but no raw scratch buffer, or a latency-critical serving loop in which a
 * cudaMalloc (which may synchronise the device) is not allowed.  The caller
 * still passes every input and output; args->workspace is ignored.
 *
 * Serves requests the two-kernel path takes (bf16 q/k/v, dk = dv = 128,
 * n_householder = 1, 16-byte-aligned pointers; per-head gates included) that
 * need at most DC_NOALLOC_SCRATCH_BYTES of workspace (dc_chunk_workspace_size
 * with DC_FLAG_FORCE_SPLIT; about 97 KB per (batch, head, 64-token chunk),
 * e.g. one sequence of 2688 tokens over 16 heads).  Larger requests return
 * DC_ESCRATCH and others the two-kernel path does not take DC_EUNSUPPORTED,
 * before anything is enqueued; DC_FLAG_FORCE_SIMT / DC_FLAG_RECURRENT are
 * DC_EINVAL_ARG.
 *
 * Every GPU that loads the library holds the array until the process exits.
 * The first call on a device looks up the array's device address (with that
 * device current) and keeps it for the device's current context; make that
 * first call before any stream capture.  After cudaDeviceReset the device has
 * a new context, and the next call looks the address up again (so, again,
 * outside any capture).  All calls share the one array, which keeps the last call's
 * contents (nothing in it needs to start at zero), so calls whose work
 * overlaps on the GPU (different streams, or different host threads) race:
 * serialise them.
 */
#define DC_NOALLOC_SCRATCH_BYTES (64ull << 20)
DC_API int dc_chunk_fwd_noalloc(const dc_chunk_args *args, dc_stream_t stream);

/*
 * dc_chunk_fwd from host memory: args' q, k, v, erase, write, g and state_in are read from, and y and
 * state_out written to, HOST memory (page-locked for full PCIe speed).  No counterpart in the reference,
 * whose tensors already live on the backend's device.  The batch is cut into up to 8 slices of whole
 * sequences; each slice is copied in on one stream, computed on `stream` and copied out on another, two
 * slices in flight, so the transfers in both directions overlap each other and the kernels.  `scratch`
 * is device memory of at least dc_chunk_fwd_host_scratch_size(args) bytes, 256-byte aligned (both
 * slices' device copies, plus the two-kernel path's workspace); a smaller one is DC_EWORKSPACE.  The
 * work is ordered after everything already queued on `stream`, and `stream` is made to wait for all of
 * it: once `stream` has drained, y and state_out hold the results.  Creates (and releases) two streams
 * and seven events per call; allocates no memory.
 */
DC_API uint64_t dc_chunk_fwd_host_scratch_size(const dc_chunk_args *args);
DC_API int dc_chunk_fwd_host(const dc_chunk_args *args, void *scratch, uint64_t scratch_bytes, dc_stream_t stream);

/*
 * The backward of dc_chunk_fwd: the gradients the reference's custom autodiff node returns.  Mirrors
 *   fn combined_backward(d_y_bshv, d_final_state_bhkv, q_bshk, k_bshk, v_bshv, erase_bshK, write_bshV,
 *                        g_bshK: Option<_>, state_bhkv, chunk_len, scale) -> DeltaChunkGrads
 * (src/delta/chunk_recalculated/combined_backward.rs:72-84), i.e. the derivatives of
 * L = <y, d_y> + <final_state, d_state_final> with respect to every input of the forward call
 * described by `fwd` (its y, state_out and workspace fields are not used).  Gradients are float32 in
 * the layouts of their inputs, gate gradients at the gate's own width (summed over a broadcast axis);
 * d_g is written when fwd.g_w > 0.  d_state_final may be NULL (zero).  Needs dk, dv <= 128 and a device
 * workspace of dc_chunk_bwd_workspace_size(args) bytes (16-byte aligned).  Two implementations, both
 * deterministic (every gradient element written once):
 *   - a log-decay per head or none (fwd.g_w <= 1): chunked, chunks of 32 micro-steps, three kernels
 *     (the chunks' WY factors, a forward and reverse scan over the chunks per 32 value columns, the
 *     chunks' gradients), fp32-accurate tf32 products on the tensor cores.  Workspace per chunk: its WY
 *     factors, V' and dV', and the state and state gradient at its boundary (about 240 KB at dk = dv = 128);
 *   - per-channel log-decays (fwd.g_w == dk), or DC_FLAG_RECURRENT in fwd.flags: the recurrence walked
 *     back token by token on the CUDA cores, one CTA per (batch, head, 32 value columns).  Workspace: per
 *     (batch, head, 32 value columns) the state at every 16th micro-step and a 16-step replay buffer, and
 *     with dv > 32 the slices' partial sums of the gradients that sum over value columns.
 */
typedef struct dc_chunk_bwd_args {
    dc_chunk_args fwd;
    const float *d_y;           /* [batch, seq, heads, dv] */
    const float *d_state_final; /* [batch, heads, dk, dv], or NULL */
    float *d_q;                 /* [batch, seq, heads, dk] */
    float *d_k;                 /* [batch, seq*u, heads, dk] */
    float *d_v;                 /* [batch, seq*u, heads, dv] */
    float *d_erase;             /* [batch, seq*u, heads, erase_w] */
    float *d_write;             /* [batch, seq*u, heads, write_w] */
    float *d_g;                 /* [batch, seq, heads, g_w], or NULL when g_w == 0 */
    float *d_state;             /* [batch, heads, dk, dv] */
    void *workspace;
    uint64_t workspace_bytes;
} dc_chunk_bwd_args;

DC_API uint64_t dc_chunk_bwd_workspace_size(const dc_chunk_bwd_args *args);
DC_API int dc_chunk_bwd(const dc_chunk_bwd_args *args, dc_stream_t stream);

/*
 * The per-head output normalisation after the read-out.  Mirrors OutNorm::forward
 * (src/common/norm.rs:129-135): over each row of y [rows, dv] (rows = batch * seq * heads; one head's
 * dv values),
 *   gate != NULL (OutNorm::Gated, burn-stack RmsNormGated):  out = y / sqrt(mean(y^2) + eps) * weight * silu(gate)
 *   gate == NULL (OutNorm::Plain, burn-stack RmsNorm):       out = y / sqrt(mean(y^2) + eps) * weight
 * with silu(x) = x / (1 + e^-x), fp32 arithmetic.  y and gate share in_dtype, out has out_dtype
 * (DC_F32 or DC_BF16); weight is float32 [dv].  1 <= dv <= 256; rows may be 0.  out may alias y.
 * The reference panics on a gate / norm mismatch; here the presence of gate selects the form.
 */
typedef struct dc_out_norm_args {
    int64_t rows;
    int64_t dv;
    int32_t in_dtype, out_dtype;
    float eps;
    const void *y;
    const void *gate;
    const float *weight;
    void *out;
} dc_out_norm_args;

DC_API int dc_out_norm(const dc_out_norm_args *args, dc_stream_t stream);

/*
 * The prefill followed by the output norm: what a block's forward does with the core's read-out before
 * out_proj (src/common/norm.rs:129-135 on the y of chunk_recalculated.rs:115-126).  No single reference
 * function; the two reference steps in one call.  `chunk` is exactly dc_chunk_fwd's argument; `norm`
 * gives the norm's gate (NULL: OutNorm::Plain), weight [dv] float32 and eps, with rows = batch * seq *
 * heads, dv = chunk->dv, out_dtype = chunk->out_dtype and, with a gate, in_dtype = chunk->out_dtype (the
 * gate's dtype); its y and out must be NULL.  The normalised rows are written to chunk->y in place of the
 * read-out, and the final state to chunk->state_out as usual.
 * Where the fused tensor-core kernel serves the call (dc_chunk_kernel_choice 1) and the norm is plain,
 * each row is normalised inside the kernel's read-out, from the float32 accumulator, before y is
 * rounded to out_dtype: the read-out never makes the round trip through HBM.  Otherwise the call is
 * dc_chunk_fwd followed by dc_out_norm in place on y.
 */
DC_API int dc_chunk_fwd_out_norm(const dc_chunk_args *chunk, const dc_out_norm_args *norm, dc_stream_t stream);
/* 1 if dc_chunk_fwd_out_norm fuses the norm for these arguments, 0 if it runs the two kernels; negative
 * = the dc_status the call would return.  Pure host logic. */
DC_API int dc_chunk_fwd_out_norm_fused(const dc_chunk_args *chunk, const dc_out_norm_args *norm);

/*
 * The front-end between the fused input projection and the core, on the projection's [q | u k | u v]
 * channel segment (QkvProjection::forward / step after in_proj, src/common/qkv.rs:373-500):
 *   the causal depthwise short convolution with its rolling window (src/common/conv.rs:81-160): x is
 *   left-padded with window_in's newest conv_kernel - 1 columns (zeros when NULL), y[c, t] = bias[c] +
 *   sum_j weight[c, j] x_pad[c, t + j], and window_out receives the padded input's last conv_kernel
 *   columns (the next call's window; not written when NULL; must not overlap window_in);
 *   then SiLU on every channel (DC_PROLOGUE_CONV_SILU), or else SiLU on v and, with
 *   DC_PROLOGUE_QK_SILU, on q and k (qkv.rs:405-413);
 *   then, with DC_PROLOGUE_L2, q and k over each head: x / sqrt(sum x^2 + 1e-6) (norm.rs:83-90).
 * Outputs: q [batch, seq, heads, dk], k [batch, seq*u, heads, dk], v [batch, seq*u, heads, dv] (micro-step
 * m of token t is row t*u + m), in out_dtype.  x holds channel c of token t at (b*seq + t)*x_stride + c
 * (x_stride >= channels = heads*dk*(1 + u) + u*heads*dv, so x may be a column slice of the whole
 * projection), in in_dtype; conv_weight [channels, conv_kernel], conv_bias [channels] or NULL, windows
 * [batch, channels, conv_kernel], all float32.  seq >= 1 (conv.rs asserts it); a single-token step() is
 * seq = 1.  1 <= conv_kernel <= 8, dk, dv <= 128.  No GQA expansion (value heads = heads).
 */
#define DC_PROLOGUE_CONV_SILU 0x1u
#define DC_PROLOGUE_QK_SILU 0x2u
#define DC_PROLOGUE_L2 0x4u

typedef struct dc_qkv_prologue_args {
    int64_t batch, seq, heads, dk, dv;
    int32_t n_householder;
    int32_t conv_kernel;
    int32_t in_dtype, out_dtype;
    uint32_t flags;
    int64_t x_stride;
    const void *x;
    const float *conv_weight;
    const float *conv_bias;
    const float *window_in;
    float *window_out;
    void *q, *k, *v;
} dc_qkv_prologue_args;

DC_API int dc_qkv_prologue(const dc_qkv_prologue_args *args, dc_stream_t stream);

/*
 * The front-end's gate producers: one elementwise map from a [rows, cols] column slice of the input
 * projection (x: element (r, c) at r*x_stride + c, in_dtype) to a contiguous float32 out [rows, cols]:
 *   DC_GATE_WRITE          out = scale * sigma(x): squash_write (src/common/qkv.rs:333-368), scale 2 for
 *                          the erase gate under allow_neg_eigval, else 1 (rows = batch*seq*u, cols = the
 *                          gate's heads, or heads*head_dim for WriteGate::Channel)
 *   DC_GATE_HEAD_DECAY     out = -exp(a_log[c]) * clamp(softplus(x + bias[c]), lo, hi): ForgetGate::log_decay
 *                          (src/common/gate.rs:51-59), cols = heads (rows = batch*seq)
 *   DC_GATE_CHANNEL_DECAY  out = scale * sigma((x + bias[c]) * exp(a_log[c / group])): ChannelForgetGate::
 *                          log_decay (gate.rs:178-196) applied to its `up` projection's output, cols =
 *                          heads*group (group = head_k_dim), scale = the lower bound
 * softplus(x) = log(1 + e^x).  bias and a_log are float32 (unused ones may be NULL).  rows may be 0.
 */
#define DC_GATE_WRITE 0
#define DC_GATE_HEAD_DECAY 1
#define DC_GATE_CHANNEL_DECAY 2

typedef struct dc_gate_args {
    int64_t rows, cols, x_stride;
    int32_t kind, in_dtype, group;
    float scale, lo, hi;
    const void *x;
    const float *bias;
    const float *a_log;
    float *out;
} dc_gate_args;

DC_API int dc_gates(const dc_gate_args *args, dc_stream_t stream);

/* Human-readable name of a dc_status. */
DC_API const char *dc_status_string(int status);

/* The cudaError_t behind the most recent DC_ECUDA returned on this thread (0 if none). */
DC_API int dc_last_cuda_error(void);

/* The device status word of the current device (synchronising): 0 while every kernel
 * ran to completion; 1 after a kernel's bounded wait on its own tensor-core or TMA
 * work ran out (its outputs are then invalid).  `reset` != 0 clears it.  A negative
 * value is -dc_status of a failed query. */
DC_API int dc_device_status(int reset);

/* Which chunk kernel dc_chunk_fwd would launch for `args`: 1 = tensor-core (tcgen05),
 * 2 = the two-kernel tensor-core path over the workspace, 3 = the fp32-accurate chunked
 * path over the workspace, 0 = CUDA-core; negative = the dc_status the call would
 * return.  Pure host logic. */
DC_API int dc_chunk_kernel_choice(const dc_chunk_args *args);

/* Bytes of workspace the call's workspace path needs for `args` (0 when the call takes a
 * path that needs none).  Replaces nothing in the reference, whose chunk path
 * materialises its intermediates as backend tensors (forward.rs:235-266).  Pure
 * host logic; about 97 KB per (batch, head, 64-token chunk) for per-channel gates,
 * about 68 KB per (batch, head, 32 micro-steps) at d = 128 for the fp32-accurate path. */
DC_API uint64_t dc_chunk_workspace_size(const dc_chunk_args *args);

/* Number of kernels dc_chunk_fwd enqueues for `args` (for launch accounting); dc_step enqueues one.
 * Negative: -dc_status of a call dc_chunk_fwd would reject. */
DC_API int dc_chunk_launches(const dc_chunk_args *args);

/* ABI version: major * 10000 + minor * 100 + patch. */
DC_API int dc_version(void);

#ifdef __cplusplus
}
#endif
#endif /* DELTACORE_H */
