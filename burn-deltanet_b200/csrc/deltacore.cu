// deltacore.cu — the C ABI (include/deltacore.h): host-side validation and
// kernel dispatch for the delta-rule core on sm_100a.
//
// Validation mirrors the reference's asserts (src/delta/path.rs:177-208,
// src/delta/recurrent.rs:51-54, path.rs:219) but returns a status code before
// anything is enqueued instead of panicking.  Nothing here allocates device
// memory and nothing falls back to the host: an unsupported request is an
// error, not a slower path.
#include <math.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include <cuda_runtime.h>

#include "../../include/deltacore.h"
#include "chunk_simt.cuh"
#include "chunk_split.cuh"
#include "bwd_chunk.cuh"
#include "bwd_recurrent.cuh"
#include "chunk_f32.cuh"
#include "chunk_tc.cuh"
#include "out_norm.cuh"
#include "prologue.cuh"
#include "common.cuh"
#include "step.cuh"
#include "step_stream.cuh"

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return DC_ECUDA;
}

// Whether the current device is an sm_100 part, checked once per device.
int check_device(int *dev_out) {
    static int verdict[64];  // 0 unknown, 1 ok, 2 wrong arch
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev_out) *dev_out = dev;
    if (dev >= 0 && dev < 64 && verdict[dev]) return verdict[dev] == 1 ? DC_OK : DC_EDEVICE;
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return cuda_fail(e);
    const int ok = (major == 10 && minor == 0);
    if (dev >= 0 && dev < 64) verdict[dev] = ok ? 1 : 2;
    return ok ? DC_OK : DC_EDEVICE;
}

bool valid_dtype(int32_t t) { return t == DC_F32 || t == DC_BF16; }
size_t dtype_size(int32_t t) { return t == DC_F32 ? 4 : 2; }
bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// Shared checks of the two entry points.  `rows` is the number of token rows
// of q, g and y (seq for the prefill, 1 for the step).
int validate_common(int64_t batch, int64_t rows, int64_t heads, int64_t dk, int64_t dv, int32_t u,
                    int32_t ew, int32_t ww, int32_t gw, int32_t in_dt, int32_t gate_dt, int32_t out_dt,
                    double scale, const void *q, const void *k, const void *v, const void *erase,
                    const void *write, const void *g, const float *s_in, const void *y, const float *s_out) {
    if (batch < 0 || heads < 0 || dk < 1 || dv < 1 || rows < 1) return DC_EINVAL_SHAPE;
    if (!(ew == 1 || ew == dk)) return DC_EINVAL_WIDTH;
    if (!(ww == 1 || ww == dv)) return DC_EINVAL_WIDTH;
    if (!(gw == 0 || gw == 1 || gw == dk)) return DC_EINVAL_WIDTH;
    if (!valid_dtype(in_dt) || !valid_dtype(gate_dt) || !valid_dtype(out_dt)) return DC_EUNSUPPORTED_DTYPE;
    if (u < 1) return DC_EINVAL_ARG;
    if (!isfinite(scale)) return DC_EINVAL_ARG;
    if (dk > dc::kMaxDk || u > dc::kMaxHouseholder) return DC_EUNSUPPORTED;
    if (batch == 0 || heads == 0) return DC_OK;  // empty: nothing to do
    if (!q || !k || !v || !erase || !write || !s_in || !y || !s_out) return DC_EINVAL_ARG;
    if (gw != 0 && !g) return DC_EINVAL_ARG;
    const size_t is = dtype_size(in_dt), gs = dtype_size(gate_dt), os = dtype_size(out_dt);
    if (!aligned(q, is) || !aligned(k, is) || !aligned(v, is)) return DC_EINVAL_ARG;
    if (!aligned(erase, gs) || !aligned(write, gs) || (g && !aligned(g, gs))) return DC_EINVAL_ARG;
    if (!aligned(y, os) || !aligned(s_in, 4) || !aligned(s_out, 4)) return DC_EINVAL_ARG;
    // Outputs must not alias inputs (state_out == state_in is the one allowed in-place update).
    const void *ins[] = {q, k, v, erase, write, g};
    for (const void *in : ins)
        if (in && (in == y || in == (const void *)s_out)) return DC_EINVAL_ARG;
    if ((const void *)y == (const void *)s_in || (const void *)y == (const void *)s_out) return DC_EINVAL_ARG;
    return DC_OK;
}

dc::CoreParams make_params(int64_t batch, int64_t seq, int64_t heads, int64_t dk, int64_t dv, int32_t u,
                           int32_t ew, int32_t ww, int32_t gw, double scale, const void *q, const void *k,
                           const void *v, const void *erase, const void *write, const void *g,
                           const float *s_in, void *y, float *s_out) {
    dc::CoreParams p;
    p.batch = batch; p.seq = seq; p.heads = heads; p.dk = dk; p.dv = dv;
    p.u = u; p.ew = ew; p.ww = ww; p.gw = gw;
    p.scale = (float)scale;
    p.q = q; p.k = k; p.v = v; p.erase = erase; p.write = write; p.g = gw ? g : nullptr;
    p.state_in = s_in; p.y = y; p.state_out = s_out;
    p.kv_bstride = (int64_t)u * seq;
    p.q_bstride = seq;
    p.stall = 0;
    p.norm = 0;
    p.norm_eps = 0.f;
    p.norm_weight = nullptr;
    return p;
}

// ---------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------
// Decode ticks are short kernels launched back to back (config 5: about 9 us each), so the gap between two
// dependent launches is a large share of a tick.  They are launched with programmatic stream
// serialization: the next tick is scheduled while the previous one runs, and each tick's kernel waits
// (griddepcontrol.wait) for the previous kernel in the stream to complete before it reads anything, so the
// ordering with whatever kernel precedes it is the ordinary stream order.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename TI, typename TG, typename TO, int VEC, int CW, int NP>
int launch_step_cfg(const dc::CoreParams &p, cudaStream_t stream) {
    const dim3 grid((unsigned)(p.batch * p.heads), (unsigned)((p.dv + CW - 1) / CW));
    const size_t smem = dc::step_smem_bytes((int)p.dk, p.u, CW);
    cudaError_t e = launch_pdl(dc::step_kernel<TI, TG, TO, VEC, CW, NP>, grid, dim3(dc::kStepThreads), smem, stream, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

// Multiprocessors of the current device (cached per device).
int sm_count() {
    static int count[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        count[dev] = n;
    }
    return count[dev];
}

// Whether the streaming decode kernel serves this tick: one micro-step, dk = dv = 128, 16-byte-aligned rows.
bool stream_applies(const dc::CoreParams &p, size_t in_size, size_t gate_size) {
    if (p.u != 1 || p.dk != 128 || p.dv != 128) return false;
    if (!aligned(p.state_in, 16) || !aligned(p.state_out, 16) || !aligned(p.q, 16) || !aligned(p.k, 16) ||
        !aligned(p.v, 16))
        return false;
    if ((p.ew != 1 && !aligned(p.erase, 16)) || (p.ww != 1 && !aligned(p.write, 16)) || (p.gw > 1 && !aligned(p.g, 16)))
        return false;
    (void)in_size;
    (void)gate_size;
    return true;
}

template <typename TI, typename TG, typename TO>
int launch_step_stream(const dc::CoreParams &p, cudaStream_t stream) {
    int *status = dc::device_status_ptr();
    if (!status) return cuda_fail(cudaErrorInvalidSymbol);
    auto kern = dc::stream::step_stream_kernel<TI, TG, TO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dc::stream::kSmem);
    if (e != cudaSuccess) return cuda_fail(e);
    const int64_t bh = p.batch * p.heads;
    const unsigned grid = (unsigned)(bh < sm_count() ? bh : sm_count());
    e = launch_pdl(kern, dim3(grid), dim3(dc::stream::kThreads), dc::stream::kSmem, stream, p, status);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

// Below this many (batch, head) pairs a tick is latency-bound and the per-tile kernel's 2 CTAs per head
// balance the SMs better than one streaming CTA per SM walking whole heads (measured on B200: 256 heads
// 7.6 vs 8.7 us per tick; 1024 heads 24.0 vs 21.4 us).
constexpr int64_t kStreamMinHeads = 1024;

template <typename TI, typename TG, typename TO>
int launch_step_typed(const dc::CoreParams &p, cudaStream_t stream, bool allow_stream = true) {
    const bool big = p.batch * p.heads >= kStreamMinHeads || p.stall;
    if (allow_stream && big && stream_applies(p, sizeof(TI), sizeof(TG))) return launch_step_stream<TI, TG, TO>(p, stream);
    const bool vec4 = (p.dv % 4 == 0) && aligned(p.state_in, 16) && aligned(p.state_out, 16);
    if (vec4) {
        if (p.dk <= 128) return launch_step_cfg<TI, TG, TO, 4, 64, 16>(p, stream);
        return launch_step_cfg<TI, TG, TO, 4, 32, 16>(p, stream);
    }
    if (p.dk <= 128) return launch_step_cfg<TI, TG, TO, 1, 16, 16>(p, stream);
    return launch_step_cfg<TI, TG, TO, 1, 8, 16>(p, stream);
}

template <template <typename, typename, typename> class F, typename... A>
int dispatch_types(int32_t in_dt, int32_t gate_dt, int32_t out_dt, A &&...args) {
    using f32 = float;
    using b16 = __nv_bfloat16;
    const int key = in_dt * 4 + gate_dt * 2 + out_dt;
    switch (key) {
        case 0: return F<f32, f32, f32>::run(args...);
        case 1: return F<f32, f32, b16>::run(args...);
        case 2: return F<f32, b16, f32>::run(args...);
        case 3: return F<f32, b16, b16>::run(args...);
        case 4: return F<b16, f32, f32>::run(args...);
        case 5: return F<b16, f32, b16>::run(args...);
        case 6: return F<b16, b16, f32>::run(args...);
        case 7: return F<b16, b16, b16>::run(args...);
    }
    return DC_EUNSUPPORTED_DTYPE;
}

template <typename TI, typename TG, typename TO>
struct StepLauncher {
    static int run(const dc::CoreParams &p, cudaStream_t s, bool allow_stream) {
        return launch_step_typed<TI, TG, TO>(p, s, allow_stream);
    }
};

// ---------------------------------------------------------------------------
// Prefill
// ---------------------------------------------------------------------------
template <typename TI, typename TG, typename TO, int LC>
int launch_simt_cfg(const dc::CoreParams &p, int cw, cudaStream_t stream) {
    const dc::SimtLayout ly((int)p.dk, cw, LC, p.gw);
    const size_t smem = sizeof(float) * (size_t)ly.total;
    auto kern = dc::chunk_simt_kernel<TI, TG, TO, LC>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e);
    const dim3 grid((unsigned)(p.batch * p.heads), (unsigned)((p.dv + cw - 1) / cw));
    kern<<<grid, dc::kSimtThreads, smem, stream>>>(p, cw);
    e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

template <typename TI, typename TG, typename TO>
struct SimtLauncher {
    static int run(const dc::CoreParams &p, cudaStream_t s) {
        if (p.dk <= 128) return launch_simt_cfg<TI, TG, TO, 32>(p, (int)(p.dv < 64 ? p.dv : 64), s);
        return launch_simt_cfg<TI, TG, TO, 16>(p, (int)(p.dv < 32 ? p.dv : 32), s);
    }
};

int validate_chunk(const dc_chunk_args *a) {
    if (!a) return DC_EINVAL_ARG;
    if (a->chunk_len < 1) return DC_EINVAL_ARG;
    if (a->workspace && !aligned(a->workspace, 16)) return DC_EINVAL_ARG;
    return validate_common(a->batch, a->seq, a->heads, a->dk, a->dv, a->n_householder, a->erase_w, a->write_w,
                           a->g_w, a->in_dtype, a->gate_dtype, a->out_dtype, a->scale, a->q, a->k, a->v,
                           a->erase, a->write, a->g, a->state_in, a->y, a->state_out);
}

int validate_step(const dc_step_args *a) {
    if (!a) return DC_EINVAL_ARG;
    return validate_common(a->batch, 1, a->heads, a->dk, a->dv, a->n_householder, a->erase_w, a->write_w, a->g_w,
                           a->in_dtype, a->gate_dtype, a->out_dtype, a->scale, a->q, a->k, a->v, a->erase,
                           a->write, a->g, a->state_in, a->y, a->state_out);
}

}  // namespace

extern "C" {

int dc_version(void) { return 200; }

const char *dc_status_string(int status) {
    switch (status) {
        case DC_OK: return "ok";
        case DC_EINVAL_SHAPE: return "invalid shape";
        case DC_EINVAL_WIDTH: return "gate width must be 1 or the full channel count";
        case DC_EUNSUPPORTED_DTYPE: return "unsupported dtype";
        case DC_EINVAL_ARG: return "invalid argument";
        case DC_EUNSUPPORTED: return "unsupported size (dk > 256 or n_householder > 8)";
        case DC_ECUDA: return "CUDA error";
        case DC_EDEVICE: return "current device is not an sm_100 GPU";
        case DC_EWORKSPACE: return "workspace smaller than dc_chunk_workspace_size";
        case DC_ESCRATCH: return "request needs more scratch than the no-allocation entry point holds";
    }
    return "unknown status";
}

int dc_last_cuda_error(void) { return g_last_cuda_error; }

int dc_device_status(int reset) {
    int st = check_device(nullptr);
    if (st != DC_OK) return -st;
    int value = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&value, dc::g_device_status, sizeof(int));
    if (e == cudaSuccess && reset) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(dc::g_device_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess) return -cuda_fail(e);
    return value;
}

}  // extern "C"

namespace {

dc::CoreParams chunk_params(const dc_chunk_args *a) {
    return make_params(a->batch, a->seq, a->heads, a->dk, a->dv, a->n_householder, a->erase_w, a->write_w, a->g_w,
                       a->scale, a->q, a->k, a->v, a->erase, a->write, a->g, a->state_in, a->y, a->state_out);
}

// The fp32-accurate chunked path (chunk_f32.cuh) takes what the bf16 tensor-core kernels do not.
bool f32_chunked_applies(const dc_chunk_args *a, const dc::CoreParams &p) {
    return !dc::split_applies(p, a->in_dtype, a->flags) && !dc::tc_applies(p, a->in_dtype, a->flags) &&
           dc::f32c::applies(p, a->flags);
}

// The prefill's device workspace: the split path's, the fp32-accurate chunked path's, or none.
uint64_t fwd_workspace_bytes(const dc_chunk_args *a, const dc::CoreParams &p) {
    if (dc::split_applies(p, a->in_dtype, a->flags)) return dc::split_workspace_bytes(p);
    if (f32_chunked_applies(a, p)) return dc::f32c::plan(p).total_bytes;
    return 0;
}

// The chunk kernel a validated call takes: 3 fp32-accurate chunked (workspace), 2 split (workspace),
// 1 fused tensor-core, 0 CUDA-core, or -DC_EWORKSPACE when a workspace is given (or the split path is
// forced) but short.
int chunk_choice_any(const dc_chunk_args *a, const dc::CoreParams &p) {
    if (a->flags & DC_FLAG_RECURRENT) return 0;
    if (dc::split_applies(p, a->in_dtype, a->flags)) {
        if (a->workspace && a->workspace_bytes >= dc::split_workspace_bytes(p)) return 2;
        if (a->workspace || (a->flags & DC_FLAG_FORCE_SPLIT)) return -DC_EWORKSPACE;
    }
    if (dc::tc_applies(p, a->in_dtype, a->flags)) return 1;
    if (f32_chunked_applies(a, p) && a->workspace) {
        return a->workspace_bytes >= dc::f32c::plan(p).total_bytes ? 3 : -DC_EWORKSPACE;
    }
    return 0;
}

// The fp32-accurate chunked prefill: the backward's prep kernel (chunk-parallel, without the arrays only
// the backward reads), then the forward scan: one CTA per (head, 32-column slice) when those fit on the
// device's SMs in one wave (two per SM), else one CTA per head over all columns (fewer, larger warp
// tiles; every chunk operand read once per head).
template <typename TI, typename TG, typename TO>
int launch_chunk_f32_typed(const dc::bwdc::Params &p, int64_t bh, cudaStream_t s) {
    using namespace dc::bwdc;
    const bool wide = bh * p.nslice > 2 * (int64_t)sm_count();
    const size_t sp = kPrepSmemFloats * sizeof(float);
    const size_t ss = (wide ? dc::f32c::kWideSmemFloats : dc::f32c::kScanSmemFloats) * sizeof(float);
    auto scan = wide ? dc::f32c::fwd_scan_wide_kernel<TO> : dc::f32c::fwd_scan_kernel<TO>;
    cudaError_t e = cudaFuncSetAttribute(prep_kernel<TI, TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ss);
    if (e != cudaSuccess) return cuda_fail(e);
    prep_kernel<TI, TG><<<(unsigned)(bh * p.nc), kThreads, sp, s>>>(p);
    scan<<<dim3((unsigned)bh, wide ? 1u : (unsigned)p.nslice), wide ? dc::f32c::kWideThreads : kThreads, ss, s>>>(p);
    e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

int launch_chunk_f32(const dc_chunk_args *a, const dc::CoreParams &f, cudaStream_t s) {
    const dc::f32c::Plan pl = dc::f32c::plan(f);
    dc::bwdc::Params p{};
    p.f = f;
    float *ws = static_cast<float *>(a->workspace);
    p.W = ws;
    p.Kh = p.W + pl.w;
    p.Qp = p.Kh + pl.w;
    p.U = p.Qp + pl.w;
    p.att = p.U + pl.uv;
    p.gl = p.att + pl.sq;
    p.nc = pl.nc;
    p.dkp = pl.dkp;
    p.dvp = pl.dvp;
    p.nslice = pl.nslice;
    const int64_t bh = f.batch * f.heads;
    switch (a->in_dtype * 4 + a->gate_dtype * 2 + a->out_dtype) {
        case 0: return launch_chunk_f32_typed<float, float, float>(p, bh, s);
        case 1: return launch_chunk_f32_typed<float, float, __nv_bfloat16>(p, bh, s);
        case 2: return launch_chunk_f32_typed<float, __nv_bfloat16, float>(p, bh, s);
        case 3: return launch_chunk_f32_typed<float, __nv_bfloat16, __nv_bfloat16>(p, bh, s);
        case 4: return launch_chunk_f32_typed<__nv_bfloat16, float, float>(p, bh, s);
        case 5: return launch_chunk_f32_typed<__nv_bfloat16, float, __nv_bfloat16>(p, bh, s);
        case 6: return launch_chunk_f32_typed<__nv_bfloat16, __nv_bfloat16, float>(p, bh, s);
        case 7: return launch_chunk_f32_typed<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(p, bh, s);
        default: return DC_EUNSUPPORTED_DTYPE;
    }
}

// As above; the stall test hook is taken by the tensor-core kernel only.
int chunk_choice(const dc_chunk_args *a, const dc::CoreParams &p) {
    const int choice = chunk_choice_any(a, p);
    if ((a->flags & DC_FLAG_TEST_STALL) && choice != 1) return -DC_EINVAL_ARG;
    return choice;
}

}  // namespace

extern "C" {

int dc_chunk_kernel_choice(const dc_chunk_args *a) {
    const int st = validate_chunk(a);
    if (st != DC_OK) return -st;
    return chunk_choice(a, chunk_params(a));
}

uint64_t dc_chunk_workspace_size(const dc_chunk_args *a) {
    if (validate_chunk(a) != DC_OK) return 0;
    const dc::CoreParams p = chunk_params(a);
    return fwd_workspace_bytes(a, p);
}

int dc_chunk_launches(const dc_chunk_args *a) {
    const int st = validate_chunk(a);
    if (st != DC_OK) return -st;
    if (a->batch == 0 || a->heads == 0) return 0;
    const int choice = chunk_choice(a, chunk_params(a));
    if (choice < 0) return choice;
    if (a->flags & DC_FLAG_RECURRENT) return (int)a->seq;
    return choice >= 2 ? 2 : 1;
}

// DeltaPath::Recurrent: the fused tick walks the sequence in place, one launch
// per token, reading each token's rows through the batch strides (no copies).
static int run_recurrent(const dc_chunk_args *a, cudaStream_t s) {
    const size_t isz = a->in_dtype == DC_F32 ? 4 : 2, gsz = a->gate_dtype == DC_F32 ? 4 : 2;
    const size_t osz = a->out_dtype == DC_F32 ? 4 : 2;
    const int64_t H = a->heads, u = a->n_householder;
    for (int64_t t = 0; t < a->seq; ++t) {
        const char *q = static_cast<const char *>(a->q) + (size_t)(t * H * a->dk) * isz;
        const char *k = static_cast<const char *>(a->k) + (size_t)(t * u * H * a->dk) * isz;
        const char *v = static_cast<const char *>(a->v) + (size_t)(t * u * H * a->dv) * isz;
        const char *e = static_cast<const char *>(a->erase) + (size_t)(t * u * H * a->erase_w) * gsz;
        const char *w = static_cast<const char *>(a->write) + (size_t)(t * u * H * a->write_w) * gsz;
        const char *g = a->g_w ? static_cast<const char *>(a->g) + (size_t)(t * H * a->g_w) * gsz : nullptr;
        char *y = static_cast<char *>(a->y) + (size_t)(t * H * a->dv) * osz;
        dc::CoreParams p = make_params(a->batch, 1, a->heads, a->dk, a->dv, a->n_householder, a->erase_w, a->write_w,
                                       a->g_w, a->scale, q, k, v, e, w, g, t == 0 ? a->state_in : a->state_out, y,
                                       a->state_out);
        p.kv_bstride = a->seq * u;
        p.q_bstride = a->seq;
        const int st = dispatch_types<StepLauncher>(a->in_dtype, a->gate_dtype, a->out_dtype, p, s, true);
        if (st != DC_OK) return st;
    }
    return DC_OK;
}

}  // extern "C"

namespace {

// dc_chunk_fwd after validation and the device check.
int chunk_fwd_launch(const dc_chunk_args *a, cudaStream_t s) {
    const dc::CoreParams p = chunk_params(a);
    const int choice = chunk_choice(a, p);
    if (choice < 0) return -choice;
    if (a->flags & DC_FLAG_RECURRENT) return run_recurrent(a, s);
    int st;
    if (choice == 3) return launch_chunk_f32(a, p, s);
    if (choice == 2) {
        st = dc::launch_chunk_split(p, a->gate_dtype, a->out_dtype, a->workspace, s);
        if (st == DC_ECUDA) g_last_cuda_error = dc::tc_last_error();
        return st;
    }
    if (choice == 1) {
        dc::CoreParams pt = p;
        pt.stall = (a->flags & DC_FLAG_TEST_STALL) ? 1 : 0;
        st = dc::launch_chunk_tc(pt, a->gate_dtype, a->out_dtype, s);
        if (st == DC_ECUDA) g_last_cuda_error = dc::tc_last_error();
        return st;
    }
    return dispatch_types<SimtLauncher>(a->in_dtype, a->gate_dtype, a->out_dtype, p, s);
}

}  // namespace

extern "C" {

int dc_chunk_fwd(const dc_chunk_args *a, dc_stream_t stream) {
    int st = validate_chunk(a);
    if (st != DC_OK || a->batch == 0 || a->heads == 0) return st;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    return chunk_fwd_launch(a, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_chunk_fwd_noalloc: the two-kernel path over a fixed device array, for
// callers that cannot allocate device memory (an engine whose memory belongs
// to its own pool and hands an FFI call no raw scratch; a serving loop where
// a cudaMalloc, which may synchronise the device, is not allowed).
// ---------------------------------------------------------------------------
namespace {

// The scratch: every GPU that loads this library holds it until exit.  All
// calls share it; nothing in it needs to start at zero (the prep kernel
// writes every element the scan kernel reads).
static __device__ __align__(256) uint8_t g_noalloc_scratch[DC_NOALLOC_SCRATCH_BYTES];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory:
// its device address is looked up with the device current, once per device and
// context (a cudaDeviceReset gives the device a new context, and the address is
// looked up again under it).
void *noalloc_scratch(int dev, int *status) {
    static dc::SymbolCache cache;
    if (dev < 0 || dev >= 64) {
        *status = DC_EUNSUPPORTED;
        return nullptr;
    }
    int err = 0;
    void *ptr = cache.get(reinterpret_cast<const void *>(&g_noalloc_scratch), &err);
    if (!ptr) *status = cuda_fail((cudaError_t)err);
    return ptr;
}

}  // namespace

extern "C" {

int dc_chunk_fwd_noalloc(const dc_chunk_args *a, dc_stream_t stream) {
    int st = validate_chunk(a);
    if (st != DC_OK || a->batch == 0 || a->heads == 0) return st;
    if (a->flags & (DC_FLAG_FORCE_SIMT | DC_FLAG_RECURRENT | DC_FLAG_TEST_STALL)) return DC_EINVAL_ARG;
    int dev = 0;
    st = check_device(&dev);
    if (st != DC_OK) return st;
    const dc::CoreParams p = chunk_params(a);
    if (!dc::split_applies(p, a->in_dtype, DC_FLAG_FORCE_SPLIT)) return DC_EUNSUPPORTED;
    if (dc::split_workspace_bytes(p) > DC_NOALLOC_SCRATCH_BYTES) return DC_ESCRATCH;
    void *scratch = noalloc_scratch(dev, &st);
    if (!scratch) return st;
    st = dc::launch_chunk_split(p, a->gate_dtype, a->out_dtype, scratch, reinterpret_cast<cudaStream_t>(stream));
    if (st == DC_ECUDA) g_last_cuda_error = dc::tc_last_error();
    return st;
}

int dc_step(const dc_step_args *a, dc_stream_t stream) {
    int st = validate_step(a);
    if (st != DC_OK || a->batch == 0 || a->heads == 0) return st;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    dc::CoreParams p = make_params(a->batch, 1, a->heads, a->dk, a->dv, a->n_householder, a->erase_w, a->write_w,
                                   a->g_w, a->scale, a->q, a->k, a->v, a->erase, a->write, a->g, a->state_in, a->y,
                                   a->state_out);
    const bool allow_stream = (a->flags & DC_FLAG_FORCE_SIMT) == 0;
    if (a->flags & DC_FLAG_TEST_STALL) {  // the streaming kernel is the one that takes the hook
        const size_t is = a->in_dtype == DC_F32 ? 4 : 2, gs = a->gate_dtype == DC_F32 ? 4 : 2;
        if (!allow_stream || !stream_applies(p, is, gs)) return DC_EINVAL_ARG;
        p.stall = 1;
    }
    return dispatch_types<StepLauncher>(a->in_dtype, a->gate_dtype, a->out_dtype, p,
                                        reinterpret_cast<cudaStream_t>(stream), allow_stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_chunk_fwd_host: the prefill from host memory, with the PCIe transfers of
// one slice of sequences overlapping the kernels of the previous one and the
// copies back of the one before (three streams, two device slots).
// ---------------------------------------------------------------------------
namespace {

constexpr int kHostSlices = 8;  // the batch is cut into at most this many slices of whole sequences

struct HostPlan {
    int64_t per_slice;   // sequences per slice
    size_t seq_bytes[9]; // bytes of one sequence: q, k, v, erase, write, g, state_in, y, state_out
    size_t off[9];       // offsets of those regions inside a slot
    size_t slot;         // bytes of one slot
    size_t ws;           // the two-kernel path's workspace for one slice (kernels run in order: one is enough)
    size_t total;
};

size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

HostPlan host_plan(const dc_chunk_args *a) {
    HostPlan hp{};
    hp.per_slice = (a->batch + kHostSlices - 1) / kHostSlices;
    const size_t is = dtype_size(a->in_dtype), gs = dtype_size(a->gate_dtype), os = dtype_size(a->out_dtype);
    const size_t s = (size_t)a->seq, su = s * (size_t)a->n_householder, h = (size_t)a->heads;
    const size_t dk = (size_t)a->dk, dv = (size_t)a->dv;
    const size_t per[9] = {s * h * dk * is, su * h * dk * is, su * h * dv * is,
                           su * h * (size_t)a->erase_w * gs, su * h * (size_t)a->write_w * gs,
                           a->g_w ? s * h * (size_t)a->g_w * gs : 0, h * dk * dv * 4, s * h * dv * os, h * dk * dv * 4};
    size_t o = 0;
    for (int i = 0; i < 9; ++i) {
        hp.seq_bytes[i] = per[i];
        hp.off[i] = o;
        o += round256(per[i] * (size_t)hp.per_slice);
    }
    hp.slot = o;
    // The slice's kernel choice is taken on 256-aligned device pointers: stand-ins suffice for the size.
    dc_chunk_args sl = *a;
    sl.batch = a->batch < hp.per_slice ? a->batch : hp.per_slice;
    const void *fake = reinterpret_cast<const void *>((uintptr_t)4096);
    sl.q = sl.k = sl.v = sl.erase = sl.write = fake;
    sl.g = a->g_w ? fake : nullptr;
    sl.state_in = sl.state_out = reinterpret_cast<float *>((uintptr_t)8192);
    sl.y = reinterpret_cast<void *>((uintptr_t)12288);
    const dc::CoreParams p = chunk_params(&sl);
    hp.ws = round256(fwd_workspace_bytes(&sl, p));
    hp.total = 2 * hp.slot + hp.ws;
    return hp;
}

// Streams and events of one call, released when it returns (CUDA defers the release until their work is done).
struct HostStreams {
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t start = nullptr, up_done[2] = {}, compute_done[2] = {}, down_done[2] = {};
    ~HostStreams() {
        for (cudaEvent_t e : {start, up_done[0], up_done[1], compute_done[0], compute_done[1], down_done[0], down_done[1]})
            if (e) cudaEventDestroy(e);
        if (up) cudaStreamDestroy(up);
        if (down) cudaStreamDestroy(down);
    }
    cudaError_t create() {
        cudaError_t e = cudaStreamCreateWithFlags(&up, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&down, cudaStreamNonBlocking);
        for (cudaEvent_t *ev : {&start, &up_done[0], &up_done[1], &compute_done[0], &compute_done[1], &down_done[0],
                                &down_done[1]})
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
        return e;
    }
};

}  // namespace

extern "C" {

uint64_t dc_chunk_fwd_host_scratch_size(const dc_chunk_args *a) {
    if (validate_chunk(a) != DC_OK || a->batch == 0 || a->heads == 0) return 0;
    return host_plan(a).total;
}

int dc_chunk_fwd_host(const dc_chunk_args *a, void *scratch, uint64_t scratch_bytes, dc_stream_t stream) {
    int st = validate_chunk(a);
    if (st != DC_OK || a->batch == 0 || a->heads == 0) return st;
    if (a->flags & DC_FLAG_TEST_STALL) return DC_EINVAL_ARG;
    if (!scratch || !aligned(scratch, 256)) return DC_EINVAL_ARG;
    const HostPlan hp = host_plan(a);
    if (scratch_bytes < hp.total) return DC_EWORKSPACE;
    st = check_device(nullptr);
    if (st != DC_OK) return st;

    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    HostStreams hs;
    cudaError_t e = hs.create();
    // Nothing starts before the work already queued on the caller's stream (it may still use the scratch).
    if (e == cudaSuccess) e = cudaEventRecord(hs.start, cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.up, hs.start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.down, hs.start, 0);
    if (e != cudaSuccess) return cuda_fail(e);

    // On an error after copies were queued: the caller's stream waits for everything already on the two
    // internal streams, so that neither the scratch nor the host buffers are reused under a copy in flight.
    auto fail_drained = [&](int status) {
        if (cudaEventRecord(hs.up_done[0], hs.up) == cudaSuccess) cudaStreamWaitEvent(cs, hs.up_done[0], 0);
        if (cudaEventRecord(hs.down_done[0], hs.down) == cudaSuccess) cudaStreamWaitEvent(cs, hs.down_done[0], 0);
        return status;
    };
    const void *src[7] = {a->q, a->k, a->v, a->erase, a->write, a->g, a->state_in};
    void *dst_host[2] = {a->y, a->state_out};
    char *const base = static_cast<char *>(scratch);
    const int64_t nslices = (a->batch + hp.per_slice - 1) / hp.per_slice;
    for (int64_t i = 0; i < nslices; ++i) {
        const int slot = (int)(i & 1);
        const int64_t b0 = i * hp.per_slice;
        const int64_t nb = (a->batch - b0) < hp.per_slice ? (a->batch - b0) : hp.per_slice;
        char *sb = base + (size_t)slot * hp.slot;
        dc_chunk_args sl = *a;
        sl.batch = nb;
        sl.q = sb + hp.off[0];
        sl.k = sb + hp.off[1];
        sl.v = sb + hp.off[2];
        sl.erase = sb + hp.off[3];
        sl.write = sb + hp.off[4];
        sl.g = a->g_w ? sb + hp.off[5] : nullptr;
        sl.state_in = reinterpret_cast<const float *>(sb + hp.off[6]);
        sl.y = sb + hp.off[7];
        sl.state_out = reinterpret_cast<float *>(sb + hp.off[8]);
        sl.workspace = hp.ws ? base + 2 * hp.slot : nullptr;
        sl.workspace_bytes = hp.ws;
        const void *dst[7] = {sl.q, sl.k, sl.v, sl.erase, sl.write, sl.g, sl.state_in};

        // in: once the kernels of slice i-2 (the slot's last reader) are done
        if (i >= 2) e = cudaStreamWaitEvent(hs.up, hs.compute_done[slot], 0);
        for (int r = 0; r < 7 && e == cudaSuccess; ++r)
            if (hp.seq_bytes[r])
                e = cudaMemcpyAsync(const_cast<void *>(dst[r]), static_cast<const char *>(src[r]) + b0 * hp.seq_bytes[r],
                                    (size_t)nb * hp.seq_bytes[r], cudaMemcpyHostToDevice, hs.up);
        if (e == cudaSuccess) e = cudaEventRecord(hs.up_done[slot], hs.up);
        // compute on the caller's stream: after the slice landed and slice i-2's results left the slot
        if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, hs.up_done[slot], 0);
        if (e == cudaSuccess && i >= 2) e = cudaStreamWaitEvent(cs, hs.down_done[slot], 0);
        if (e != cudaSuccess) return fail_drained(cuda_fail(e));
        st = chunk_fwd_launch(&sl, cs);
        if (st != DC_OK) return fail_drained(st);
        e = cudaEventRecord(hs.compute_done[slot], cs);
        // out
        if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.down, hs.compute_done[slot], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<char *>(dst_host[0]) + b0 * hp.seq_bytes[7], sl.y, (size_t)nb * hp.seq_bytes[7],
                                cudaMemcpyDeviceToHost, hs.down);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<char *>(dst_host[1]) + b0 * hp.seq_bytes[8], sl.state_out,
                                (size_t)nb * hp.seq_bytes[8], cudaMemcpyDeviceToHost, hs.down);
        if (e == cudaSuccess) e = cudaEventRecord(hs.down_done[slot], hs.down);
        if (e != cudaSuccess) return fail_drained(cuda_fail(e));
    }
    // The caller's stream drains only after the last results reached the host.
    e = cudaStreamWaitEvent(cs, hs.down_done[0], 0);
    if (e == cudaSuccess && nslices > 1) e = cudaStreamWaitEvent(cs, hs.down_done[1], 0);
    return e == cudaSuccess ? DC_OK : fail_drained(cuda_fail(e));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_chunk_bwd: the backward, chunk by chunk (bwd_chunk.cuh) for a log-decay per head or none, token by
// token (bwd_recurrent.cuh) for per-channel log-decays or with DC_FLAG_RECURRENT.
// ---------------------------------------------------------------------------
namespace {

int validate_bwd(const dc_chunk_bwd_args *a) {
    if (!a) return DC_EINVAL_ARG;
    const dc_chunk_args &f = a->fwd;
    // The forward's own checks, with stand-ins for the outputs this call does not use.
    dc_chunk_args chk = f;
    chk.y = reinterpret_cast<void *>((uintptr_t)1 << 12);
    chk.state_out = reinterpret_cast<float *>((uintptr_t)1 << 13);
    chk.out_dtype = DC_F32;
    chk.workspace = nullptr;
    chk.workspace_bytes = 0;
    chk.flags = 0;
    int st = validate_chunk(&chk);
    if (st != DC_OK) return st;
    if (f.dk > dc::bwd::kMaxD || f.dv > dc::bwd::kMaxD) return DC_EUNSUPPORTED;
    if (!a->d_y || !a->d_q || !a->d_k || !a->d_v || !a->d_erase || !a->d_write || !a->d_state) return DC_EINVAL_ARG;
    if (f.g_w > 0 && !a->d_g) return DC_EINVAL_ARG;
    if (a->workspace && !aligned(a->workspace, 16)) return DC_EINVAL_ARG;
    return DC_OK;
}

// The backward's workspace: checkpoints and the replay scratch per (batch, head, slice), then, with more
// than one value slice, the slices' partial sums of the column-summed gradients.
struct BwdPlan {
    int32_t nslice;
    int64_t nblk;
    uint64_t ckpt, scratch, pq, pk, pe, pg, pw1, total;  // element counts (floats) / total bytes
};

BwdPlan bwd_plan(const dc_chunk_args &f) {
    BwdPlan pl{};
    const int64_t n = f.seq * f.n_householder, bh = f.batch * f.heads;
    pl.nslice = (int32_t)((f.dv + dc::bwd::kSlice - 1) / dc::bwd::kSlice);
    pl.nblk = (n + dc::bwd::kBlk - 1) / dc::bwd::kBlk;
    const uint64_t st = (uint64_t)f.dk * dc::bwd::kSlice;
    pl.ckpt = (uint64_t)(bh * pl.nslice * pl.nblk) * st;
    pl.scratch = (uint64_t)(bh * pl.nslice * dc::bwd::kBlk) * st;
    if (pl.nslice > 1) {
        pl.pq = (uint64_t)(f.batch * f.seq * f.heads * f.dk);
        pl.pk = (uint64_t)(f.batch * n * f.heads * f.dk);
        pl.pe = (uint64_t)(f.batch * n * f.heads * f.erase_w);
        pl.pg = (uint64_t)(f.batch * f.seq * f.heads * f.g_w);
        pl.pw1 = f.write_w == 1 ? (uint64_t)(f.batch * n * f.heads) : 0;
    }
    pl.total = 4ull * (pl.ckpt + pl.scratch + (uint64_t)pl.nslice * (pl.pq + pl.pk + pl.pe + pl.pg + pl.pw1));
    return pl;
}

// The chunked backward's workspace (floats; every region a multiple of 4 floats, so 16-byte aligned).
struct ChunkBwdPlan {
    int64_t nc, nch;
    int32_t dkp, dvp, nslice;
    uint64_t w, uv, sq, gl, st, total;  // element counts per array / total bytes
};

bool chunk_bwd_applies(const dc_chunk_args &f) { return f.g_w <= 1 && (f.flags & DC_FLAG_RECURRENT) == 0; }

ChunkBwdPlan chunk_bwd_plan(const dc_chunk_args &f) {
    using namespace dc::bwdc;
    ChunkBwdPlan pl{};
    const int64_t n = f.seq * f.n_householder;
    pl.nc = (n + kBL - 1) / kBL;
    pl.nch = f.batch * f.heads * pl.nc;
    pl.dkp = (int32_t)((f.dk + 7) / 8 * 8);
    pl.dvp = (int32_t)((f.dv + 7) / 8 * 8);
    pl.nslice = (pl.dvp + kSlice - 1) / kSlice;
    pl.w = (uint64_t)pl.nch * kBL * pl.dkp;
    pl.uv = (uint64_t)pl.nch * kBL * pl.dvp;
    pl.sq = (uint64_t)pl.nch * kBL * kBL;
    pl.gl = ((uint64_t)pl.nch + 3) / 4 * 4;
    pl.st = (uint64_t)pl.nch * pl.dvp * pl.dkp;
    pl.total = 4ull * (3 * pl.w + 3 * pl.uv + 3 * pl.sq + pl.gl + 2 * pl.st);
    return pl;
}

uint64_t bwd_workspace_bytes(const dc_chunk_args &f) {
    return chunk_bwd_applies(f) ? chunk_bwd_plan(f).total : bwd_plan(f).total;
}

template <typename TI, typename TG>
int launch_chunk_bwd_typed(const dc::bwdc::Params &p, int64_t bh, cudaStream_t s) {
    using namespace dc::bwdc;
    const int64_t nch = bh * p.nc;
    // The scan: one CTA per (head, 32-column slice) when those fit in one wave at two per SM, else one
    // 16-warp CTA per head over every column (the same results bit for bit).
    const bool wide = bh * p.nslice > 2 * (int64_t)sm_count();
    const size_t sp = kPrepSmemFloats * sizeof(float),
                 ss = (wide ? kScanWideSmemFloats : kScanSmemFloats) * sizeof(float),
                 sg = kGradSmemFloats * sizeof(float);
    auto scan = wide ? scan_wide_kernel : scan_kernel;
    cudaError_t e = cudaFuncSetAttribute(prep_kernel<TI, TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ss);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(grad_kernel<TI, TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sg);
    if (e != cudaSuccess) return cuda_fail(e);
    prep_kernel<TI, TG><<<(unsigned)nch, kThreads, sp, s>>>(p);
    scan<<<dim3((unsigned)bh, wide ? 1u : (unsigned)p.nslice), wide ? kWideThreads : kThreads, ss, s>>>(p);
    grad_kernel<TI, TG><<<(unsigned)nch, kThreads, sg, s>>>(p);
    e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

int run_chunk_bwd(const dc_chunk_bwd_args *a, cudaStream_t s) {
    const dc_chunk_args &f = a->fwd;
    const ChunkBwdPlan pl = chunk_bwd_plan(f);
    if (pl.nch > 0x7fffffffLL || f.batch * f.heads > 0x7fffffffLL) return DC_EUNSUPPORTED;
    dc::bwdc::Params p{};
    p.f = chunk_params(&f);
    p.dy = a->d_y;
    p.dS_final = a->d_state_final;
    p.dq = a->d_q;
    p.dk = a->d_k;
    p.dv = a->d_v;
    p.de = a->d_erase;
    p.dw = a->d_write;
    p.dg = a->d_g;
    p.dS0 = a->d_state;
    float *ws = static_cast<float *>(a->workspace);
    p.W = ws;
    p.Kh = p.W + pl.w;
    p.Qp = p.Kh + pl.w;
    p.U = p.Qp + pl.w;
    p.Vp = p.U + pl.uv;
    p.dVp = p.Vp + pl.uv;
    p.att = p.dVp + pl.uv;
    p.T = p.att + pl.sq;
    p.A = p.T + pl.sq;
    p.gl = p.A + pl.sq;
    p.ST = p.gl + pl.gl;
    p.dSnT = p.ST + pl.st;
    p.nc = pl.nc;
    p.dkp = pl.dkp;
    p.dvp = pl.dvp;
    p.nslice = pl.nslice;
    p.dy_vec = (f.dv % 4 == 0 && aligned(a->d_y, 16)) ? 1 : 0;
    const int64_t bh = f.batch * f.heads;
    switch (f.in_dtype * 2 + f.gate_dtype) {
        case 0: return launch_chunk_bwd_typed<float, float>(p, bh, s);
        case 1: return launch_chunk_bwd_typed<float, __nv_bfloat16>(p, bh, s);
        case 2: return launch_chunk_bwd_typed<__nv_bfloat16, float>(p, bh, s);
        case 3: return launch_chunk_bwd_typed<__nv_bfloat16, __nv_bfloat16>(p, bh, s);
        default: return DC_EUNSUPPORTED_DTYPE;
    }
}

template <typename TI, typename TG>
int launch_bwd_typed(const dc::bwd::Params &p, cudaStream_t s) {
    const dc::bwd::Layout L((int)p.f.dk);
    const size_t smem = (size_t)L.total * sizeof(float);
    auto kern = dc::bwd::bwd_recurrent_kernel<TI, TG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e);
    kern<<<dim3((unsigned)(p.f.batch * p.f.heads), (unsigned)p.nslice), dc::bwd::kThreads, smem, s>>>(p);
    e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

}  // namespace

extern "C" {

uint64_t dc_chunk_bwd_workspace_size(const dc_chunk_bwd_args *a) {
    if (validate_bwd(a) != DC_OK) return 0;
    return bwd_workspace_bytes(a->fwd);
}

int dc_chunk_bwd(const dc_chunk_bwd_args *a, dc_stream_t stream) {
    int st = validate_bwd(a);
    if (st != DC_OK) return st;
    const dc_chunk_args &f = a->fwd;
    if (f.batch == 0 || f.heads == 0) return DC_OK;
    if (!a->workspace || a->workspace_bytes < bwd_workspace_bytes(f)) return DC_EWORKSPACE;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    if (chunk_bwd_applies(f)) return run_chunk_bwd(a, reinterpret_cast<cudaStream_t>(stream));
    const BwdPlan pl = bwd_plan(f);
    dc::bwd::Params p{};
    p.f = chunk_params(&f);
    p.dy = a->d_y;
    p.dS_final = a->d_state_final;
    p.dv = a->d_v;
    p.dw_full = f.write_w == 1 ? nullptr : a->d_write;
    p.dS0 = a->d_state;
    p.nblk = pl.nblk;
    p.nslice = pl.nslice;
    float *ws = static_cast<float *>(a->workspace);
    p.ckpt = ws;
    p.scratch = ws + pl.ckpt;
    float *part = p.scratch + pl.scratch;
    if (pl.nslice > 1) {  // column-summed gradients go to per-slice partials first
        p.dq = part;
        p.dk = p.dq + pl.nslice * pl.pq;
        p.de = p.dk + pl.nslice * pl.pk;
        p.dg = p.de + pl.nslice * pl.pe;
        p.dw1 = f.write_w == 1 ? p.dg + pl.nslice * pl.pg : nullptr;
        p.sq = (int64_t)pl.pq;
        p.sk = (int64_t)pl.pk;
        p.se = (int64_t)pl.pe;
        p.sg = (int64_t)pl.pg;
        p.sw1 = (int64_t)pl.pw1;
    } else {
        p.dq = a->d_q;
        p.dk = a->d_k;
        p.de = a->d_erase;
        p.dg = a->d_g;
        p.dw1 = f.write_w == 1 ? a->d_write : nullptr;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int key = f.in_dtype * 2 + f.gate_dtype;
    switch (key) {
        case 0: st = launch_bwd_typed<float, float>(p, s); break;
        case 1: st = launch_bwd_typed<float, __nv_bfloat16>(p, s); break;
        case 2: st = launch_bwd_typed<__nv_bfloat16, float>(p, s); break;
        case 3: st = launch_bwd_typed<__nv_bfloat16, __nv_bfloat16>(p, s); break;
        default: return DC_EUNSUPPORTED_DTYPE;
    }
    if (st != DC_OK || pl.nslice == 1) return st;
    // add the slices' partial sums up (in slice order: deterministic)
    auto reduce = [&](const float *src, uint64_t n, float *dst) -> int {
        if (!n) return DC_OK;
        const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
        dc::bwd::reduce_partials<<<blocks, 256, 0, s>>>(src, (int64_t)n, pl.nslice, dst, (int64_t)n);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? DC_OK : cuda_fail(e);
    };
    if ((st = reduce(p.dq, pl.pq, a->d_q)) != DC_OK) return st;
    if ((st = reduce(p.dk, pl.pk, a->d_k)) != DC_OK) return st;
    if ((st = reduce(p.de, pl.pe, a->d_erase)) != DC_OK) return st;
    if (f.g_w > 0 && (st = reduce(p.dg, pl.pg, a->d_g)) != DC_OK) return st;
    if (f.write_w == 1 && (st = reduce(p.dw1, pl.pw1, a->d_write)) != DC_OK) return st;
    return DC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_out_norm: the per-head output normalisation (out_norm.cuh).
// ---------------------------------------------------------------------------
namespace {

int validate_out_norm(const dc_out_norm_args *a) {
    if (!a) return DC_EINVAL_ARG;
    if (a->rows < 0 || a->dv < 1) return DC_EINVAL_SHAPE;
    if (a->dv > 32 * dc::onorm::kMaxPer) return DC_EUNSUPPORTED;
    if (!(a->eps >= 0.f) || !isfinite(a->eps)) return DC_EINVAL_ARG;
    if ((a->in_dtype != DC_F32 && a->in_dtype != DC_BF16) || (a->out_dtype != DC_F32 && a->out_dtype != DC_BF16))
        return DC_EUNSUPPORTED_DTYPE;
    if (a->rows > 0 && (!a->y || !a->weight || !a->out)) return DC_EINVAL_ARG;
    return DC_OK;
}

template <typename TI, typename TO>
int launch_out_norm(const dc::onorm::Params &p, cudaStream_t s) {
    using namespace dc::onorm;
    const int64_t cap = (int64_t)sm_count() * 16;  // grid-stride beyond 16 CTAs per SM of the current device
    auto grid = [&](int64_t rows_per_cta) {
        const int64_t blocks = (p.rows + rows_per_cta - 1) / rows_per_cta;
        return (unsigned)(blocks < cap ? blocks : cap);
    };
    // 16-byte rows: a power-of-two number of 16-byte chunks per row, every row start 16-byte aligned
    constexpr int64_t vec = 16 / sizeof(TI);
    const int64_t lpr = p.dv / vec;
    const bool rows16 = p.dv % vec == 0 && (lpr & (lpr - 1)) == 0 && lpr >= 4 && lpr <= 32 &&
                        aligned(p.y, 16) && aligned(p.out, 16) && (!p.gate || aligned(p.gate, 16)) &&
                        (p.dv * (int64_t)sizeof(TO)) % 16 == 0;
    if (rows16) {
        const int64_t rows_per_cta = (kThreads / 32) * (32 / lpr) * slots_for<TI>();
        switch (lpr) {
            case 4: out_norm_vec_kernel<TI, TO, 4><<<grid(rows_per_cta), kThreads, 0, s>>>(p); break;
            case 8: out_norm_vec_kernel<TI, TO, 8><<<grid(rows_per_cta), kThreads, 0, s>>>(p); break;
            case 16: out_norm_vec_kernel<TI, TO, 16><<<grid(rows_per_cta), kThreads, 0, s>>>(p); break;
            default: out_norm_vec_kernel<TI, TO, 32><<<grid(rows_per_cta), kThreads, 0, s>>>(p); break;
        }
    } else if (p.dv <= 128) {
        out_norm_kernel<TI, TO, 4><<<grid((kThreads / 32) * kRowsPerWarp), kThreads, 0, s>>>(p);
    } else {
        out_norm_kernel<TI, TO, kMaxPer><<<grid((kThreads / 32) * kRowsPerWarp), kThreads, 0, s>>>(p);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

}  // namespace

extern "C" {

int dc_out_norm(const dc_out_norm_args *a, dc_stream_t stream) {
    int st = validate_out_norm(a);
    if (st != DC_OK) return st;
    if (a->rows == 0) return DC_OK;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    dc::onorm::Params p{};
    p.rows = a->rows;
    p.dv = (int32_t)a->dv;
    p.eps = a->eps;
    p.y = a->y;
    p.gate = a->gate;
    p.weight = a->weight;
    p.out = a->out;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (a->in_dtype * 2 + a->out_dtype) {
        case 0: return launch_out_norm<float, float>(p, s);
        case 1: return launch_out_norm<float, __nv_bfloat16>(p, s);
        case 2: return launch_out_norm<__nv_bfloat16, float>(p, s);
        default: return launch_out_norm<__nv_bfloat16, __nv_bfloat16>(p, s);
    }
}

// The checks of dc_chunk_fwd_out_norm and its query: the prefill's, then the norm's against it.
static int validate_chunk_norm(const dc_chunk_args *a, const dc_out_norm_args *n) {
    const int st = validate_chunk(a);
    if (st != DC_OK) return st;
    if (!n || n->y || n->out) return DC_EINVAL_ARG;  // the normalised rows replace y in a->y
    if (!(n->eps >= 0.f) || !isfinite(n->eps)) return DC_EINVAL_ARG;
    if (n->dv != a->dv || n->rows != a->batch * a->seq * a->heads) return DC_EINVAL_SHAPE;
    if (n->out_dtype != a->out_dtype || (n->gate && n->in_dtype != a->out_dtype)) return DC_EUNSUPPORTED_DTYPE;
    if (a->dv > 32 * dc::onorm::kMaxPer) return DC_EUNSUPPORTED;
    if (a->batch > 0 && a->heads > 0 && !n->weight) return DC_EINVAL_ARG;
    return DC_OK;
}

// The prefill with the output norm after it.  Fused into the tensor-core kernel's read-out for the plain
// norm; otherwise dc_chunk_fwd, then dc_out_norm in place on y.
int dc_chunk_fwd_out_norm(const dc_chunk_args *a, const dc_out_norm_args *n, dc_stream_t stream) {
    int st = validate_chunk_norm(a, n);
    if (st != DC_OK) return st;
    if (a->batch == 0 || a->heads == 0) return DC_OK;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    dc::CoreParams p = chunk_params(a);
    const int choice = chunk_choice(a, p);
    if (choice < 0) return -choice;
    if (choice == 1 && !n->gate && !(a->flags & DC_FLAG_RECURRENT)) {
        p.stall = (a->flags & DC_FLAG_TEST_STALL) ? 1 : 0;
        p.norm = 1;
        p.norm_eps = n->eps;
        p.norm_weight = n->weight;
        st = dc::launch_chunk_tc(p, a->gate_dtype, a->out_dtype, s);
        if (st == DC_ECUDA) g_last_cuda_error = dc::tc_last_error();
        return st;
    }
    st = chunk_fwd_launch(a, s);
    if (st != DC_OK) return st;
    dc_out_norm_args m = *n;
    m.in_dtype = a->out_dtype;
    m.y = a->y;
    m.out = a->y;
    return dc_out_norm(&m, stream);
}

int dc_chunk_fwd_out_norm_fused(const dc_chunk_args *a, const dc_out_norm_args *n) {
    const int st = validate_chunk_norm(a, n);
    if (st != DC_OK) return -st;
    const int choice = chunk_choice(a, chunk_params(a));
    if (choice < 0) return choice;
    return (choice == 1 && !n->gate && !(a->flags & DC_FLAG_RECURRENT)) ? 1 : 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_qkv_prologue: the front-end after the input projection (prologue.cuh).
// ---------------------------------------------------------------------------
namespace {

int validate_prologue(const dc_qkv_prologue_args *a) {
    if (!a) return DC_EINVAL_ARG;
    if (a->batch < 1 || a->seq < 1 || a->heads < 1 || a->dk < 1 || a->dv < 1 || a->n_householder < 1)
        return DC_EINVAL_SHAPE;
    if (a->conv_kernel < 1) return DC_EINVAL_ARG;
    if (a->conv_kernel > dc::pro::kMaxK || a->dk > dc::pro::kThreads || a->dv > dc::pro::kThreads)
        return DC_EUNSUPPORTED;
    if (a->batch > 65535 || (a->seq + dc::pro::kTile - 1) / dc::pro::kTile > 65535) return DC_EUNSUPPORTED;
    if ((a->in_dtype != DC_F32 && a->in_dtype != DC_BF16) || (a->out_dtype != DC_F32 && a->out_dtype != DC_BF16))
        return DC_EUNSUPPORTED_DTYPE;
    if (a->flags & ~(DC_PROLOGUE_CONV_SILU | DC_PROLOGUE_QK_SILU | DC_PROLOGUE_L2)) return DC_EINVAL_ARG;
    const int64_t channels = a->heads * a->dk * (1 + a->n_householder) + a->n_householder * a->heads * a->dv;
    if (a->x_stride < channels) return DC_EINVAL_SHAPE;
    if (!a->x || !a->conv_weight || !a->q || !a->k || !a->v) return DC_EINVAL_ARG;
    if (a->window_out && a->window_in) {  // the next window must not overwrite the one being read
        const char *i0 = reinterpret_cast<const char *>(a->window_in), *o0 = reinterpret_cast<const char *>(a->window_out);
        const int64_t bytes = a->batch * channels * a->conv_kernel * (int64_t)sizeof(float);
        if (o0 < i0 + bytes && i0 < o0 + bytes) return DC_EINVAL_ARG;
    }
    return DC_OK;
}

// The kernel by head width and output alignment: even widths take two channels per thread (two segments
// per CTA; channel-pair stores, so the outputs must be aligned), odd widths or outputs that are not
// 16-byte aligned one channel per thread (one segment per CTA).
template <typename TI, typename TO>
void launch_prologue(bool k4, dim3 grid, const dc::pro::Params &p, cudaStream_t s) {
    const bool out16 = aligned(p.q, 16) && aligned(p.k, 16) && aligned(p.v, 16);
    if (out16 && p.dk % 2 == 0 && p.dv % 2 == 0) {
        grid.x = (grid.x + 1) / 2;
        if (k4) dc::pro::prologue_pair_kernel<TI, TO, 4><<<grid, dc::pro::kThreads, 0, s>>>(p);
        else dc::pro::prologue_pair_kernel<TI, TO, dc::pro::kMaxK><<<grid, dc::pro::kThreads, 0, s>>>(p);
    } else {
        if (k4) dc::pro::prologue_kernel<TI, TO, 4><<<grid, dc::pro::kThreads, 0, s>>>(p);
        else dc::pro::prologue_kernel<TI, TO, dc::pro::kMaxK><<<grid, dc::pro::kThreads, 0, s>>>(p);
    }
}

}  // namespace

extern "C" {

int dc_qkv_prologue(const dc_qkv_prologue_args *a, dc_stream_t stream) {
    int st = validate_prologue(a);
    if (st != DC_OK) return st;
    st = check_device(nullptr);
    if (st != DC_OK) return st;
    dc::pro::Params p{};
    p.batch = a->batch;
    p.seq = a->seq;
    p.heads = a->heads;
    p.dk = a->dk;
    p.dv = a->dv;
    p.u = a->n_householder;
    p.K = a->conv_kernel;
    p.channels = a->heads * a->dk * (1 + a->n_householder) + a->n_householder * a->heads * a->dv;
    p.x_stride = a->x_stride;
    p.conv_silu = (a->flags & DC_PROLOGUE_CONV_SILU) ? 1 : 0;
    p.qk_silu = (a->flags & DC_PROLOGUE_QK_SILU) ? 1 : 0;
    p.l2 = (a->flags & DC_PROLOGUE_L2) ? 1 : 0;
    {
        const int64_t esz = a->in_dtype == DC_BF16 ? 2 : 4;
        p.vec_rows = (aligned(a->x, 16) && (a->x_stride * esz) % 16 == 0) ? 1 : 0;
    }
    p.x = a->x;
    p.weight = a->conv_weight;
    p.bias = a->conv_bias;
    p.window_in = a->window_in;
    p.window_out = a->window_out;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    const dim3 grid((unsigned)(a->heads * (1 + 2 * (int64_t)a->n_householder)),
                    (unsigned)((a->seq + dc::pro::kTile - 1) / dc::pro::kTile), (unsigned)a->batch);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool k4 = a->conv_kernel == 4;
    switch (a->in_dtype * 2 + a->out_dtype) {
        case 0: launch_prologue<float, float>(k4, grid, p, s); break;
        case 1: launch_prologue<float, __nv_bfloat16>(k4, grid, p, s); break;
        case 2: launch_prologue<__nv_bfloat16, float>(k4, grid, p, s); break;
        default: launch_prologue<__nv_bfloat16, __nv_bfloat16>(k4, grid, p, s); break;
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dc_gates: the front-end's gate producers (prologue.cuh).
// ---------------------------------------------------------------------------
extern "C" {

int dc_gates(const dc_gate_args *a, dc_stream_t stream) {
    if (!a) return DC_EINVAL_ARG;
    if (a->rows < 0 || a->cols < 1 || a->x_stride < a->cols) return DC_EINVAL_SHAPE;
    if (a->kind < DC_GATE_WRITE || a->kind > DC_GATE_CHANNEL_DECAY) return DC_EINVAL_ARG;
    if (a->in_dtype != DC_F32 && a->in_dtype != DC_BF16) return DC_EUNSUPPORTED_DTYPE;
    if (!isfinite(a->scale) || (a->kind == DC_GATE_HEAD_DECAY && !(a->lo <= a->hi))) return DC_EINVAL_ARG;
    if (a->kind == DC_GATE_CHANNEL_DECAY && (a->group < 1 || a->cols % a->group != 0)) return DC_EINVAL_SHAPE;
    if (a->rows == 0) return DC_OK;
    if (!a->x || !a->out || (a->kind != DC_GATE_WRITE && (!a->bias || !a->a_log))) return DC_EINVAL_ARG;
    const int st = check_device(nullptr);
    if (st != DC_OK) return st;
    dc::pro::GateParams p{};
    p.rows = a->rows;
    p.cols = a->cols;
    p.x_stride = a->x_stride;
    p.kind = a->kind;
    p.group = a->group;
    p.scale = a->scale;
    p.lo = a->lo;
    p.hi = a->hi;
    p.x = a->x;
    p.bias = a->bias;
    p.a_log = a->a_log;
    p.out = a->out;
    if (a->cols > 0x7fffffffLL) return DC_EUNSUPPORTED;
    const int64_t cap = (int64_t)sm_count() * 16;  // of the current device
    const int64_t blocks = a->rows < cap ? a->rows : cap;  // one row per CTA at a time
    // four columns per thread: whole 4-column groups whose loads (8 or 16 bytes) and stores (16) are aligned
    const int64_t esz = a->in_dtype == DC_BF16 ? 2 : 4;
    const int vec4 = (a->cols % 4 == 0 && (a->x_stride * esz) % (4 * esz) == 0 && aligned(a->x, 4 * esz) &&
                      aligned(a->out, 16)) ? 1 : 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (a->in_dtype == DC_BF16) dc::pro::gates_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(p, vec4);
    else dc::pro::gates_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(p, vec4);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DC_OK : cuda_fail(e);
}

}  // extern "C"
