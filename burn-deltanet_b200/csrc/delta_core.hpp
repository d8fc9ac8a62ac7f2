// delta_core.hpp — C++17 host-side mirror of burn-deltanet's delta-rule core
// interface (src/delta/mod.rs:132-137) over the C ABI of include/deltacore.h.
//
// Same names and argument meaning as the reference:
//   DeltaPath   src/delta/path.rs:21-99      (Recurrent / Chunk / ChunkRecalculated, DEFAULT_CHUNK_LEN = 64)
//   TriSolve    src/delta/tri.rs:53-64
//   DeltaInput  src/delta/path.rs:120-231    (dims, resolved_scale, has_channel_decay, sanity, run)
//   delta_step  src/delta/recurrent.rs:41-99
// and the reference's error behaviour: its assert! panics become exceptions —
// std::invalid_argument for the shape and width checks (path.rs:177-208),
// std::runtime_error for everything the C ABI reports.
//
// Tensors are non-owning views of device memory in the reference's layouts.
// Unlike the reference (which returns new tensors), outputs are caller-owned
// buffers passed in: this layer allocates nothing, like the ABI below it.
#pragma once

#include <cmath>
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>

#include "../../include/deltacore.h"

namespace burn_deltanet {
namespace delta {

enum class DType : int32_t { F32 = DC_F32, BF16 = DC_BF16 };

// A non-owning view of a contiguous 3-D or 4-D device tensor.
struct TensorView {
    const void *data = nullptr;
    int64_t dims[4] = {0, 0, 0, 0};
    int rank = 4;
    DType dtype = DType::F32;

    int64_t dim(int i) const { return dims[i]; }
    int64_t last() const { return dims[rank - 1]; }
};

inline TensorView view4(const void *data, int64_t d0, int64_t d1, int64_t d2, int64_t d3, DType dt) {
    TensorView t;
    t.data = data;
    t.dims[0] = d0; t.dims[1] = d1; t.dims[2] = d2; t.dims[3] = d3;
    t.rank = 4;
    t.dtype = dt;
    return t;
}

inline TensorView view3(const void *data, int64_t d0, int64_t d1, int64_t d2, DType dt) {
    TensorView t = view4(data, d0, d1, d2, 0, dt);
    t.rank = 3;
    return t;
}

// How (I - N)^-1 is evaluated.  The kernels substitute; both variants are
// the same T and are accepted (tri.rs:53-64).
enum class TriSolve { Blocked, Neumann };

struct DeltaPath {
    enum class Kind { Recurrent, Chunk, ChunkRecalculated };
    Kind kind = Kind::ChunkRecalculated;
    std::optional<size_t> chunk_len;
    TriSolve solve = TriSolve::Blocked;

    static constexpr size_t DEFAULT_CHUNK_LEN = 64;

    static DeltaPath recurrent() { return DeltaPath{Kind::Recurrent, std::nullopt, TriSolve::Blocked}; }
    static DeltaPath chunk() { return DeltaPath{}; }
    static DeltaPath with_chunk_len(size_t l) { return DeltaPath{Kind::ChunkRecalculated, l, TriSolve::Blocked}; }
    static DeltaPath chunk_len_on_tape(size_t l) { return DeltaPath{Kind::Chunk, l, TriSolve::Blocked}; }
    size_t resolved_chunk_len() const {
        return kind == Kind::Recurrent ? 1 : chunk_len.value_or(DEFAULT_CHUNK_LEN);
    }
};

inline void check_status(int status, const char *what) {
    if (status == DC_OK) return;
    std::string msg = std::string(what) + ": " + dc_status_string(status);
    if (status == DC_ECUDA) msg += " (cudaError " + std::to_string(dc_last_cuda_error()) + ")";
    if (status == DC_EINVAL_SHAPE || status == DC_EINVAL_WIDTH) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

// Everything the core consumes, per head (path.rs:120-141).  q/k arrive
// normalised but unscaled; gates at their broadcast widths (1 or full).
struct DeltaInput {
    TensorView q_bshk;                 // [batch, seq, heads, dk]
    TensorView k_bshk;                 // [batch, seq * u, heads, dk]
    TensorView v_bshv;                 // [batch, seq * u, heads, dv]
    TensorView erase_bshK;             // [batch, seq * u, heads, 1 | dk]
    TensorView write_bshV;             // [batch, seq * u, heads, 1 | dv]
    std::optional<TensorView> g_bshK;  // [batch, seq, heads, 1 | dk], log forget gate
    const float *state_bhkv = nullptr; // [batch, heads, dk, dv]
    std::optional<double> scale;       // None => 1 / sqrt(dk)
    int n_householder = 1;             // micro-steps folded in-kernel (DeltaProduct's u)

    struct Dims {
        int64_t batch, sequence, nheads, head_k_dim, head_v_dim;
    };

    Dims dims() const { return {q_bshk.dim(0), q_bshk.dim(1), q_bshk.dim(2), q_bshk.dim(3), v_bshv.dim(3)}; }

    double resolved_scale() const {
        return scale ? *scale : 1.0 / std::sqrt(static_cast<double>(q_bshk.dim(3)));
    }

    bool has_channel_decay() const { return g_bshK && g_bshK->last() > 1; }

    // The reference's shape asserts (path.rs:177-208) as std::invalid_argument.
    void sanity() const {
        const Dims d = dims();
        const int64_t rows = d.sequence * n_householder;
        auto require = [](bool ok, const std::string &what) {
            if (!ok) throw std::invalid_argument(what);
        };
        require(d.sequence > 0, "sequence length must be at least 1");
        require(n_householder >= 1, "n_householder must be at least 1");
        require(k_bshk.dim(0) == d.batch && k_bshk.dim(1) == rows && k_bshk.dim(2) == d.nheads &&
                    k_bshk.dim(3) == d.head_k_dim,
                "k does not match q");
        require(v_bshv.dim(0) == d.batch && v_bshv.dim(1) == rows && v_bshv.dim(2) == d.nheads, "v does not match q");
        auto gate = [&](const TensorView &t, int64_t trows, int64_t full, const char *what) {
            require(t.dim(0) == d.batch && t.dim(1) == trows && t.dim(2) == d.nheads, what);
            require(t.dim(3) == 1 || t.dim(3) == full,
                    std::string(what) + ": last axis must be 1 or " + std::to_string(full) + ", got " +
                        std::to_string(t.dim(3)));
        };
        gate(erase_bshK, rows, d.head_k_dim, "erase gate");
        gate(write_bshV, rows, d.head_v_dim, "write gate");
        if (g_bshK) gate(*g_bshK, d.sequence, d.head_k_dim, "forget gate");
        require(q_bshk.dtype == k_bshk.dtype && q_bshk.dtype == v_bshv.dtype, "q, k, v must share one dtype");
        require(erase_bshK.dtype == write_bshV.dtype && (!g_bshK || g_bshK->dtype == erase_bshK.dtype),
                "erase, write and g must share one dtype");
        require(state_bhkv != nullptr, "state is required");
    }

    // Bytes of device workspace run() can use for `path` (0: none needed).  With
    // per-channel gates (GDN-2) a workspace of this size lets the tensor cores
    // take the prefill; without one it runs on the CUDA cores.
    uint64_t workspace_size(const DeltaPath &path, DType y_dtype) const {
        const dc_chunk_args a = args(path, placeholder_y(), y_dtype, placeholder_state(), nullptr, 0);
        return dc_chunk_workspace_size(&a);
    }

    // Run the selected algorithm (path.rs:215-231) into caller-owned outputs:
    // y [batch, seq, heads, dv] of y_dtype, final state [batch, heads, dk, dv]
    // (final_state may equal state_bhkv: an in-place update), with an optional
    // caller-owned workspace (see workspace_size).
    void run(const DeltaPath &path, void *y, DType y_dtype, float *final_state, dc_stream_t stream = nullptr,
             void *workspace = nullptr, uint64_t workspace_bytes = 0) const {
        sanity();
        const dc_chunk_args a = args(path, y, y_dtype, final_state, workspace, workspace_bytes);
        check_status(dc_chunk_fwd(&a, stream), "DeltaInput::run");
    }

    // Bytes of device scratch run_from_host() needs for `path`.
    uint64_t host_scratch_size(const DeltaPath &path, DType y_dtype) const {
        const dc_chunk_args a = args(path, placeholder_y(), y_dtype, placeholder_state(), nullptr, 0);
        return dc_chunk_fwd_host_scratch_size(&a);
    }

    // run() for a caller whose tensors are in HOST memory (every view, y and
    // final_state; page-locked for full PCIe speed): the library streams the
    // batch through the GPU in slices of whole sequences, the copies in both
    // directions overlapping the kernels, over `scratch` (device memory of
    // host_scratch_size() bytes, 256-byte aligned).  Returns once the work is
    // queued; the results are on the host when `stream` has drained.
    void run_from_host(const DeltaPath &path, void *y, DType y_dtype, float *final_state, void *scratch,
                       uint64_t scratch_bytes, dc_stream_t stream = nullptr) const {
        sanity();
        const dc_chunk_args a = args(path, y, y_dtype, final_state, nullptr, 0);
        check_status(dc_chunk_fwd_host(&a, scratch, scratch_bytes, stream), "DeltaInput::run_from_host");
    }

  private:
    // Size queries depend on the shapes and on whether the outputs are 16-byte aligned, not on where they
    // are: they pass these stand-ins (aligned, distinct, never dereferenced), i.e. assume aligned outputs
    // such as any device allocation.
    static void *placeholder_y() { return reinterpret_cast<void *>(uintptr_t{1} << 12); }
    static float *placeholder_state() { return reinterpret_cast<float *>(uintptr_t{1} << 13); }

    dc_chunk_args args(const DeltaPath &path, void *y, DType y_dtype, float *final_state, void *workspace,
                       uint64_t workspace_bytes) const {
        const Dims d = dims();
        dc_chunk_args a{};
        a.batch = d.batch;
        a.seq = d.sequence;
        a.heads = d.nheads;
        a.dk = d.head_k_dim;
        a.dv = d.head_v_dim;
        a.n_householder = n_householder;
        a.erase_w = static_cast<int32_t>(erase_bshK.dim(3));
        a.write_w = static_cast<int32_t>(write_bshV.dim(3));
        a.g_w = g_bshK ? static_cast<int32_t>(g_bshK->dim(3)) : 0;
        a.chunk_len = static_cast<int32_t>(path.resolved_chunk_len());
        if (path.kind != DeltaPath::Kind::Recurrent && a.chunk_len < 1)
            throw std::invalid_argument("chunk_len must be at least 1");
        a.in_dtype = static_cast<int32_t>(q_bshk.dtype);
        a.gate_dtype = static_cast<int32_t>(erase_bshK.dtype);
        a.out_dtype = static_cast<int32_t>(y_dtype);
        a.flags = path.kind == DeltaPath::Kind::Recurrent ? DC_FLAG_RECURRENT : 0u;
        a.scale = resolved_scale();
        a.q = q_bshk.data;
        a.k = k_bshk.data;
        a.v = v_bshv.data;
        a.erase = erase_bshK.data;
        a.write = write_bshV.data;
        a.g = g_bshK ? g_bshK->data : nullptr;
        a.state_in = state_bhkv;
        a.y = y;
        a.state_out = final_state;
        a.workspace = workspace;
        a.workspace_bytes = workspace_bytes;
        return a;
    }
};

// The (erase, write) pair a per-head beta stands for (path.rs:147-150): the
// same [.., heads] buffer viewed with a trailing axis of 1.
inline std::pair<TensorView, TensorView> beta_gates(const TensorView &beta_bsh) {
    TensorView g = view4(beta_bsh.data, beta_bsh.dim(0), beta_bsh.dim(1), beta_bsh.dim(2), 1, beta_bsh.dtype);
    return {g, g};
}

// One delta-rule tick for all heads (recurrent.rs:41-99): q [b, h, dk],
// k [b, h, dk], v [b, h, dv], erase [b, h, 1|dk], write [b, h, 1|dv],
// g [b, h, 1|dk] or none; state [b, h, dk, dv] in, next_state out
// (next_state may equal state).
inline void delta_step(const TensorView &q_bhk, const TensorView &k_bhk, const TensorView &v_bhv,
                       const TensorView &erase_bhK, const TensorView &write_bhV,
                       const std::optional<TensorView> &g_bhK, const float *state_bhkv, double scale, void *y,
                       DType y_dtype, float *next_state, dc_stream_t stream = nullptr) {
    const int64_t b = q_bhk.dim(0), h = q_bhk.dim(1), dk = q_bhk.dim(2), dv = v_bhv.dim(2);
    if (k_bhk.dim(0) != b || k_bhk.dim(1) != h || k_bhk.dim(2) != dk)
        throw std::invalid_argument("k does not match q");
    if (v_bhv.dim(0) != b || v_bhv.dim(1) != h) throw std::invalid_argument("v does not match q");
    dc_step_args a{};
    a.batch = b;
    a.heads = h;
    a.dk = dk;
    a.dv = dv;
    a.n_householder = 1;
    a.erase_w = static_cast<int32_t>(erase_bhK.dim(2));
    a.write_w = static_cast<int32_t>(write_bhV.dim(2));
    a.g_w = g_bhK ? static_cast<int32_t>(g_bhK->dim(2)) : 0;
    a.in_dtype = static_cast<int32_t>(q_bhk.dtype);
    a.gate_dtype = static_cast<int32_t>(erase_bhK.dtype);
    a.out_dtype = static_cast<int32_t>(y_dtype);
    a.scale = scale;
    a.q = q_bhk.data;
    a.k = k_bhk.data;
    a.v = v_bhv.data;
    a.erase = erase_bhK.data;
    a.write = write_bhV.data;
    a.g = g_bhK ? g_bhK->data : nullptr;
    a.state_in = state_bhkv;
    a.y = y;
    a.state_out = next_state;
    check_status(dc_step(&a, stream), "delta_step");
}

}  // namespace delta
}  // namespace burn_deltanet
