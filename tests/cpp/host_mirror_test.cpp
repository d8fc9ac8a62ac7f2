// GPU test of the C++ host mirror (burn-deltanet_b200/csrc/delta_core.hpp):
// DeltaInput::run on the chunk and recurrent paths, delta_step and the
// sanity exceptions, checked against the CPU oracle (oracle/oracle.h, linked
// as test infrastructure).  Exit 0 = pass, 1 = fail, 77 = no CUDA device.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "../../burn-deltanet_b200/csrc/delta_core.hpp"
#include "../../oracle/oracle.h"

using namespace burn_deltanet::delta;

namespace {

struct Rng {
    uint64_t s;
    double uniform() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return ((s >> 11) + 0.5) / 9007199254740992.0;
    }
    double normal() { return std::sqrt(-2.0 * std::log(uniform())) * std::cos(6.283185307179586 * uniform()); }
};

template <typename T>
T *to_device(const std::vector<T> &h) {
    T *d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

template <typename T>
std::vector<T> to_host(const T *d, size_t n) {
    std::vector<T> h(n);
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}

uint16_t bf16_bits(double x) {  // round to nearest even
    float f = (float)x;
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
double bf16_value(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

struct Problem {
    long B, S, H, K, V, gw;
    std::vector<double> q, k, v, beta, g, s0;
};

Problem make(long B, long S, long H, long K, long V, bool channel_gate, uint64_t seed) {
    Problem p{B, S, H, K, V, channel_gate ? K : 1, {}, {}, {}, {}, {}, {}};
    Rng r{seed};
    auto l2 = [&](std::vector<double> &x, long width) {
        for (size_t o = 0; o < x.size(); o += width) {
            double n = 1e-6;
            for (long i = 0; i < width; ++i) n += x[o + i] * x[o + i];
            for (long i = 0; i < width; ++i) x[o + i] /= std::sqrt(n);
        }
    };
    p.q.resize(B * S * H * K); p.k.resize(B * S * H * K); p.v.resize(B * S * H * V);
    for (auto &x : p.q) x = r.normal();
    for (auto &x : p.k) x = r.normal();
    for (auto &x : p.v) x = r.normal();
    l2(p.q, K); l2(p.k, K);
    p.beta.resize(B * S * H);
    for (auto &x : p.beta) x = 0.05 + 0.9 * r.uniform();
    p.g.resize(B * S * H * p.gw);
    for (auto &x : p.g) x = -(0.01 + 0.5 * r.uniform());
    p.s0.resize(B * H * K * V);
    for (auto &x : p.s0) x = 0.2 * r.normal();
    return p;
}

double max_abs(const std::vector<double> &a, const std::vector<double> &b) {
    double m = 0;
    for (size_t i = 0; i < a.size(); ++i) m = std::fmax(m, std::fabs(a[i] - b[i]));
    return m;
}

int failures = 0;
void expect(bool ok, const char *what, double err) {
    std::printf("%-52s %s (max err %.3e)\n", what, ok ? "ok" : "FAIL", err);
    if (!ok) ++failures;
}

// fp32 inputs through DeltaInput::run on `path`, against the fp64 oracle.
void check_fp32(const char *name, const Problem &p, const DeltaPath &path) {
    std::vector<float> qf(p.q.begin(), p.q.end()), kf(p.k.begin(), p.k.end()), vf(p.v.begin(), p.v.end());
    std::vector<float> bf(p.beta.begin(), p.beta.end()), gf(p.g.begin(), p.g.end()), sf(p.s0.begin(), p.s0.end());
    float *dq = to_device(qf), *dk = to_device(kf), *dv = to_device(vf), *db = to_device(bf), *dg = to_device(gf);
    float *ds = to_device(sf), *dy = nullptr, *dso = nullptr;
    cudaMalloc(&dy, sizeof(float) * p.B * p.S * p.H * p.V);
    cudaMalloc(&dso, sizeof(float) * p.B * p.H * p.K * p.V);
    DeltaInput in;
    in.q_bshk = view4(dq, p.B, p.S, p.H, p.K, DType::F32);
    in.k_bshk = view4(dk, p.B, p.S, p.H, p.K, DType::F32);
    in.v_bshv = view4(dv, p.B, p.S, p.H, p.V, DType::F32);
    auto gates = beta_gates(view3(db, p.B, p.S, p.H, DType::F32));
    in.erase_bshK = gates.first;
    in.write_bshV = gates.second;
    in.g_bshK = view4(dg, p.B, p.S, p.H, p.gw, DType::F32);
    in.state_bhkv = ds;
    in.run(path, dy, DType::F32, dso);
    cudaDeviceSynchronize();
    auto y = to_host(dy, p.B * p.S * p.H * p.V);
    auto s = to_host(dso, p.B * p.H * p.K * p.V);
    orc_dims d{p.B, p.S, p.H, p.K, p.V, 1, 1, p.gw, 1.0 / std::sqrt((double)p.K), 0};
    std::vector<double> y0(y.size()), s0(s.size());
    orc_recurrent_f64(&d, p.q.data(), p.k.data(), p.v.data(), p.beta.data(), p.beta.data(), p.g.data(),
                      p.s0.data(), y0.data(), s0.data());
    std::vector<double> yd(y.begin(), y.end()), sd(s.begin(), s.end());
    const double ey = max_abs(yd, y0), es = max_abs(sd, s0);
    expect(ey < 1e-4 && es < 1e-4, name, std::fmax(ey, es));
    for (void *ptr : {(void *)dq, (void *)dk, (void *)dv, (void *)db, (void *)dg, (void *)ds, (void *)dy, (void *)dso})
        cudaFree(ptr);
}

}  // namespace

int main() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        std::printf("no CUDA device\n");
        return 77;
    }
    // The reference's own test shapes (src/delta/tests.rs), fp32.
    check_fp32("chunk path, scalar gate, partial chunk", make(2, 13, 2, 8, 8, false, 1), DeltaPath::chunk());
    check_fp32("chunk path, chunk_len 3, channel gate", make(2, 16, 3, 8, 6, true, 2), DeltaPath::with_chunk_len(3));
    check_fp32("recurrent path, dv != dk", make(2, 12, 2, 8, 16, false, 3), DeltaPath::recurrent());
    check_fp32("chunk path, dk = dv = 128", make(1, 70, 2, 128, 128, true, 4), DeltaPath::chunk_len_on_tape(64));

    // delta_step, in place, against one oracle tick.
    {
        Problem p = make(3, 1, 4, 16, 12, false, 5);
        std::vector<float> qf(p.q.begin(), p.q.end()), kf(p.k.begin(), p.k.end()), vf(p.v.begin(), p.v.end());
        std::vector<float> bf(p.beta.begin(), p.beta.end()), gf(p.g.begin(), p.g.end()), sf(p.s0.begin(), p.s0.end());
        float *dq = to_device(qf), *dk = to_device(kf), *dv = to_device(vf), *db = to_device(bf);
        float *dg = to_device(gf), *ds = to_device(sf), *dy = nullptr;
        cudaMalloc(&dy, sizeof(float) * 3 * 4 * 12);
        delta_step(view3(dq, 3, 4, 16, DType::F32), view3(dk, 3, 4, 16, DType::F32), view3(dv, 3, 4, 12, DType::F32),
                   view3(db, 3, 4, 1, DType::F32), view3(db, 3, 4, 1, DType::F32), view3(dg, 3, 4, 1, DType::F32),
                   ds, 0.25, dy, DType::F32, ds);
        cudaDeviceSynchronize();
        auto y = to_host(dy, 3 * 4 * 12);
        auto s = to_host(ds, 3 * 4 * 16 * 12);
        orc_dims d{3, 1, 4, 16, 12, 1, 1, 1, 0.25, 0};
        std::vector<double> y0(y.size()), s0(s.size());
        orc_recurrent_f64(&d, p.q.data(), p.k.data(), p.v.data(), p.beta.data(), p.beta.data(), p.g.data(),
                          p.s0.data(), y0.data(), s0.data());
        std::vector<double> yd(y.begin(), y.end()), sd(s.begin(), s.end());
        const double e = std::fmax(max_abs(yd, y0), max_abs(sd, s0));
        expect(e < 1e-5, "delta_step in place", e);
        for (void *ptr : {(void *)dq, (void *)dk, (void *)dv, (void *)db, (void *)dg, (void *)ds, (void *)dy})
            cudaFree(ptr);
    }

    // bf16 q/k/v, d = 128: the tensor-core route, 2e-2 max-abs vs the oracle on the rounded inputs.
    {
        Problem p = make(2, 200, 2, 128, 128, false, 6);
        std::vector<uint16_t> qb(p.q.size()), kb(p.k.size()), vb(p.v.size());
        for (size_t i = 0; i < qb.size(); ++i) { qb[i] = bf16_bits(p.q[i]); p.q[i] = bf16_value(qb[i]); }
        for (size_t i = 0; i < kb.size(); ++i) { kb[i] = bf16_bits(p.k[i]); p.k[i] = bf16_value(kb[i]); }
        for (size_t i = 0; i < vb.size(); ++i) { vb[i] = bf16_bits(p.v[i]); p.v[i] = bf16_value(vb[i]); }
        std::vector<float> bf(p.beta.begin(), p.beta.end()), gf(p.g.begin(), p.g.end()), sf(p.s0.begin(), p.s0.end());
        uint16_t *dq = to_device(qb), *dk = to_device(kb), *dv = to_device(vb);
        float *db = to_device(bf), *dg = to_device(gf), *ds = to_device(sf), *dy = nullptr, *dso = nullptr;
        cudaMalloc(&dy, sizeof(float) * 2 * 200 * 2 * 128);
        cudaMalloc(&dso, sizeof(float) * 2 * 2 * 128 * 128);
        DeltaInput in;
        in.q_bshk = view4(dq, 2, 200, 2, 128, DType::BF16);
        in.k_bshk = view4(dk, 2, 200, 2, 128, DType::BF16);
        in.v_bshv = view4(dv, 2, 200, 2, 128, DType::BF16);
        in.erase_bshK = view4(db, 2, 200, 2, 1, DType::F32);
        in.write_bshV = view4(db, 2, 200, 2, 1, DType::F32);
        in.g_bshK = view4(dg, 2, 200, 2, 1, DType::F32);
        in.state_bhkv = ds;
        in.run(DeltaPath::chunk(), dy, DType::F32, dso);
        cudaDeviceSynchronize();
        auto y = to_host(dy, 2 * 200 * 2 * 128);
        auto s = to_host(dso, 2 * 2 * 128 * 128);
        orc_dims d{2, 200, 2, 128, 128, 1, 1, 1, 1.0 / std::sqrt(128.0), 0};
        std::vector<double> y0(y.size()), s0(s.size());
        orc_recurrent_f64(&d, p.q.data(), p.k.data(), p.v.data(), p.beta.data(), p.beta.data(), p.g.data(),
                          p.s0.data(), y0.data(), s0.data());
        std::vector<double> yd(y.begin(), y.end()), sd(s.begin(), s.end());
        const double e = std::fmax(max_abs(yd, y0), max_abs(sd, s0));
        expect(e < 2e-2, "bf16 tensor-core chunk path (d = 128)", e);

        // The same call from host memory (pinned): bit-identical to the device call.
        DeltaInput hin = in;
        uint16_t *hq, *hk, *hv;
        float *hb, *hg, *hs, *hy, *hso;
        cudaMallocHost(&hq, qb.size() * 2);
        cudaMallocHost(&hk, kb.size() * 2);
        cudaMallocHost(&hv, vb.size() * 2);
        cudaMallocHost(&hb, bf.size() * 4);
        cudaMallocHost(&hg, gf.size() * 4);
        cudaMallocHost(&hs, sf.size() * 4);
        cudaMallocHost(&hy, y.size() * 4);
        cudaMallocHost(&hso, s.size() * 4);
        std::memcpy(hq, qb.data(), qb.size() * 2);
        std::memcpy(hk, kb.data(), kb.size() * 2);
        std::memcpy(hv, vb.data(), vb.size() * 2);
        std::memcpy(hb, bf.data(), bf.size() * 4);
        std::memcpy(hg, gf.data(), gf.size() * 4);
        std::memcpy(hs, sf.data(), sf.size() * 4);
        hin.q_bshk = view4(hq, 2, 200, 2, 128, DType::BF16);
        hin.k_bshk = view4(hk, 2, 200, 2, 128, DType::BF16);
        hin.v_bshv = view4(hv, 2, 200, 2, 128, DType::BF16);
        hin.erase_bshK = view4(hb, 2, 200, 2, 1, DType::F32);
        hin.write_bshV = view4(hb, 2, 200, 2, 1, DType::F32);
        hin.g_bshK = view4(hg, 2, 200, 2, 1, DType::F32);
        hin.state_bhkv = hs;
        const uint64_t need = hin.host_scratch_size(DeltaPath::chunk(), DType::F32);
        void *scratch = nullptr;
        cudaMalloc(&scratch, need);
        hin.run_from_host(DeltaPath::chunk(), hy, DType::F32, hso, scratch, need);
        cudaDeviceSynchronize();
        const bool same = std::memcmp(hy, y.data(), y.size() * 4) == 0 && std::memcmp(hso, s.data(), s.size() * 4) == 0;
        expect(same, "run_from_host == run (bit-identical)", 0.0);
        for (void *ptr : {(void *)hq, (void *)hk, (void *)hv, (void *)hb, (void *)hg, (void *)hs, (void *)hy, (void *)hso})
            cudaFreeHost(ptr);
        cudaFree(scratch);
        for (void *ptr : {(void *)dq, (void *)dk, (void *)dv, (void *)db, (void *)dg, (void *)ds, (void *)dy, (void *)dso})
            cudaFree(ptr);
    }

    // Size queries are host logic: per-channel gates need a workspace (the two-kernel tensor-core path),
    // per-head gates do not; the host entry point always needs its scratch.
    {
        auto fake = [](int i) { return reinterpret_cast<const void *>(uintptr_t{1} << (20 + i)); };
        DeltaInput in;
        in.q_bshk = view4(fake(0), 1, 128, 2, 128, DType::BF16);
        in.k_bshk = view4(fake(1), 1, 128, 2, 128, DType::BF16);
        in.v_bshv = view4(fake(2), 1, 128, 2, 128, DType::BF16);
        in.erase_bshK = view4(fake(3), 1, 128, 2, 128, DType::F32);
        in.write_bshV = view4(fake(4), 1, 128, 2, 128, DType::F32);
        TensorView g = view4(fake(5), 1, 128, 2, 128, DType::F32);
        in.g_bshK = g;
        in.state_bhkv = reinterpret_cast<const float *>(fake(6));
        const uint64_t ws = in.workspace_size(DeltaPath::chunk(), DType::F32);
        expect(ws == 2ull * 2 * 98816, "workspace_size: per-channel gates, 2 chunks x 2 heads", (double)ws);
        in.erase_bshK = view4(fake(3), 1, 128, 2, 1, DType::F32);
        in.write_bshV = view4(fake(4), 1, 128, 2, 1, DType::F32);
        in.g_bshK = view4(fake(5), 1, 128, 2, 1, DType::F32);
        expect(in.workspace_size(DeltaPath::chunk(), DType::F32) == 0, "workspace_size: per-head gates need none", 0.0);
        expect(in.host_scratch_size(DeltaPath::chunk(), DType::F32) > 0, "host_scratch_size > 0", 0.0);
    }

    // The reference's panics as exceptions.
    {
        DeltaInput in;
        float dummy = 0;
        in.q_bshk = view4(&dummy, 1, 4, 1, 8, DType::F32);
        in.k_bshk = view4(&dummy, 1, 4, 1, 8, DType::F32);
        in.v_bshv = view4(&dummy, 1, 4, 1, 8, DType::F32);
        in.erase_bshK = view4(&dummy, 1, 4, 1, 3, DType::F32);  // width 3: neither 1 nor dk
        in.write_bshV = view4(&dummy, 1, 4, 1, 1, DType::F32);
        in.state_bhkv = &dummy;
        bool threw = false;
        try {
            in.sanity();
        } catch (const std::invalid_argument &) {
            threw = true;
        }
        expect(threw, "sanity(): bad gate width -> std::invalid_argument", 0.0);
    }
    std::printf("%s\n", failures ? "FAILED" : "PASSED");
    return failures ? 1 : 0;
}
