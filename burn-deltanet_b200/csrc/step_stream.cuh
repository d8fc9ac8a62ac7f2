// step_stream.cuh — the decode tick as a persistent stream over heads (dk = dv = 128, one micro-step).
//
// The tick is bound by reading and writing every head's 64 KB fp32 state once (recurrent.rs:41-99,
// the same arithmetic as step.cuh).  Here one CTA per SM walks heads blockIdx.x, + gridDim.x, ...; a
// producer warp moves each head's state (one contiguous 64 KB block) and its q, k, v and full-width gate
// rows with bulk async copies into a three-slot shared-memory ring (up to three heads in flight), stores each
// updated state back with a bulk copy, so that the SM's load and store streams keep going while eight
// consumer warps update the head in the slot:
//
//     S-  = exp(g) (.) S                          (key axis)
//     u_j = w_j v_j - sum_i (b_i k_i) S-_ij
//     S   = S- + k u^T
//     y_j = sum_i (s q_i) S_ij = (s q^T S-)_j + (s q . k) u_j
//
// Slot layout: S [128][128] fp32 row-major, then q, k, v rows (as stored) and the erase, write, g rows
// when they are per channel.  Consumer thread (warp w, lane l) owns columns 4l..4l+3 of rows w, w+8, ...
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace dc {
namespace stream {

constexpr int kConsumers = 256, kThreads = kConsumers + 32, kSlots = 3;
constexpr uint32_t kSBytes = 128 * 128 * 4;
constexpr uint32_t kRowMax = 128 * 4;                       // one input row, up to fp32
constexpr uint32_t kSlotBytes = kSBytes + 6 * kRowMax;      // S, q, k, v, erase, write, g
constexpr uint32_t OFF_RED = kSlots * kSlotBytes;           // [8 warps][3][128] fp32 partial sums
constexpr uint32_t OFF_BAR = OFF_RED + 8 * 3 * 128 * 4;     // full[3], empty[3]
constexpr uint32_t OFF_FLAG = OFF_BAR + 2 * kSlots * 8;
constexpr uint32_t kSmem = OFF_FLAG + 16 + 128;            // (+ alignment slack)
static_assert(kSmem <= 232448, "stream decode over the shared-memory limit");

template <typename T>
__device__ __forceinline__ float rowval(const uint8_t *row, int i) {
    return ld(reinterpret_cast<const T *>(row) + i);
}

template <typename TI, typename TG, typename TO>
__global__ void __launch_bounds__(kThreads, 1) step_stream_kernel(const CoreParams p, int *status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = smem_raw + ((128u - (ptx::smem_u32(smem_raw) & 127u)) & 127u);  // stays a shared pointer
    const uint32_t sb = ptx::smem_u32(base);
    uint64_t *full = reinterpret_cast<uint64_t *>(base + OFF_BAR), *empty = full + kSlots;
    volatile int *flag = reinterpret_cast<volatile int *>(base + OFF_FLAG);
    float *red = reinterpret_cast<float *>(base + OFF_RED);

    ptx::launch_dependents();     // the next tick may be scheduled as this one's CTAs leave their SMs
    ptx::grid_dependency_wait();  // nothing is read before the previous kernel in the stream has finished
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t BH = p.batch * p.heads, H = p.heads;
    const int64_t first = blockIdx.x, stride = gridDim.x;
    const int64_t nitems = first < BH ? (BH - first + stride - 1) / stride : 0;
    constexpr uint32_t kIn = 128 * sizeof(TI), kGate = 128 * sizeof(TG);
    const bool e_full = p.ew != 1, w_full = p.ww != 1, g_full = p.gw > 1;

    if (tid == 0) {
        *flag = 0;
        for (int s = 0; s < kSlots; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();

    // Rows of head bh: q, g, y at (b * q_bstride) * H + h; k, v, erase, write at (b * kv_bstride) * H + h.
    auto qrow = [&](int64_t bh) { return (bh / H) * p.q_bstride * H + bh % H; };
    auto kvrow = [&](int64_t bh) { return (bh / H) * p.kv_bstride * H + bh % H; };

    if (warp == kConsumers / 32) {
        // ================= producer: loads heads into free slots, stores each head once its slot is released ===
        if (lane == 0) {
            auto issue_load = [&](int64_t n) {
                const int s = (int)(n % kSlots);
                const int64_t bh = first + n * stride, qr = qrow(bh), kr = kvrow(bh);
                const uint32_t slot = sb + s * kSlotBytes;
                const uint32_t bytes = kSBytes + 3 * kIn + (e_full ? kGate : 0) + (w_full ? kGate : 0) + (g_full ? kGate : 0);
                ptx::mbar_arrive_expect_tx(&full[s], bytes);
                ptx::bulk_load(slot, p.state_in + bh * 128 * 128, kSBytes, &full[s]);
                ptx::bulk_load(slot + kSBytes, static_cast<const TI *>(p.q) + qr * 128, kIn, &full[s]);
                ptx::bulk_load(slot + kSBytes + kRowMax, static_cast<const TI *>(p.k) + kr * 128, kIn, &full[s]);
                ptx::bulk_load(slot + kSBytes + 2 * kRowMax, static_cast<const TI *>(p.v) + kr * 128, kIn, &full[s]);
                if (e_full)
                    ptx::bulk_load(slot + kSBytes + 3 * kRowMax, static_cast<const TG *>(p.erase) + kr * 128, kGate, &full[s]);
                if (w_full)
                    ptx::bulk_load(slot + kSBytes + 4 * kRowMax, static_cast<const TG *>(p.write) + kr * 128, kGate, &full[s]);
                if (g_full)
                    ptx::bulk_load(slot + kSBytes + 5 * kRowMax, static_cast<const TG *>(p.g) + qr * 128, kGate, &full[s]);
            };
            auto store_done = [&](int64_t n) {  // head n's slot has been updated: write it back
                const int s = (int)(n % kSlots);
                if (!ptx::mbar_wait(&empty[s], (uint32_t)((n / kSlots) & 1))) {
                    *flag = 1;
                    return false;
                }
                ptx::bulk_store(p.state_out + (first + n * stride) * 128 * 128, sb + s * kSlotBytes, kSBytes);
                ptx::bulk_commit();
                return true;
            };
            bool ok = !p.stall;  // (the stall test hook issues nothing: the consumers' waits run out)
            int last_parity[kSlots] = {-1, -1, -1};  // of the load last issued into each slot
            for (int64_t m = 0; m < nitems && ok; ++m) {
                if (m >= kSlots) {  // head m takes the slot of head m - 3: store that one, let the store read it
                    ok = store_done(m - kSlots);
                    if (!ok) break;
                    ptx::bulk_wait_read_all();
                }
                issue_load(m);
                last_parity[m % kSlots] = (int)((m / kSlots) & 1);
            }
            for (int64_t m = nitems > kSlots ? nitems - kSlots : 0; m < nitems && ok; ++m) ok = store_done(m);
            if (!ok && !p.stall) {  // an abort: let every load issued into this CTA's shared memory land before it goes away
                for (int sl = 0; sl < kSlots; ++sl)
                    if (last_parity[sl] >= 0) ptx::mbar_wait(&full[sl], (uint32_t)last_parity[sl]);
            }
            ptx::bulk_wait_all();
        }
        __syncwarp();
    } else {
        // ================= consumers: one head per slot ==========================================================
        const int c0 = 4 * lane;
        TO *y = static_cast<TO *>(p.y);
        for (int64_t n = 0; n < nitems; ++n) {
            const int s = (int)(n % kSlots);
            const int64_t bh = first + n * stride;
            const bool got = ptx::mbar_wait(&full[s], (uint32_t)((n / kSlots) & 1));
            if (ptx::named_sync_or(1, kConsumers, !got || *flag != 0)) {
                *flag = 1;
                break;
            }
            const uint8_t *slot = base + s * kSlotBytes;
            const uint32_t slot_u = sb + s * kSlotBytes;
            const uint8_t *rq = slot + kSBytes, *rk = rq + kRowMax, *rv = rk + kRowMax;
            const uint8_t *re = rv + kRowMax, *rw = re + kRowMax, *rg = rw + kRowMax;
            const int64_t qr = qrow(bh), kr = kvrow(bh);
            // broadcast gates of this head (read directly when not per channel)
            const float e1 = e_full ? 0.f : ld(static_cast<const TG *>(p.erase) + kr);
            const float w1 = w_full ? 0.f : ld(static_cast<const TG *>(p.write) + kr);
            const float g1 = (p.gw == 1) ? __expf(ld(static_cast<const TG *>(p.g) + qr)) : 1.f;
            float sv[16][4];
            float ret[4] = {0.f, 0.f, 0.f, 0.f}, qs[4] = {0.f, 0.f, 0.f, 0.f}, qk = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int row = warp + 8 * j;
                const uint4 raw = ptx::ld_shared_v4(slot_u + row * 512 + 16 * lane);
                const float dec = g_full ? __expf(rowval<TG>(rg, row)) : g1;
                const float kx = rowval<TI>(rk, row);
                const float bk = (e_full ? rowval<TG>(re, row) : e1) * kx;
                const float sq = p.scale * rowval<TI>(rq, row);
                sv[j][0] = __uint_as_float(raw.x) * dec;
                sv[j][1] = __uint_as_float(raw.y) * dec;
                sv[j][2] = __uint_as_float(raw.z) * dec;
                sv[j][3] = __uint_as_float(raw.w) * dec;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    ret[e] = fmaf(bk, sv[j][e], ret[e]);
                    qs[e] = fmaf(sq, sv[j][e], qs[e]);
                }
                qk = fmaf(sq, kx, qk);
            }
            // column sums across the eight warps (rows), and s q . k
            float *rw8 = red + warp * 3 * 128;
            *reinterpret_cast<float4 *>(rw8 + c0) = make_float4(ret[0], ret[1], ret[2], ret[3]);
            *reinterpret_cast<float4 *>(rw8 + 128 + c0) = make_float4(qs[0], qs[1], qs[2], qs[3]);
            if (lane == 0) rw8[256] = qk;
            ptx::named_sync(1, kConsumers);
            float du[4], yv[4];
            float sqk = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) sqk += red[w * 3 * 128 + 256];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float r = 0.f, q = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    r += red[w * 3 * 128 + c0 + e];
                    q += red[w * 3 * 128 + 128 + c0 + e];
                }
                const float wv = (w_full ? rowval<TG>(rw, c0 + e) : w1) * rowval<TI>(rv, c0 + e);
                du[e] = wv - r;
                yv[e] = q + sqk * du[e];
            }
            // S = S- + k u^T, back into the slot
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int row = warp + 8 * j;
                const float kx = rowval<TI>(rk, row);
                ptx::st_shared_v4(slot_u + row * 512 + 16 * lane, __float_as_uint(fmaf(kx, du[0], sv[j][0])),
                                  __float_as_uint(fmaf(kx, du[1], sv[j][1])), __float_as_uint(fmaf(kx, du[2], sv[j][2])),
                                  __float_as_uint(fmaf(kx, du[3], sv[j][3])));
            }
            if (warp == 0) {
                TO *yr = y + qr * 128 + c0;
#pragma unroll
                for (int e = 0; e < 4; ++e) st(yr + e, yv[e]);
            }
            ptx::fence_async_smem();
            ptx::named_sync(1, kConsumers);  // the slot is written (and the partial sums are read)
            if (tid == 0) ptx::mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();
    if (*flag && tid == 0) atomicExch(status, kStatusTimeout);
}

}  // namespace stream
}  // namespace dc
