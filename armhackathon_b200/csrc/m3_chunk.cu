// Mamba-3 SISO / MIMO scan in chunked (dual) form, fp32 on CUDA cores.
//
// One CTA per (batch, head) walks the sequence in chunks of QR = 64 rows,
// where a row is a (step, rank) pair: 64 steps for SISO, 64/R steps of R
// ranks for MIMO (R in {1, 2, 4}).  With l_t the within-chunk inclusive
// cumulative sum of adt (traversal order), w_s = exp(l_last - l_s) * scale_s,
// and S the (dv x dqk) state entering the chunk, the recurrence of
// mamba3/scalar.rs:50-196 and mimo.rs:98-284 unrolls to
//
//   W[i][j] = (q_i . k_j) * ( exp(l_ti - l_tj) * scale_tj   if t_j < t_i
//                             gamma_ti                      if t_j = t_i
//                             0                             otherwise )
//   Y[i]    = sum_j W[i][j] x_j  +  exp(l_ti) * (q_i . S^T)  +  D * x_i
//   S      <- exp(l_last) * S  +  sum_j w_tj * x_j (x) k_j
//
// (alpha_t * exp(l_{t-1}) = exp(l_t) folds the per-step decay of the
// sequential form into the chunk's cumulative decay; the diagonal of W is
// the trapezoid's current-step term gamma_t (q.k) x, including MIMO's
// rank-by-rank Gram).  SISO output is Y * silu(z); MIMO output sums the R
// rows of a step: sum_r phi_r * silu(z * zeta_r) * Y[(t, r)].
//
// Shared memory holds q^T, k^T (dqk-major, for the Gram and q.S^T), w*k
// row-major (for the state update; its last valid row is scale_T * k_T, the
// SISO last_bx), x row-major, W^T and S^T (dqk-major).  Every product is a
// register-tiled loop with 16-byte shared loads; four barriers per chunk.
// Requires dv % 4 == 0, dqk % 8 == 0, dv <= 128, dqk <= 128.
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "m1_scan.h"
#include "m3_scan.h"

namespace b200scan {

namespace {

constexpr int kCkThreads = 256;
constexpr int kQR = 64;  // rows (step, rank) per chunk

// kCkFull: every array (sequential form); kCkDs: w*k, x and gates (state
// contributions); kCkOut: everything but w*k (outputs; W^T over k^T).
enum CkMode { kCkFull = 0, kCkDs = 1, kCkOut = 2 };

struct CkLayout {
    int N, P, NP4, PP4, QP4;  // dims and padded strides
    int qT, kT, kw, x, WT, ST, gate;  // float offsets
    int total;
    __host__ __device__ CkLayout(int dqk, int dv, int mode = kCkFull) {
        N = dqk;
        P = dv;
        QP4 = kQR + 4;
        NP4 = N + 4;
        PP4 = P + 4;
        const bool q = mode != kCkDs, k = mode != kCkOut;
        qT = 0;
        kT = qT + (q ? N * QP4 : 0);
        kw = kT + (q ? N * QP4 : 0);
        x = kw + (k ? kQR * NP4 : 0);
        // outputs-only mode: W^T over k^T (N >= kQR rows), written once
        // every thread has read k^T, where that lets more CTAs fit an SM
        // (227 KB each): 64 x 64 heads go from 2 to 3
        const int plain = (N * QP4 * 2 + kQR * PP4 + kQR * QP4 + N * PP4 + 4 * kQR + 8) * 4;
        const int aliased = plain - kQR * QP4 * 4;
        const bool alias = mode == kCkOut && N >= kQR && (227 * 1024) / aliased > (227 * 1024) / plain;
        WT = alias ? kT : x + kQR * PP4;
        ST = alias ? x + kQR * PP4 : WT + (q ? kQR * QP4 : 0);
        gate = ST + (q ? N * PP4 : 0);
        total = gate + 4 * kQR + 8;  // lcum, scale, gamma, w  + eQ
    }
};

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Shared-memory view of one chunk (every array of CkLayout).
struct CkSmem {
    float *qT, *kT, *kw, *xs, *WT, *ST, *lcum, *scl, *gam, *wdec, *eQ;
    __device__ CkSmem(float* sm, const CkLayout& ly) {
        qT = sm + ly.qT;
        kT = sm + ly.kT;
        kw = sm + ly.kw;
        xs = sm + ly.x;
        WT = sm + ly.WT;
        ST = sm + ly.ST;
        lcum = sm + ly.gate;
        scl = lcum + kQR;
        gam = scl + kQR;
        wdec = gam + kQR;
        eQ = wdec + kQR;
    }
};

// A1. gates of the chunk's steps (warp 0): cumulative log-decay, trapezoid
// scale, gamma, state weight, total decay.
template <int R>
__device__ __forceinline__ void ck_gates(const M3Params& p, int64_t bh, int64_t it0, const CkSmem& s) {
    constexpr int QS = kQR / R;
    const int lane = threadIdx.x & 31;
    const int64_t L = p.len, gate_base = bh * L;
    float lv[2], sc[2], gm[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int j = lane + 32 * e;
        const int64_t it = it0 + j;
        lv[e] = 0.f;
        sc[e] = 0.f;
        gm[e] = 0.f;
        if (j < QS && it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t g = gate_base + m3_phys(p, t);
            const float gamma = p.dt[g] * sigmoid_f(p.trap[g]);
            float shifted = 0.f;
            if (it + 1 < L) {
                const int64_t nx = gate_base + m3_phys(p, p.reverse ? t - 1 : t + 1);
                shifted = p.dt[nx] * (1.f - sigmoid_f(p.trap[nx]));
            }
            lv[e] = p.adt[g];
            sc[e] = gamma + shifted;
            gm[e] = gamma;
        }
    }
    // inclusive prefix sum over the 64 slots (lane, lane + 32)
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float v = __shfl_up_sync(0xffffffffu, lv[e], o);
            if (lane >= o) lv[e] += v;
        }
    lv[1] += __shfl_sync(0xffffffffu, lv[0], 31);
    const float last = QS > 32 ? __shfl_sync(0xffffffffu, lv[1], 31)
                               : __shfl_sync(0xffffffffu, lv[0], QS - 1);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int j = lane + 32 * e;
        if (j < QS) {
            s.lcum[j] = lv[e];
            s.scl[j] = sc[e];
            s.gam[j] = gm[e];
            s.wdec[j] = expf(last - lv[e]) * sc[e];
        }
    }
    if (lane == 0) s.eQ[0] = expf(last);
}

// A2. rotated q (WITH_Q), k into q^T, k^T (WITH_QT) and w*k rows (WITH_KW),
// and x rows.  Element-by-element form (any alignment).
template <int R, bool WITH_QT, bool WITH_KW>
__device__ __forceinline__ void ck_stage_scalar(const M3Params& p, const CkLayout& ly, int64_t bi,
                                         int64_t h, int64_t it0, const CkSmem& s) {
    constexpr int QS = kQR / R;
    const int tid = threadIdx.x;
    const int64_t H = p.heads, L = p.len;
    const int N = ly.N, P = ly.P, half = N / 2;
    const bool mimo = R > 1 || p.psi != nullptr;
    for (int idx = tid; idx < kQR * half; idx += kCkThreads) {
        const int i = idx / half, pi = idx - (idx / half) * half;
        const int j = i / R, r = i - (i / R) * R;  // step, rank
        const int64_t it = it0 + j;
        float q0 = 0.f, q1 = 0.f, k0 = 0.f, k1 = 0.f;
        const int i0 = mimo ? pi : 2 * pi, i1 = mimo ? pi + half : 2 * pi + 1;
        if (j < QS && it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t pt = m3_phys(p, t);
            const int64_t qk_off = (bi * L + pt) * (mimo ? R : 1) * N + r * N;
            const float* qb = p.q_bias + (h * (mimo ? R : 1) + r) * N;
            const float* kb = p.k_bias + (h * (mimo ? R : 1) + r) * N;
            const int64_t cs = ((bi * L + t) * H + h) * half + pi;
            const float c = p.cos[cs], sn = p.sin[cs];
            float a0, a1;
            if (WITH_QT) {
                a0 = p.q[qk_off + i0] + qb[i0];
                a1 = p.q[qk_off + i1] + qb[i1];
                q0 = a0 * c - a1 * sn;
                q1 = a0 * sn + a1 * c;
            }
            a0 = p.k[qk_off + i0] + kb[i0];
            a1 = p.k[qk_off + i1] + kb[i1];
            k0 = a0 * c - a1 * sn;
            k1 = a0 * sn + a1 * c;
        }
        if (WITH_QT) {
            s.qT[i0 * ly.QP4 + i] = q0;
            s.qT[i1 * ly.QP4 + i] = q1;
            s.kT[i0 * ly.QP4 + i] = k0;
            s.kT[i1 * ly.QP4 + i] = k1;
        }
        if (WITH_KW) {
            const float w = j < QS ? s.wdec[j] : 0.f;
            s.kw[i * ly.NP4 + i0] = w * k0;
            s.kw[i * ly.NP4 + i1] = w * k1;
        }
    }
    for (int idx = tid; idx < kQR * P; idx += kCkThreads) {
        const int i = idx / P, pp = idx - (idx / P) * P;
        const int j = i / R, r = i - (i / R) * R;
        const int64_t it = it0 + j;
        float v = 0.f;
        if (j < QS && it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            v = p.v[((bi * L + m3_phys(p, t)) * H + h) * P + pp];
            if (mimo) v *= p.psi[(h * R + r) * P + pp];
        }
        s.xs[i * ly.PP4 + pp] = v;
    }
}

__host__ __device__ inline bool ck_aligned16(const void* q) {
    return (reinterpret_cast<uintptr_t>(q) & 15u) == 0;
}
// whether the vector form of A2 applies (dims and 16-byte alignment)
__host__ __device__ inline bool ck_vec_ok(const M3Params& p) {
    return p.dqk % 8 == 0 && p.dv % 4 == 0 && ck_aligned16(p.q) && ck_aligned16(p.k) &&
           ck_aligned16(p.cos) && ck_aligned16(p.sin) && ck_aligned16(p.q_bias) &&
           ck_aligned16(p.k_bias) && ck_aligned16(p.v) && (p.psi == nullptr || ck_aligned16(p.psi));
}

// A2, vector form (16-byte aligned q, k, cos, sin, biases, v): one item =
// one row x 4 rotation pairs, read with 16-byte loads (interleaved SISO: 8
// consecutive dims; MIMO split halves: 4 dims of each half).  Rows vary
// fastest across threads, so the transposed q^T / k^T stores are
// conflict-free and a warp's loads cover whole 32-byte sectors.
template <int R, bool WITH_QT, bool WITH_KW>
__device__ __forceinline__ void ck_stage_vec(const M3Params& p, const CkLayout& ly, int64_t bi,
                                             int64_t h, int64_t it0, const CkSmem& s) {
    constexpr int QS = kQR / R;
    const int tid = threadIdx.x;
    const int64_t H = p.heads, L = p.len;
    const int N = ly.N, P = ly.P, half = N / 2;
    const bool mimo = R > 1 || p.psi != nullptr;
    const int n_chunks = half / 4;
    for (int idx = tid; idx < kQR * n_chunks; idx += kCkThreads) {
        const int i = idx % kQR, c = idx / kQR;
        const int j = i / R, r = i - (i / R) * R;  // step, rank
        const int64_t it = it0 + j;
        // dims of the 4 pairs: lo[e] rotates with hi[e]
        const int d_lo = mimo ? 4 * c : 8 * c;
        float qlo[4] = {0.f, 0.f, 0.f, 0.f}, qhi[4] = {0.f, 0.f, 0.f, 0.f};
        float klo[4] = {0.f, 0.f, 0.f, 0.f}, khi[4] = {0.f, 0.f, 0.f, 0.f};
        if (j < QS && it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t qk_off = (bi * L + m3_phys(p, t)) * (mimo ? R : 1) * N + r * N;
            const int64_t bo = (h * (mimo ? R : 1) + r) * N;
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cos + ((bi * L + t) * H + h) * half + 4 * c));
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sin + ((bi * L + t) * H + h) * half + 4 * c));
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
            auto rot = [&](const float* src, const float* bias, float (&lo)[4], float (&hi)[4]) {
                float a[4], b[4];
                if (mimo) {
                    const float4 x0 = __ldg(reinterpret_cast<const float4*>(src + d_lo));
                    const float4 x1 = __ldg(reinterpret_cast<const float4*>(src + d_lo + half));
                    const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + d_lo));
                    const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + d_lo + half));
                    a[0] = x0.x + b0.x; a[1] = x0.y + b0.y; a[2] = x0.z + b0.z; a[3] = x0.w + b0.w;
                    b[0] = x1.x + b1.x; b[1] = x1.y + b1.y; b[2] = x1.z + b1.z; b[3] = x1.w + b1.w;
                } else {
                    const float4 x0 = __ldg(reinterpret_cast<const float4*>(src + d_lo));
                    const float4 x1 = __ldg(reinterpret_cast<const float4*>(src + d_lo + 4));
                    const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + d_lo));
                    const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + d_lo + 4));
                    a[0] = x0.x + b0.x; b[0] = x0.y + b0.y; a[1] = x0.z + b0.z; b[1] = x0.w + b0.w;
                    a[2] = x1.x + b1.x; b[2] = x1.y + b1.y; a[3] = x1.z + b1.z; b[3] = x1.w + b1.w;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    lo[e] = a[e] * cc[e] - b[e] * ss[e];
                    hi[e] = a[e] * ss[e] + b[e] * cc[e];
                }
            };
            if (WITH_QT) rot(p.q + qk_off, p.q_bias + bo, qlo, qhi);
            rot(p.k + qk_off, p.k_bias + bo, klo, khi);
        }
        const float w = (WITH_KW && j < QS) ? s.wdec[j] : 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i0 = mimo ? d_lo + e : d_lo + 2 * e;
            const int i1 = mimo ? d_lo + e + half : d_lo + 2 * e + 1;
            if (WITH_QT) {
                s.qT[i0 * ly.QP4 + i] = qlo[e];
                s.qT[i1 * ly.QP4 + i] = qhi[e];
                s.kT[i0 * ly.QP4 + i] = klo[e];
                s.kT[i1 * ly.QP4 + i] = khi[e];
            }
            if (WITH_KW) {
                s.kw[i * ly.NP4 + i0] = w * klo[e];
                s.kw[i * ly.NP4 + i1] = w * khi[e];
            }
        }
    }
    // x rows: 4 channels per item, rows fastest
    for (int idx = tid; idx < kQR * (P / 4); idx += kCkThreads) {
        const int i = idx % kQR, c = idx / kQR;
        const int j = i / R, r = i - (i / R) * R;
        const int64_t it = it0 + j;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < QS && it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            v = __ldg(reinterpret_cast<const float4*>(p.v + ((bi * L + m3_phys(p, t)) * H + h) * P + 4 * c));
            if (mimo) {
                const float4 ps = __ldg(reinterpret_cast<const float4*>(p.psi + (h * R + r) * P + 4 * c));
                v.x *= ps.x; v.y *= ps.y; v.z *= ps.z; v.w *= ps.w;
            }
        }
        *reinterpret_cast<float4*>(s.xs + i * ly.PP4 + 4 * c) = v;
    }
}

template <int R, bool WITH_QT, bool WITH_KW>
__device__ __forceinline__ void ck_stage(const M3Params& p, const CkLayout& ly, int64_t bi,
                                         int64_t h, int64_t it0, const CkSmem& s, bool vec) {
    if (vec)
        ck_stage_vec<R, WITH_QT, WITH_KW>(p, ly, bi, h, it0, s);
    else
        ck_stage_scalar<R, WITH_QT, WITH_KW>(p, ly, bi, h, it0, s);
}

// B. W^T[j][i] = mask(t_i, t_j) * (q_i . k_j); 4x4 tiles
template <int R>
__device__ __forceinline__ void ck_w(const CkLayout& ly, const CkSmem& s) {
    constexpr int QS = kQR / R;
    const int tid = threadIdx.x, N = ly.N;
    const int ti = tid / 16, tj = tid % 16;  // 16 x 16 tiles of 4 x 4
    const int i0 = ti * 4, j0 = tj * 4;
    float acc[4][4] = {};
    if (j0 / R <= (i0 + 3) / R) {
        for (int n = 0; n < N; ++n) {
            const float4 a = ld4(s.qT + n * ly.QP4 + i0);
            const float4 b = ld4(s.kT + n * ly.QP4 + j0);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
        }
    }
    if (ly.WT == ly.kT) __syncthreads();  // W^T replaces k^T: every read of k^T first
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        float out[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int si = (i0 + u) / R, sj = (j0 + v) / R;
            float m = 0.f;
            if (sj < si) m = expf(s.lcum[si] - s.lcum[sj]) * s.scl[sj];
            else if (sj == si) m = s.gam[si];
            out[u] = (si < QS) ? m * acc[u][v] : 0.f;
        }
        *reinterpret_cast<float4*>(s.WT + (j0 + v) * ly.QP4 + i0) =
            make_float4(out[0], out[1], out[2], out[3]);
    }
}

// C. Y = W x + exp(l) q S^T (with_state) + D x; gate and store
template <int R>
__device__ __forceinline__ void ck_out(const M3Params& p, const CkLayout& ly, int64_t bi, int64_t h,
                                       int64_t it0, bool with_state, const CkSmem& s) {
    constexpr int QS = kQR / R;
    const int tid = threadIdx.x, N = ly.N, P = ly.P;
    const int64_t H = p.heads, L = p.len;
    const bool mimo = R > 1 || p.psi != nullptr;
    const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
    for (int tile = tid; tile < (kQR / 4) * (P / 4); tile += kCkThreads) {
        const int i0 = (tile / (P / 4)) * 4, p0 = (tile % (P / 4)) * 4;
        float acc[4][4] = {}, inter[4][4] = {};
        for (int j = 0; j < kQR; ++j) {
            const float4 a = ld4(s.WT + j * ly.QP4 + i0);
            const float4 b = ld4(s.xs + j * ly.PP4 + p0);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
        }
        if (with_state) {
            for (int n = 0; n < N; ++n) {
                const float4 a = ld4(s.qT + n * ly.QP4 + i0);
                const float4 b = ld4(s.ST + n * ly.PP4 + p0);
                const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int v = 0; v < 4; ++v) inter[u][v] = fmaf(av[u], bv[v], inter[u][v]);
            }
        }
        float y[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int si = (i0 + u) / R;
            const float el = si < QS ? expf(s.lcum[si]) : 0.f;
            const float4 xv = ld4(s.xs + (i0 + u) * ly.PP4 + p0);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int v = 0; v < 4; ++v) y[u][v] = acc[u][v] + el * inter[u][v] + dsk * xa[v];
        }
        // rows i0..i0+3 are steps i0/R .. (i0+3)/R; reduce ranks per step
#pragma unroll
        for (int u0 = 0; u0 < 4; u0 += R) {
            const int step = (i0 + u0) / R;
            const int64_t it = it0 + step;
            if (step >= QS || it >= L) continue;
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t pt = m3_phys(p, t);
            const int64_t voff = ((bi * L + pt) * H + h) * P + p0;
            float o[4] = {0.f, 0.f, 0.f, 0.f};
            float zv[4] = {0.f, 0.f, 0.f, 0.f};
            if (p.z) {
                const float4 z4 = *reinterpret_cast<const float4*>(p.z + voff);
                zv[0] = z4.x; zv[1] = z4.y; zv[2] = z4.z; zv[3] = z4.w;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const float yy = y[u0 + r][v];
                    if (mimo) {
                        const int64_t po = (h * R + r) * P + p0 + v;
                        const float g = p.z ? silu_f(zv[v] * p.zeta[po]) : 1.f;
                        o[v] += p.phi[po] * g * yy;
                    } else {
                        o[v] = p.z ? yy * silu_f(zv[v]) : yy;
                    }
                }
            }
            float4* dst = reinterpret_cast<float4*>(
                p.out + (p.out_blh ? (bi * L + pt) * H + h : (bi * H + h) * L + pt) * P + p0);
            if (p.out_acc) {
                const float4 prev = *dst;
                o[0] += prev.x; o[1] += prev.y; o[2] += prev.z; o[3] += prev.w;
            }
            *dst = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

// D. dS^T[n][p] = sum_j kw[j][n] x[j][p] for one 8(n) x 4(p) tile
__device__ __forceinline__ void ck_ds_tile(const CkLayout& ly, const CkSmem& s, int n0, int p0,
                                           float (&acc)[8][4]) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = 0.f;
    for (int j = 0; j < kQR; ++j) {
        const float4 k0 = ld4(s.kw + j * ly.NP4 + n0);
        const float4 k1 = ld4(s.kw + j * ly.NP4 + n0 + 4);
        const float4 b = ld4(s.xs + j * ly.PP4 + p0);
        const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(kv[u], bv[v], acc[u][v]);
    }
}

// SISO last_bx: scale_T * k_T, the last valid row of w*k in the final chunk
template <int R>
__device__ __forceinline__ void ck_last_bx(const M3Params& p, const CkLayout& ly, int64_t bh,
                                           int64_t it0, const CkSmem& s) {
    const int lastrow = static_cast<int>(p.len - 1 - it0);
    for (int n = threadIdx.x; n < ly.N; n += kCkThreads) p.last_bx[bh * ly.N + n] = s.kw[lastrow * ly.NP4 + n];
}

// Sequential form: one CTA per (batch, head) walks the chunks, S in shared
// memory.
template <int R>
__global__ void __launch_bounds__(kCkThreads, 1) m3_chunk_kernel(M3Params p) {
    const bool vec = ck_vec_ok(p);
    constexpr int QS = kQR / R;
    extern __shared__ float4 smem4[];
    const CkLayout ly(static_cast<int>(p.dqk), static_cast<int>(p.dv));
    const CkSmem s(reinterpret_cast<float*>(smem4), ly);
    const int N = ly.N, P = ly.P, tid = threadIdx.x, warp = tid >> 5;
    const int64_t bh = blockIdx.x, H = p.heads, L = p.len;
    const int64_t bi = bh / H, h = bh % H;
    const bool mimo = R > 1 || p.psi != nullptr;
    const int n_chunks = static_cast<int>((L + QS - 1) / QS);

    for (int i = tid; i < N * ly.PP4; i += kCkThreads) s.ST[i] = 0.f;
    for (int ch = 0; ch < n_chunks; ++ch) {
        const int64_t it0 = static_cast<int64_t>(ch) * QS;  // first traversal index
        if (warp == 0) ck_gates<R>(p, bh, it0, s);
        __syncthreads();
        ck_stage<R, true, true>(p, ly, bi, h, it0, s, vec);
        __syncthreads();
        ck_w<R>(ly, s);
        __syncthreads();
        ck_out<R>(p, ly, bi, h, it0, ch > 0, s);
        __syncthreads();
        // S^T = eQ S^T + dS^T
        const float e = s.eQ[0];
        for (int tile = tid; tile < (N / 8) * (P / 4); tile += kCkThreads) {
            const int n0 = (tile / (P / 4)) * 8, p0 = (tile % (P / 4)) * 4;
            float acc[8][4];
            ck_ds_tile(ly, s, n0, p0, acc);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                float* st = s.ST + (n0 + u) * ly.PP4 + p0;
                const float4 old = ld4(st);
                *reinterpret_cast<float4*>(st) =
                    make_float4(fmaf(e, old.x, acc[u][0]), fmaf(e, old.y, acc[u][1]),
                                fmaf(e, old.z, acc[u][2]), fmaf(e, old.w, acc[u][3]));
            }
        }
        if (!mimo && p.last_bx && ch == n_chunks - 1) ck_last_bx<R>(p, ly, bh, it0, s);
        __syncthreads();
    }
    if (p.last_state) {
        for (int idx = tid; idx < P * N; idx += kCkThreads) {
            const int pp = idx / N, n = idx - (idx / N) * N;
            p.last_state[(bh * P + pp) * N + n] = s.ST[n * ly.PP4 + pp];
        }
    }
}

// ---------------------------------------------------------------------------
// Chunk-parallel form (three launches; every (batch*head, chunk) tile is an
// independent CTA, so the GPU fills even with few heads):
//   1. m3_chunk_ds_kernel: dS^T(c) = sum_j (w k)_j x_j^T and decay(c) = e^{l_last};
//   2. m3_chunk_state_kernel: S_in(c+1) = decay(c) S_in(c) + dS(c), written over
//      dS(c) (loads run ahead of the dependent update); the final S is last_state;
//   3. m3_chunk_out_kernel: W, Y = W x + e^l q S_in^T + D x, gating.
struct CkWs {
    float* st;     // [bh][chunk][N][P]
    float* decay;  // [bh][chunk]
};

template <int R>
__global__ void __launch_bounds__(kCkThreads, 4) m3_chunk_ds_kernel(M3Params p, CkWs ws, int n_chunks) {
    const bool vec = ck_vec_ok(p);
    constexpr int QS = kQR / R;
    extern __shared__ float4 smem4[];
    const CkLayout ly(static_cast<int>(p.dqk), static_cast<int>(p.dv), kCkDs);
    const CkSmem s(reinterpret_cast<float*>(smem4), ly);
    const int N = ly.N, P = ly.P, tid = threadIdx.x, warp = tid >> 5;
    const int ch = blockIdx.x;
    const int64_t bh = blockIdx.y, H = p.heads;
    const int64_t bi = bh / H, h = bh % H;
    const int64_t it0 = static_cast<int64_t>(ch) * QS;
    const bool mimo = R > 1 || p.psi != nullptr;
    if (warp == 0) ck_gates<R>(p, bh, it0, s);
    __syncthreads();
    if (tid == 0) ws.decay[bh * n_chunks + ch] = s.eQ[0];
    ck_stage<R, false, true>(p, ly, bi, h, it0, s, vec);
    __syncthreads();
    float* out = ws.st + (bh * n_chunks + ch) * static_cast<int64_t>(N) * P;
    for (int tile = tid; tile < (N / 8) * (P / 4); tile += kCkThreads) {
        const int n0 = (tile / (P / 4)) * 8, p0 = (tile % (P / 4)) * 4;
        float acc[8][4];
        ck_ds_tile(ly, s, n0, p0, acc);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(out + (n0 + u) * P + p0) =
                make_float4(acc[u][0], acc[u][1], acc[u][2], acc[u][3]);
    }
    if (!mimo && p.last_bx && ch == n_chunks - 1) ck_last_bx<R>(p, ly, bh, it0, s);
}

__global__ void __launch_bounds__(kCkThreads) m3_chunk_state_kernel(M3Params p, CkWs ws, int n_chunks) {
    const int64_t bh = blockIdx.x;
    const int64_t NP = p.dqk * p.dv;
    const int64_t e0 = (static_cast<int64_t>(blockIdx.y) * kCkThreads + threadIdx.x) * 4;
    if (e0 >= NP) return;
    float* base = ws.st + bh * n_chunks * NP + e0;
    const float* dec = ws.decay + bh * n_chunks;
    float4 S = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 nd = *reinterpret_cast<const float4*>(base);
    float nq = dec[0];
    for (int c = 0; c < n_chunks; ++c) {
        const float4 d = nd;
        const float q = nq;
        if (c + 1 < n_chunks) {
            nd = *reinterpret_cast<const float4*>(base + (c + 1) * NP);
            nq = dec[c + 1];
        }
        *reinterpret_cast<float4*>(base + c * NP) = S;
        S.x = fmaf(q, S.x, d.x);
        S.y = fmaf(q, S.y, d.y);
        S.z = fmaf(q, S.z, d.z);
        S.w = fmaf(q, S.w, d.w);
    }
    if (p.last_state) {
        // entries are (n, p) row-major; last_state is (p, n)
        const float sv[4] = {S.x, S.y, S.z, S.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int64_t n = (e0 + e) / p.dv, pp = (e0 + e) % p.dv;
            p.last_state[(bh * p.dv + pp) * p.dqk + n] = sv[e];
        }
    }
}

template <int R>
__global__ void __launch_bounds__(kCkThreads) m3_chunk_out_kernel(M3Params p, CkWs ws, int n_chunks) {
    const bool vec = ck_vec_ok(p);
    constexpr int QS = kQR / R;
    extern __shared__ float4 smem4[];
    const CkLayout ly(static_cast<int>(p.dqk), static_cast<int>(p.dv), kCkOut);
    const CkSmem s(reinterpret_cast<float*>(smem4), ly);
    const int N = ly.N, P = ly.P, tid = threadIdx.x, warp = tid >> 5;
    const int ch = blockIdx.x;
    const int64_t bh = blockIdx.y, H = p.heads;
    const int64_t bi = bh / H, h = bh % H;
    const int64_t it0 = static_cast<int64_t>(ch) * QS;
    if (warp == 0) ck_gates<R>(p, bh, it0, s);
    if (ch > 0) {
        const float* src = ws.st + (bh * n_chunks + ch) * static_cast<int64_t>(N) * P;
        for (int idx = tid; idx < N * (P / 4); idx += kCkThreads) {
            const int n = idx / (P / 4), p0 = (idx % (P / 4)) * 4;
            *reinterpret_cast<float4*>(s.ST + n * ly.PP4 + p0) = ld4(src + n * P + p0);
        }
    }
    __syncthreads();
    ck_stage<R, true, false>(p, ly, bi, h, it0, s, vec);
    __syncthreads();
    ck_w<R>(ly, s);
    __syncthreads();
    ck_out<R>(p, ly, bi, h, it0, ch > 0, s);
}

}  // namespace

bool m3_chunk_applicable(const M3Params& p) {
    const int R = p.psi ? static_cast<int>(p.rank) : 1;
    if (!(R == 1 || R == 2 || R == 4)) return false;
    if (p.dv % 4 || p.dqk % 8 || p.dv > 128 || p.dqk > 128) return false;
    const CkLayout ly(static_cast<int>(p.dqk), static_cast<int>(p.dv));
    if (static_cast<size_t>(ly.total) * sizeof(float) > 227 * 1024) return false;
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return al(p.v) && al(p.z) && al(p.out);
}

template <int R>
cudaError_t m3_chunk_launch_split(const M3Params& p, cudaStream_t stream) {
    constexpr int QS = kQR / R;
    const int64_t bh = p.batch * p.heads;
    const int n_chunks = static_cast<int>((p.len + QS - 1) / QS);
    const int64_t np = p.dqk * p.dv;
    const int N = static_cast<int>(p.dqk), P = static_cast<int>(p.dv);
    const size_t smem_ds = static_cast<size_t>(CkLayout(N, P, kCkDs).total) * sizeof(float);
    const size_t smem_out = static_cast<size_t>(CkLayout(N, P, kCkOut).total) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(m3_chunk_ds_kernel<R>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_ds));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(m3_chunk_out_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem_out));
    if (e != cudaSuccess) return e;
    cudaMemPool_t pool = nullptr;
    if ((e = device_workspace_pool(&pool)) != cudaSuccess) return e;
    const size_t units = static_cast<size_t>(bh) * n_chunks;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, units * (np + 1) * sizeof(float) + 256, pool, stream);
    if (e != cudaSuccess) return e;
    CkWs ws;
    ws.st = static_cast<float*>(raw);
    ws.decay = ws.st + units * np;
    const dim3 grid(static_cast<unsigned>(n_chunks), static_cast<unsigned>(bh));
    m3_chunk_ds_kernel<R><<<grid, kCkThreads, smem_ds, stream>>>(p, ws, n_chunks);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess) {
        const unsigned slices = static_cast<unsigned>((np / 4 + kCkThreads - 1) / kCkThreads);
        m3_chunk_state_kernel<<<dim3(static_cast<unsigned>(bh), slices), kCkThreads, 0, stream>>>(
            p, ws, n_chunks);
        note_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        m3_chunk_out_kernel<R><<<grid, kCkThreads, smem_out, stream>>>(p, ws, n_chunks);
        note_launch();
        e = cudaGetLastError();
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

cudaError_t m3_chunk_launch(const M3Params& p, cudaStream_t stream) {
    const int R = p.psi ? static_cast<int>(p.rank) : 1;
    const CkLayout ly(static_cast<int>(p.dqk), static_cast<int>(p.dv));
    const size_t smem = static_cast<size_t>(ly.total) * sizeof(float);
    // The chunk-parallel form (every (batch*head, chunk) its own CTA, at the
    // cost of a second staging pass and a state round trip through memory)
    // measured faster than the sequential form (one CTA per (batch, head)) on
    // every benchmarked shape (config 2 1.81 vs 2.19 ms, config 3 23.2 vs 30.2,
    // config 4a 7.8 vs 17.4); the sequential form remains for single-chunk
    // sequences.  The kKnobM3ChunkForm override forces one or the other.
    bool split = p.len > kQR / R;  // more than one chunk of (step, rank) rows
    if (const int f = kernel_override(kKnobM3ChunkForm)) split = f == 2;
    if (split && (p.dqk * p.dv) % 4 == 0)
        return R == 4 ? m3_chunk_launch_split<4>(p, stream)
             : R == 2 ? m3_chunk_launch_split<2>(p, stream)
                      : m3_chunk_launch_split<1>(p, stream);
    auto kern = R == 4 ? m3_chunk_kernel<4> : R == 2 ? m3_chunk_kernel<2> : m3_chunk_kernel<1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<dim3(static_cast<unsigned>(p.batch * p.heads)), kCkThreads, smem, stream>>>(p);
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
