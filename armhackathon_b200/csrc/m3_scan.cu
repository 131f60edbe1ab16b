// Mamba-3 SISO / MIMO scans on sm_100a.
//
// Recurrence (reference kernel/arm-scan-core/src/mamba3/scalar.rs:50-196 and
// mimo.rs:98-284), per (batch, head), state S (dv x dqk), traversal step i
// (time t = i, or L-1-i when reverse; "next" = the following traversal step):
//   lam = sigmoid(trap_t); gamma = dt_t * lam
//   scale = gamma + dt_next * (1 - sigmoid(trap_next))   (0 term at the end)
//   alpha = exp(adt_t)
//   q_r, k_r = rope(q_r + q_bias_r), rope(k_r + k_bias_r)
//     SISO: interleaved lane pairs (2i, 2i+1); MIMO: split halves (i, i+dqk/2)
//   x_r = psi_r * v (MIMO) or v (SISO, rank 1)
//   y_r = alpha * (q_r . S^T) + gamma * sum_r2 (q_r . k_r2) x_r2 + D * x_r
//         (SISO: y = alpha * (q . S^T) + (D + gamma * q.k) * v)
//   S   = alpha * S + scale * sum_r x_r (x) k_r
//   out = SISO: y * silu(z);  MIMO: sum_r phi_r * silu(z * zeta_r) * y_r
//
// m3_sequential_kernel: one CTA per (batch, head), 16 warps, S held in
// registers (warp w owns rows p = w + 16j, lane l owns columns n = l + 32jj).
// Each step, the CTA first stages the rotated q/k, the projected x and the
// gates in shared memory (double-buffered, one barrier per step), then every
// warp reduces its rows' q.S^T with shuffles and updates them.
#include "common.cuh"
#include "m3_scan.h"

namespace b200scan {

namespace {

constexpr int kM3Threads = 512;
constexpr int kM3Warps = kM3Threads / 32;
constexpr int kMaxDv = 128;
constexpr int kMaxDqk = 256;
constexpr int kMaxRank = 8;
constexpr int kRowsPerWarp = kMaxDv / kM3Warps;  // 8
constexpr int kColsPerLane = kMaxDqk / 32;       // 8

struct StepBuf {
    float* qr;    // [R][dqk]
    float* kr;    // [R][dqk]
    float* x;     // [R][dv]
    float* zz;    // [dv]
    float* gate;  // gamma, scale, alpha
};

__device__ __forceinline__ StepBuf step_buf(float* base, int which, int R, int dqk, int dv) {
    const int per = 2 * R * dqk + R * dv + dv + 4;
    float* b = base + which * per;
    StepBuf s;
    s.qr = b;
    s.kr = b + R * dqk;
    s.x = b + 2 * R * dqk;
    s.zz = s.x + R * dv;
    s.gate = s.zz + dv;
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <bool MIMO>
__global__ void __launch_bounds__(kM3Threads, 1) m3_sequential_kernel(M3Params p) {
    extern __shared__ float sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t bh = blockIdx.x;
    const int64_t H = p.heads, L = p.len;
    const int64_t bi = bh / H, h = bh % H;
    const int dv = static_cast<int>(p.dv), dqk = static_cast<int>(p.dqk);
    const int R = MIMO ? static_cast<int>(p.rank) : 1;
    const int half = dqk / 2;
    const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
    const int64_t gate_base = (bi * H + h) * L;

    float S[kRowsPerWarp][kColsPerLane];
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j)
#pragma unroll
        for (int jj = 0; jj < kColsPerLane; ++jj) S[j][jj] = 0.f;

    for (int64_t i = 0; i < L; ++i) {
        const int64_t t = p.reverse ? L - 1 - i : i;
        StepBuf sb = step_buf(sm, static_cast<int>(i & 1), R, dqk, dv);
        // ---- stage: rotated q/k, projected x, z, gates -------------------
        const int64_t qk_off = (bi * L + t) * R * dqk;
        const int64_t cs_off = ((bi * L + t) * H + h) * half;
        for (int idx = tid; idx < R * half; idx += kM3Threads) {
            const int r = idx / half, pi = idx % half;
            const float cs = p.cos[cs_off + pi], sn = p.sin[cs_off + pi];
            const int i0 = MIMO ? pi : 2 * pi, i1 = MIMO ? pi + half : 2 * pi + 1;
            const float* qrow = p.q + qk_off + r * dqk;
            const float* krow = p.k + qk_off + r * dqk;
            const float* qb = p.q_bias + (h * R + r) * dqk;
            const float* kb = p.k_bias + (h * R + r) * dqk;
            float a0 = qrow[i0] + qb[i0], a1 = qrow[i1] + qb[i1];
            sb.qr[r * dqk + i0] = a0 * cs - a1 * sn;
            sb.qr[r * dqk + i1] = a0 * sn + a1 * cs;
            a0 = krow[i0] + kb[i0];
            a1 = krow[i1] + kb[i1];
            sb.kr[r * dqk + i0] = a0 * cs - a1 * sn;
            sb.kr[r * dqk + i1] = a0 * sn + a1 * cs;
        }
        const int64_t v_off = ((bi * L + t) * H + h) * dv;
        for (int pp = tid; pp < dv; pp += kM3Threads) {
            const float vv = p.v[v_off + pp];
            if (MIMO) {
                for (int r = 0; r < R; ++r) sb.x[r * dv + pp] = p.psi[(h * R + r) * dv + pp] * vv;
            } else {
                sb.x[pp] = vv;
            }
            if (p.z) sb.zz[pp] = p.z[v_off + pp];
        }
        if (tid == 0) {
            const int64_t g = gate_base + t;
            const float gamma = p.dt[g] * sigmoid_f(p.trap[g]);
            float shifted = 0.f;
            if (i + 1 < L) {
                const int64_t nx = p.reverse ? g - 1 : g + 1;
                shifted = p.dt[nx] * (1.f - sigmoid_f(p.trap[nx]));
            }
            sb.gate[0] = gamma;
            sb.gate[1] = gamma + shifted;
            sb.gate[2] = expf(p.adt[g]);
        }
        __syncthreads();

        // ---- consume ------------------------------------------------------
        const float gamma = sb.gate[0], scale = sb.gate[1], alpha = sb.gate[2];
        float gram[MIMO ? kMaxRank * kMaxRank : 1];
        for (int a = 0; a < R; ++a)
            for (int b2 = 0; b2 < R; ++b2) {
                float s = 0.f;
                for (int n = lane; n < dqk; n += 32) s = fmaf(sb.qr[a * dqk + n], sb.kr[b2 * dqk + n], s);
                s = warp_sum(s);
                if (MIMO) gram[a * kMaxRank + b2] = s; else gram[0] = s;
            }
#pragma unroll
        for (int j = 0; j < kRowsPerWarp; ++j) {
            const int pr = warp + kM3Warps * j;
            if (pr >= dv) break;
            float out_v = 0.f;
            for (int r = 0; r < R; ++r) {
                float dot = 0.f;
#pragma unroll
                for (int jj = 0; jj < kColsPerLane; ++jj) {
                    const int n = lane + 32 * jj;
                    if (n < dqk) dot = fmaf(sb.qr[r * dqk + n], S[j][jj], dot);
                }
                dot = warp_sum(dot);
                float y;
                if (MIMO) {
                    float dg = 0.f;
                    for (int r2 = 0; r2 < R; ++r2) dg = fmaf(gram[r * kMaxRank + r2], sb.x[r2 * dv + pr], dg);
                    y = alpha * dot + gamma * dg + dsk * sb.x[r * dv + pr];
                    const float ph = p.phi[(h * R + r) * dv + pr];
                    if (p.z) out_v += ph * silu_f(sb.zz[pr] * p.zeta[(h * R + r) * dv + pr]) * y;
                    else out_v += ph * y;
                } else {
                    y = alpha * dot + (dsk + gamma * gram[0]) * sb.x[pr];
                    out_v = p.z ? y * silu_f(sb.zz[pr]) : y;
                }
            }
            if (lane == 0) p.out[((bi * H + h) * L + t) * dv + pr] = out_v;
#pragma unroll
            for (int jj = 0; jj < kColsPerLane; ++jj) {
                const int n = lane + 32 * jj;
                if (n < dqk) {
                    float upd = 0.f;
                    for (int r = 0; r < R; ++r) upd = fmaf(sb.x[r * dv + pr], sb.kr[r * dqk + n], upd);
                    S[j][jj] = fmaf(alpha, S[j][jj], scale * upd);
                }
            }
        }
        if (!MIMO && p.last_bx && i + 1 == L) {
            for (int n = tid; n < dqk; n += kM3Threads)
                p.last_bx[bh * dqk + n] = scale * sb.kr[n];
        }
    }

    if (p.last_state) {
#pragma unroll
        for (int j = 0; j < kRowsPerWarp; ++j) {
            const int pr = warp + kM3Warps * j;
            if (pr >= dv) break;
#pragma unroll
            for (int jj = 0; jj < kColsPerLane; ++jj) {
                const int n = lane + 32 * jj;
                if (n < dqk) p.last_state[(bh * dv + pr) * dqk + n] = S[j][jj];
            }
        }
    }
}

}  // namespace

bool m3_shape_supported(int64_t dv, int64_t dqk, int64_t rank) {
    return dv >= 1 && dv <= kMaxDv && dqk >= 2 && dqk <= kMaxDqk && rank >= 1 &&
           rank <= kMaxRank;
}

cudaError_t m3_scan_launch(const M3Params& p, int backend, cudaStream_t stream) {
    // backend 1 ("scalar") and shapes the chunked kernel does not cover run
    // the sequential kernel; everything else the chunked dual form.
    if (backend == 3) {
        if (!m3_tc_applicable(p)) return cudaErrorNotSupported;
        return m3_tc_launch(p, stream);
    }
    if (backend != 1 && m3_chunk_applicable(p)) return m3_chunk_launch(p, stream);
    const bool mimo = p.psi != nullptr;
    const int R = mimo ? static_cast<int>(p.rank) : 1;
    const size_t per = 2 * R * p.dqk + R * p.dv + p.dv + 4;
    const size_t smem = 2 * per * sizeof(float);
    auto kern = mimo ? m3_sequential_kernel<true> : m3_sequential_kernel<false>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const dim3 grid(static_cast<unsigned>(p.batch * p.heads));
    kern<<<grid, kM3Threads, smem, stream>>>(p);
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
