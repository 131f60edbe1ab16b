// Mamba-1 selective scan, row-sequential kernel: the default when there are
// enough (batch, channel) rows to fill the GPU without splitting time.
//
// A warp owns RPW = 32/LPR rows of one (batch, B/C group); the LPR lanes of a
// row split its 16 states (SPL = 16/LPR each) and walk the whole sequence in
// blocks of 4 steps, keeping h in registers from the first step to the last.
// No segment fold, no output fix-up, no block barrier: per (step, state) the
// work is one exp2 (MUFU), two multiplies and two FMAs.  Per block, the
// partial outputs of a row's LPR lanes are summed with xor-shuffles and the
// softplus of the 4 steps is computed once (by one lane per step) and
// broadcast.
//
// Every global read goes through a per-warp cp.async ring DEPTH blocks deep:
// per block, 16-byte copies of delta/u/z for each row and of B/C for each of
// the 16 states (4 consecutive steps), so a lane reads its states' 4 steps of
// B or C with one LDS.128.  Requires len % 4 == 0 and 16-byte aligned rows
// (the dispatcher falls back to the time-split kernel otherwise).
#include <cstdint>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kRsWarps = 4;
constexpr int kRsDepth = 8;

__device__ __forceinline__ void rs_cp16(void* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void rs_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void rs_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

template <int LPR>
struct RsLayout {
    static constexpr int RPW = 32 / LPR;          // rows per warp
    static constexpr int SPL = 16 / LPR;          // states per lane
    static constexpr int X_F = RPW * 12;          // [row][delta4, u4, z4]
    static constexpr int SLOT_F = X_F + 2 * 16 * 4;  // + [B,C][state][4 steps]
    static constexpr int WARP_F = kRsDepth * SLOT_F;
};

template <int LPR, bool REV>
__global__ void __launch_bounds__(kRsWarps * 32) m1_rowseq_kernel(M1Params p, int tiles_per_group,
                                                                  int n_tiles) {
    using LY = RsLayout<LPR>;
    constexpr int RPW = LY::RPW, SPL = LY::SPL, SLOT_F = LY::SLOT_F;
    extern __shared__ float4 smem4[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    float* ring = reinterpret_cast<float*>(smem4) + wib * LY::WARP_F;
    const int r = lane / LPR, q = lane % LPR;
    const int L = static_cast<int>(p.len), N = static_cast<int>(p.state);
    const int gsz = static_cast<int>(p.dim / p.groups);
    const int n_blk = L / 4;
    const int warp_id = blockIdx.x * kRsWarps + wib;
    const int n_warps = gridDim.x * kRsWarps;

    for (int tile = warp_id; tile < n_tiles; tile += n_warps) {
        const int bg = tile / tiles_per_group, jt = tile - bg * tiles_per_group;
        const int rem = gsz - jt * RPW;
        const int n_rows = rem < RPW ? rem : RPW;
        const int64_t row0 = static_cast<int64_t>(bg) * gsz + static_cast<int64_t>(jt) * RPW;
        const int64_t bc0 = static_cast<int64_t>(bg) * N * L;
        const bool active = r < n_rows;
        const int64_t row = row0 + (active ? r : 0);
        const int64_t d = row % p.dim;

        // copies of block blk into its ring slot (one commit group)
        auto issue = [&](int blk) {
            if (blk < n_blk) {
                float* slot = ring + (blk % kRsDepth) * SLOT_F;
                const int t0 = REV ? L - 4 * blk - 4 : 4 * blk;  // time of element 0
#pragma unroll
                for (int i = lane; i < 3 * RPW; i += 32) {
                    const int rr = i / 3, a = i - rr * 3;
                    const float* src = a == 0 ? p.delta : a == 1 ? p.u : p.z;
                    const bool ok = rr < n_rows && src != nullptr;
                    rs_cp16(slot + rr * 12 + a * 4, ok ? src + (row0 + rr) * L + t0 : p.u, ok);
                }
                const int arr = lane >> 4, n = lane & 15;
                const bool ok = n < N;
                const float* src = arr == 0 ? p.B : p.C;
                rs_cp16(slot + LY::X_F + (arr * 16 + n) * 4, ok ? src + bc0 + n * L + t0 : p.B, ok);
            }
            rs_commit();
        };

        float h[SPL], al[SPL];
#pragma unroll
        for (int j = 0; j < SPL; ++j) {
            const int n = q * SPL + j;
            const bool ok = active && n < N;
            al[j] = ok ? p.A[d * N + n] * kLog2e : 0.f;
            h[j] = (ok && p.h0) ? p.h0[row * N + n] : 0.f;
        }
        const float bias = p.delta_bias ? p.delta_bias[d] : 0.f;
        const float dsk = p.d_skip ? p.d_skip[d] : 0.f;
        float* orow = p.out + row * L;

#pragma unroll
        for (int i = 0; i < kRsDepth - 1; ++i) issue(i);
        for (int blk = 0; blk < n_blk; ++blk) {
            issue(blk + kRsDepth - 1);
            rs_wait<kRsDepth - 1>();
            __syncwarp();
            const float* slot = ring + (blk % kRsDepth) * SLOT_F;
            // storage element e holds time t0 + e; traversal step k is e = k
            // (forward) or 3 - k (reverse)
            const float4 dv4 = *reinterpret_cast<const float4*>(slot + r * 12);
            const float4 uv4 = *reinterpret_cast<const float4*>(slot + r * 12 + 4);
            float dv[4] = {dv4.x, dv4.y, dv4.z, dv4.w};
            float uv[4] = {uv4.x, uv4.y, uv4.z, uv4.w};
            if (REV) {
                float t;
                t = dv[0]; dv[0] = dv[3]; dv[3] = t; t = dv[1]; dv[1] = dv[2]; dv[2] = t;
                t = uv[0]; uv[0] = uv[3]; uv[3] = t; t = uv[1]; uv[1] = uv[2]; uv[2] = t;
            }
            // softplus once per step: lane q takes steps k with k % LPR == q
            float dts[4 / LPR > 0 ? 4 / LPR : 1];
#pragma unroll
            for (int m = 0; m < 4 / LPR; ++m) {
                const int k = q + m * LPR;
                float v = k == 0 ? dv[0] : k == 1 ? dv[1] : k == 2 ? dv[2] : dv[3];
                v += bias;
                if (p.delta_softplus) v = softplus_fast(v);
                dts[m] = v;
            }
            float dt[4], du[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                dt[k] = __shfl_sync(0xffffffffu, dts[k / LPR], (lane & ~(LPR - 1)) + (k % LPR));
                du[k] = dt[k] * uv[k];
            }
            float y[4] = {0.f, 0.f, 0.f, 0.f};
            // all exps of the block first, as one burst of independent MUFU
            // ops, so their latency overlaps instead of stalling each FMA
            float a[SPL][4];
#pragma unroll
            for (int j = 0; j < SPL; ++j)
#pragma unroll
                for (int k = 0; k < 4; ++k) a[j][k] = ex2_approx(dt[k] * al[j]);
#pragma unroll
            for (int j = 0; j < SPL; ++j) {
                const int n = q * SPL + j;
                float4 b4 = *reinterpret_cast<const float4*>(slot + LY::X_F + n * 4);
                float4 c4 = *reinterpret_cast<const float4*>(slot + LY::X_F + (16 + n) * 4);
                float bb[4] = {b4.x, b4.y, b4.z, b4.w}, cc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int e = REV ? 3 - k : k;
                    h[j] = fmaf(a[j][k], h[j], du[k] * bb[e]);
                    y[k] = fmaf(cc[e], h[j], y[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
#pragma unroll
                for (int o = 1; o < LPR; o <<= 1) y[k] += __shfl_xor_sync(0xffffffffu, y[k], o);
            }
            // lane q writes the steps k with k % LPR == q
            if (active) {
                const float4 zv4 = *reinterpret_cast<const float4*>(slot + r * 12 + 8);
                float zv[4] = {zv4.x, zv4.y, zv4.z, zv4.w};
#pragma unroll
                for (int m = 0; m < 4 / LPR; ++m) {
                    const int k = q + m * LPR;
                    const int e = REV ? 3 - k : k;
                    float yk = y[0];
#pragma unroll
                    for (int kk = 1; kk < 4; ++kk)
                        if (kk == k) yk = y[kk];
                    const float uk = k == 0 ? uv[0] : k == 1 ? uv[1] : k == 2 ? uv[2] : uv[3];
                    const float ze = e == 0 ? zv[0] : e == 1 ? zv[1] : e == 2 ? zv[2] : zv[3];
                    float out = fmaf(dsk, uk, yk);
                    if (p.z) out *= silu_fast(ze);
                    const int t = REV ? L - 4 * blk - 4 + e : 4 * blk + e;
                    __stcs(orow + t, out);
                }
            }
            __syncwarp();
        }
        rs_wait<0>();
        if (active && p.last_state) {
#pragma unroll
            for (int j = 0; j < SPL; ++j) {
                const int n = q * SPL + j;
                if (n < N) p.last_state[row * N + n] = h[j];
            }
        }
        __syncwarp();
    }
}

template <int LPR>
cudaError_t launch_rowseq(const M1Params& p, cudaStream_t stream) {
    using LY = RsLayout<LPR>;
    const int64_t gsz = p.dim / p.groups;
    const int64_t tiles_per_group = (gsz + LY::RPW - 1) / LY::RPW;
    const int64_t n_tiles = p.batch * p.groups * tiles_per_group;
    const size_t smem = sizeof(float) * kRsWarps * LY::WARP_F;
    auto kern = p.reverse ? m1_rowseq_kernel<LPR, true> : m1_rowseq_kernel<LPR, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRsWarps * 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t want = (n_tiles + kRsWarps - 1) / kRsWarps;
    const int64_t cap = static_cast<int64_t>(sms) * per_sm;
    kern<<<dim3(static_cast<unsigned>(want < cap ? want : cap)), kRsWarps * 32, smem, stream>>>(
        p, static_cast<int>(tiles_per_group), static_cast<int>(n_tiles));
    note_launch();
    return cudaGetLastError();
}

}  // namespace

bool m1_rowseq_applicable(const M1Params& p) {
    return p.state <= 16 && p.len % 4 == 0 && p.len <= (INT32_MAX / 4) &&
           p.state * p.len <= INT32_MAX && m1_pointers_aligned16(p);
}

cudaError_t m1_rowseq_launch(const M1Params& p, int lanes_per_row, cudaStream_t stream) {
    if (lanes_per_row == 1) return launch_rowseq<1>(p, stream);
    if (lanes_per_row == 2) return launch_rowseq<2>(p, stream);
    return launch_rowseq<4>(p, stream);
}

}  // namespace b200scan
