// Mamba-3 mixer prologue: everything the reference's Mamba3Mixer.forward
// does between in_proj and the scan call (apps/mamba3_lm/block.py:146-177),
// in one pass over the in_proj output.
//
// One row of `proj` (batch, step) is laid out as the checkpoint fixes it
// (block.py:116-121): [z (H*P), x (H*P), B (R*N), C (R*N), dd_dt (H),
// dd_A (H), trap (H), angles (NA)] with one B/C group.  Per row the op:
//   z, x           -> copied out contiguous (batch, len, H, P)
//   B, C           -> RMSNorm over N per rank, times the norm weight
//                     (block.py:78-82): k = norm(B), q = norm(C) (block.py:179-180)
//   dd_dt          -> DT = softplus(dd_dt + dt_bias)      (block.py:166)
//   dd_A           -> A = min(-heavy_tail(dd_A), -A_floor) (block.py:52-62, 164-165)
//                     ADT = A * DT                         (block.py:167)
//   DT, ADT, trap  -> transposed to (batch, H, len)        (block.py:158, 168-169)
//   angles         -> copied out contiguous (batch, len, NA); the scan reads
//                     them broadcast over heads             (block.py:174)
//
// A CTA owns 32 consecutive steps of one batch row, so the (batch, H, len)
// gate writes are 32-step runs and every copy is a coalesced sweep.  The op
// moves bytes only: its roofline is HBM (read one proj row, write the same
// number of floats back).
#include <cstdint>

#include "common.cuh"
#include "m3_mixer.h"

namespace b200scan {

namespace {

constexpr int kMixSteps = 32;    // steps per CTA
constexpr int kMixThreads = 256;

__device__ __forceinline__ float softplus_ref(float x) {
    // torch.nn.functional.softplus, beta 1, threshold 20
    return x > 20.f ? x : log1pf(expf(x));
}

template <bool VEC>
__global__ void __launch_bounds__(kMixThreads) m3_mixer_prologue_kernel(MixerParams p) {
    const int64_t L = p.len, H = p.heads, HP = p.heads * p.headdim, RN = p.rank * p.d_state;
    const int64_t W = 2 * HP + 2 * RN + 3 * H + p.n_angles;
    const int64_t o_b = 2 * HP, o_c = o_b + RN, o_dt = o_c + RN, o_a = o_dt + H, o_tr = o_a + H,
                  o_ang = o_tr + H;
    const int64_t b = blockIdx.y;
    const int64_t l0 = static_cast<int64_t>(blockIdx.x) * kMixSteps;
    const int rows = static_cast<int>(L - l0 < kMixSteps ? L - l0 : kMixSteps);
    const float* src = p.proj + (b * L + l0) * W;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // z, x: each row's first 2HP floats, halves to their own tensors; a
    // row's columns are spread over the CTA, four loads in flight per thread
    if (VEC) {
        const int hp4 = static_cast<int>(HP / 4);
        for (int r = 0; r < rows; ++r) {
            const float4* s4 = reinterpret_cast<const float4*>(src + r * W);
            float4* z4 = reinterpret_cast<float4*>(p.z + (b * L + l0 + r) * HP);
            float4* x4 = reinterpret_cast<float4*>(p.x + (b * L + l0 + r) * HP);
            for (int c0 = tid; c0 < 2 * hp4; c0 += 4 * kMixThreads) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int c = c0 + u * kMixThreads;
                    if (c < 2 * hp4) v[u] = __ldcs(s4 + c);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int c = c0 + u * kMixThreads;
                    if (c < hp4)
                        __stcs(z4 + c, v[u]);
                    else if (c < 2 * hp4)
                        __stcs(x4 + (c - hp4), v[u]);
                }
            }
        }
    } else {
        for (int r = 0; r < rows; ++r) {
            const float* sr = src + r * W;
            float* zr = p.z + (b * L + l0 + r) * HP;
            float* xr = p.x + (b * L + l0 + r) * HP;
            for (int64_t c = tid; c < 2 * HP; c += kMixThreads) {
                const float v = __ldcs(sr + c);
                if (c < HP)
                    __stcs(zr + c, v);
                else
                    __stcs(xr + (c - HP), v);
            }
        }
    }

    // gates: lane = step, so each warp writes one head's 32-step run
    for (int64_t i = tid; i < H * kMixSteps; i += kMixThreads) {
        const int64_t h = i / kMixSteps;
        const int r = static_cast<int>(i % kMixSteps);
        if (r >= rows) continue;
        const float* row = src + r * W;
        const float dt = softplus_ref(row[o_dt + h] + p.dt_bias[h]);
        const float da = row[o_a + h];
        // heavy_tail(x) = max(x, 0) + 1 / (1 - min(x, 0))
        const float ht = fmaxf(da, 0.f) + 1.f / (1.f - fminf(da, 0.f));
        const float a = fminf(-ht, -p.a_floor);
        const int64_t o = (b * H + h) * L + l0 + r;
        p.dt[o] = dt;
        p.adt[o] = a * dt;
        p.trap[o] = row[o_tr + h];
    }

    // angles
    for (int64_t i = tid; i < static_cast<int64_t>(rows) * p.n_angles; i += kMixThreads) {
        const int64_t r = i / p.n_angles, c = i % p.n_angles;
        p.angles[(b * L + l0 + r) * p.n_angles + c] = src[r * W + o_ang + c];
    }

    // RMSNorm of B (-> k) and C (-> q): one warp per (row, B|C, rank) group
    const int64_t groups = static_cast<int64_t>(rows) * 2 * p.rank;
    const int N = static_cast<int>(p.d_state);
    for (int64_t gi = warp; gi < groups; gi += kMixThreads / 32) {
        const int64_t r = gi / (2 * p.rank);
        const int which = static_cast<int>((gi / p.rank) % 2);  // 0: B, 1: C
        const int64_t rk = gi % p.rank;
        const float* g = src + r * W + (which ? o_c : o_b) + rk * N;
        float ss = 0.f;
        for (int n = lane; n < N; n += 32) ss = fmaf(g[n], g[n], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rstd = 1.f / sqrtf(ss / static_cast<float>(N) + p.eps);
        const float* w = which ? p.c_norm_w : p.b_norm_w;
        float* dst = (which ? p.q : p.k) + ((b * L + l0 + r) * p.rank + rk) * N;
        for (int n = lane; n < N; n += 32) dst[n] = g[n] * rstd * w[n];
    }
}

}  // namespace

cudaError_t m3_mixer_prologue_launch(const MixerParams& p, cudaStream_t stream) {
    if (p.batch == 0 || p.len == 0) return cudaSuccess;
    const int64_t HP = p.heads * p.headdim, RN = p.rank * p.d_state;
    const int64_t W = 2 * HP + 2 * RN + 3 * p.heads + p.n_angles;
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool vec = W % 4 == 0 && HP % 4 == 0 && al16(p.proj) && al16(p.z) && al16(p.x);
    const dim3 grid(static_cast<unsigned>((p.len + kMixSteps - 1) / kMixSteps),
                    static_cast<unsigned>(p.batch));
    if (vec)
        m3_mixer_prologue_kernel<true><<<grid, kMixThreads, 0, stream>>>(p);
    else
        m3_mixer_prologue_kernel<false><<<grid, kMixThreads, 0, stream>>>(p);
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
