// Diagonal correction of the non-causal Mamba-3 aggregation.
//
// Unrolled, a forward scan gives y_t = sum_{s <= t} M[t,s] (q_t . k_s) v_s and
// a reverse scan the same over s >= t; both count the s == t term
// (D + gamma_t (q_t . k_t)) v_t, gated by silu(z_t).  The non-causal result
// is forward + reverse - that term (reference python/arm_scan/
// mamba3_noncausal.py:53-98 states the identity; the composition there is
// eager torch).  Here the scans accumulate into one output in place and this
// kernel subtracts the term, `count` times (once per traversal ordering of
// an SS2D grid), reading q, k, v, z, dt, trap at each token once.  q . k is
// rotation invariant (both rotate by the step's angle), so it is computed
// from the unrotated, bias-added vectors.
#include <cstdint>

#include "common.cuh"
#include "m3_scan.h"

namespace b200scan {

namespace {

// One warp per (batch, step, head): lanes split dqk for the dot product,
// then dv for the update.
__global__ void m3_diag_sub_kernel(M3Params p, float count) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t H = p.heads, L = p.len, N = p.dqk, P = p.dv;
    if (warp >= p.batch * L * H) return;
    const int64_t h = warp % H, t = (warp / H) % L, b = warp / (H * L);
    const float* q = p.q + (b * L + t) * N;
    const float* k = p.k + (b * L + t) * N;
    float dot = 0.f;
    for (int64_t n = lane; n < N; n += 32)
        dot = fmaf(q[n] + p.q_bias[h * N + n], k[n] + p.k_bias[h * N + n], dot);
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const int64_t g = (b * H + h) * L + t;
    const float gamma = p.dt[g] * sigmoid_f(p.trap[g]);
    const float coef = count * (fmaf(gamma, dot, p.d_skip ? p.d_skip[h] : 0.f));
    const int64_t row = ((b * L + t) * H + h) * P;
    for (int64_t i = lane; i < P; i += 32) {
        float d = coef * p.v[row + i];
        if (p.z) d *= silu_f(p.z[row + i]);
        p.out[row + i] -= d;
    }
}

}  // namespace

cudaError_t m3_diag_sub_launch(const M3Params& p, int count, cudaStream_t stream) {
    const int64_t warps = p.batch * p.len * p.heads;
    m3_diag_sub_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(p, static_cast<float>(count));
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
