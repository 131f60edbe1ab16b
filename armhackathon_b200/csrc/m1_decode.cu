// Mamba-1 single-token state update (decode step).
//
// For each (batch, channel): dt = softplus(dt + bias) (optional),
// h_n <- exp(dt A_n) h_n + dt x B_n in place, y = sum_n C_n h_n + D x,
// times silu(z).  The same recurrence step as the scan (reference
// kernel/arm-scan-core/src/scalar.rs:11-89 at one time step), for
// token-by-token generation from a cached state: the state is read and
// written once, so the step is bound by that traffic and by launch latency.
// One thread per (batch, channel); B/C (batch, [groups,] state) are shared by
// the channels of a group and read through the cache.
#include <cstdint>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kDecThreads = 128;

__global__ void __launch_bounds__(kDecThreads) m1_decode_kernel(M1Params p, float* state) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kDecThreads + threadIdx.x;
    const int64_t D = p.dim, N = p.state, G = p.groups;
    if (row >= p.batch * D) return;
    const int64_t b = row / D, d = row % D, g = d / (D / G);
    float dt = p.delta[row] + (p.delta_bias ? p.delta_bias[d] : 0.f);
    if (p.delta_softplus) dt = softplus_f(dt);
    const float x = p.u[row];
    const float dtx = dt * x;
    const float* A = p.A + d * N;
    const float* Bv = p.B + (b * G + g) * N;
    const float* Cv = p.C + (b * G + g) * N;
    float* h = state + row * N;
    float y = 0.f;
    for (int64_t n = 0; n < N; ++n) {
        const float hn = fmaf(expf(dt * A[n]), h[n], dtx * __ldg(Bv + n));
        h[n] = hn;
        y = fmaf(__ldg(Cv + n), hn, y);
    }
    if (p.d_skip) y = fmaf(p.d_skip[d], x, y);
    if (p.z) y *= silu_f(p.z[row]);
    p.out[row] = y;
}

}  // namespace

cudaError_t m1_decode_launch(const M1Params& p, float* state, cudaStream_t stream) {
    const int64_t rows = p.batch * p.dim;
    m1_decode_kernel<<<static_cast<unsigned>((rows + kDecThreads - 1) / kDecThreads), kDecThreads, 0,
                       stream>>>(p, state);
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
