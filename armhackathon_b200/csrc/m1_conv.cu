// Causal depthwise conv1d + SiLU over (batch, dim, len) rows: the Mamba-1
// mixer's input prologue (HF transformers MambaMixer: conv1d with padding
// kernel-1, sliced to the sequence, then the activation), in one pass.
//
//   out[b, d, t] = silu(bias[d] + sum_{j < K} w[d, j] * x[b, d, t - (K-1) + j])
// with x = 0 before the start (or taken from a K-1 step history when given).
//
// A thread produces 4 consecutive steps of one row from one 16-byte load of
// its own steps plus the previous 16 bytes (K <= 4 lookback), so each input
// element is read once from DRAM (the neighbour's load hits L1/L2).
#include <cstdint>

#include "common.cuh"

namespace b200scan {

namespace {

template <int K>
__global__ void m1_conv_silu_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    const float* __restrict__ bias, float* __restrict__ out,
                                    int64_t rows, int64_t dim, int64_t len) {
    const int64_t quads = len / 4;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * quads) return;
    const int64_t row = i / quads, t0 = (i % quads) * 4;
    const int64_t d = row % dim;
    const float* xr = x + row * len;
    const float4 cur = __ldg(reinterpret_cast<const float4*>(xr + t0));
    const float4 prv = t0 > 0 ? __ldg(reinterpret_cast<const float4*>(xr + t0 - 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float win[8] = {prv.x, prv.y, prv.z, prv.w, cur.x, cur.y, cur.z, cur.w};
    float wk[K];
#pragma unroll
    for (int j = 0; j < K; ++j) wk[j] = __ldg(w + d * K + j);
    const float b0 = bias ? __ldg(bias + d) : 0.f;
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float acc = b0;
#pragma unroll
        for (int j = 0; j < K; ++j) acc = fmaf(wk[j], win[4 + e - (K - 1) + j], acc);
        o[e] = silu_f(acc);
    }
    *reinterpret_cast<float4*>(out + row * len + t0) = make_float4(o[0], o[1], o[2], o[3]);
}

// Any K and length: one thread per output element.
__global__ void m1_conv_silu_scalar(const float* __restrict__ x, const float* __restrict__ w,
                                    const float* __restrict__ bias, float* __restrict__ out,
                                    int64_t rows, int64_t dim, int64_t len, int K) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * len) return;
    const int64_t row = i / len, t = i % len, d = row % dim;
    float acc = bias ? bias[d] : 0.f;
    for (int j = 0; j < K; ++j) {
        const int64_t s = t - (K - 1) + j;
        if (s >= 0) acc = fmaf(w[d * K + j], x[row * len + s], acc);
    }
    out[i] = silu_f(acc);
}

}  // namespace

cudaError_t m1_conv_silu_launch(const float* x, const float* w, const float* bias, float* out,
                                int64_t batch, int64_t dim, int64_t len, int K, cudaStream_t stream) {
    const int64_t rows = batch * dim;
    const bool vec = len % 4 == 0 && K >= 1 && K <= 4 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    if (vec) {
        const int64_t n = rows * (len / 4);
        const unsigned g = static_cast<unsigned>((n + 255) / 256);
        switch (K) {
            case 1: m1_conv_silu_kernel<1><<<g, 256, 0, stream>>>(x, w, bias, out, rows, dim, len); break;
            case 2: m1_conv_silu_kernel<2><<<g, 256, 0, stream>>>(x, w, bias, out, rows, dim, len); break;
            case 3: m1_conv_silu_kernel<3><<<g, 256, 0, stream>>>(x, w, bias, out, rows, dim, len); break;
            default: m1_conv_silu_kernel<4><<<g, 256, 0, stream>>>(x, w, bias, out, rows, dim, len); break;
        }
    } else {
        const int64_t n = rows * len;
        m1_conv_silu_scalar<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(x, w, bias, out, rows,
                                                                                     dim, len, K);
    }
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
