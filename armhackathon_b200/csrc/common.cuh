// Shared device helpers for the sm_100a selective-scan kernels.
//
// Numerics contract (reference kernel/arm-scan-core/src/float.rs:24-77):
//   softplus(x) = x for x > 20, else log1p(exp(x))
//   silu(x)     = x / (1 + exp(-x))
//   sigmoid(x)  branch-stable: 1/(1+e^-x) for x >= 0, e^x/(1+e^x) otherwise
// These run once per (batch, channel, step) and use CUDA's accurate expf /
// log1pf.  The per-(step, state) decay exp(dt*A) is the hot transcendental and
// runs on the MUFU unit as exp2(dt * A*log2(e)) via ex2.approx.ftz.f32
// (max relative error ~2^-22), with A pre-scaled once per channel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200scan {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float softplus_f(float x) {
    return x > 20.f ? x : log1pf(expf(x));
}

__device__ __forceinline__ float silu_f(float x) {
    return x / (1.f + expf(-x));
}

__device__ __forceinline__ float sigmoid_f(float x) {
    if (x >= 0.f) return 1.f / (1.f + expf(-x));
    const float e = expf(x);
    return e / (1.f + e);
}

// Packed fp32x2 arithmetic (PTX ISA 8.6, sm_100a): one instruction computes
// two independent IEEE fp32 results with round-to-nearest, identical to two
// scalar FFMA/FMUL.  Halves the FMA-pipe issue count of the scan's inner loop.
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
    return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) |
           __float_as_uint(v.x);
}
__device__ __forceinline__ float2 f2_from(unsigned long long r) {
    return make_float2(__uint_as_float(static_cast<unsigned>(r)),
                       __uint_as_float(static_cast<unsigned>(r >> 32)));
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_from(r);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_from(r);
}

}  // namespace b200scan
