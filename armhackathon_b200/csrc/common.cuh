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

// Counts kernel launches made by this library (host side, all threads);
// read through arm_scan_kernel_launches().  Every launcher calls it once per
// kernel it starts.
void note_launch();


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

__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Fast softplus for the hot kernels (same threshold contract as softplus_f).
// y = e^x by ex2.approx (relative error ~2^-22); softplus = log1p(y):
//   y < 0.1  : the alternating series y - y^2/2 + y^3/3 - y^4/4 + y^5/5,
//              truncation error < y^6/6 <= 1.7e-7 of the result;
//   y >= 0.1 : ln2 * lg2.approx(1 + y), absolute error ~2^-22 on a result
//              >= 0.095, i.e. relative error < 3e-6.
__device__ __forceinline__ float softplus_fast(float x) {
    if (x > 20.f) return x;
    const float y = ex2_approx(x * kLog2e);
    float ser = fmaf(y, 0.2f, -0.25f);
    ser = fmaf(y, ser, 1.f / 3.f);
    ser = fmaf(y, ser, -0.5f);
    ser = fmaf(y, ser, 1.f);
    ser *= y;
    const float lg = lg2_approx(1.f + y) * 0.6931471805599453f;
    return y < 0.1f ? ser : lg;
}

// Fast silu: x * 1/(1 + e^-x) with ex2.approx and rcp.approx (each ~1 ulp);
// for x < -87 the exponential overflows to +inf and the result is -0, the
// correctly rounded limit.
__device__ __forceinline__ float silu_fast(float x) {
    return x * rcp_approx(1.f + ex2_approx(-x * kLog2e));
}

// Packed fp32x2 arithmetic (PTX ISA 8.6, sm_100a): one instruction computes
// two independent IEEE fp32 results with round-to-nearest, identical to two
// scalar FFMA/FMUL.  Halves the FMA-pipe issue count of the scan's inner loop.
// Operands are packed into 64-bit register pairs inside the asm (mov.b64
// {lo, hi}), which ptxas resolves by register allocation, not arithmetic.
#ifdef B200SCAN_SCALAR_PAIRS
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    return make_float2(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    return make_float2(a.x * b.x, a.y * b.y);
}
#else
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
#endif

// exp2 of two values on the FMA pipe (relieves the MUFU unit).
// Method: Cody-Waite style split x = n + f with n = round(x) obtained by adding
// 1.5*2^23 (the sum's low mantissa bits are round(x) as an integer), f in
// [-1/2, 1/2]; 2^f by a degree-6 polynomial whose coefficients were fitted in
// this project by iteratively reweighted least squares on Chebyshev nodes
// (max relative error 9.6e-8 in fp32 Horner form, below ex2.approx's ~2^-22);
// 2^n is applied by adding n << 23 to the bit pattern, done with one integer
// multiply-add on the bits of the rounded sum.  Inputs below -125 are clamped
// (2^-125 ~ 2.4e-38 stands in for ex2.approx.ftz's flush to zero).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -125.f);
    x.y = fmaxf(x.y, -125.f);
    const float2 one = make_float2(1.f, 1.f);
    const float2 magic = make_float2(12582912.f, 12582912.f);
    const float2 t = ffma2(x, one, magic);
    const float2 n = ffma2(t, one, make_float2(-12582912.f, -12582912.f));
    const float2 f = ffma2(n, make_float2(-1.f, -1.f), x);
    float2 p = make_float2(1.5345810970757157e-4f, 1.5345810970757157e-4f);
    p = ffma2(p, f, make_float2(1.3399930903688073e-3f, 1.3399930903688073e-3f));
    p = ffma2(p, f, make_float2(9.618489071726799e-3f, 9.618489071726799e-3f));
    p = ffma2(p, f, make_float2(5.550328642129898e-2f, 5.550328642129898e-2f));
    p = ffma2(p, f, make_float2(0.24022646248340607f, 0.24022646248340607f));
    p = ffma2(p, f, make_float2(0.6931471824645996f, 0.6931471824645996f));
    p = ffma2(p, f, one);
    const unsigned tx = __float_as_uint(t.x), ty = __float_as_uint(t.y);
    return make_float2(__uint_as_float(tx * 8388608u + __float_as_uint(p.x)),
                       __uint_as_float(ty * 8388608u + __float_as_uint(p.y)));
}

// ---- programmatic dependent launch (sm_90+) --------------------------------
// A kernel launched with launch_pdl may start while its stream predecessor is
// still running; it calls griddep_wait() before touching anything the
// predecessor writes (that returns once the predecessor grid has completed and
// its memory is visible).  griddep_launch_dependents() lets the next
// PDL-launched kernel be scheduled early.  Both are no-ops in a kernel that
// was launched plainly.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Kernel-selection overrides for tests and measurements, set through
// arm_scan_set_kernel_override (process-wide; 0 everywhere means the
// default dispatch).
enum KernelKnob {
    kKnobM1Kernel = 0,    // 0 auto, 1 lane, 2 row-tile, 3 block-chunked, 4 row-tile with time split
    kKnobM1Segments = 1,  // 0 auto, else the segment count of the lane / time-split kernels
    kKnobM1BidirShared = 2,  // 0 shared first pass (default), 1 two independent traversals
    kKnobM3TcSplit = 3,   // 0 fused tensor-core kernel, 1 three-launch form
    kKnobM3ChunkForm = 4, // 0 auto, 1 sequential, 2 chunk-parallel (fp32 chunk kernels)
    kKnobPdl = 5,         // 0 programmatic dependent launch on, 1 off
    kKnobCount = 6,
};
int kernel_override(int knob);
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                       Args&&... args) {
    return launch_pdl_smem(kernel, grid, block, 0, stream, static_cast<Args&&>(args)...);
}

}  // namespace b200scan
