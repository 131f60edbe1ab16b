// Mamba-1 selective scan, two-pass kernel (d_state <= 16, large row counts).
//
// A CTA owns 32 rows of one (batch, B/C group): lane = row, all 16 states
// of the row in registers.  The sequence is walked in chunks of T = 8*K
// steps; warp w owns segment w (K steps) of the chunk.
//   pass 1: every warp sweeps its segment from a zero state and keeps only
//           the end state h_loc and sum(dt) of each row;
//   fold:   warp w starts from the row's carry and folds the aggregates of
//           segments 0..w-1 (decay of a segment = exp2(A*log2e * sum dt),
//           one exp2 per state), giving its incoming state;
//   pass 2: the warp re-sweeps its segment from that state and writes y.
// Every exp(dt*A) is evaluated twice (once per pass) instead of being stored,
// in exchange for no per-step storage, no per-state-group barriers and
// 16 independent state chains per lane.  B and C of the chunk are staged
// once per CTA, transposed to [step][16 states] so a step's values are four
// broadcast LDS.128; the next chunk's B/C copies (cp.async) overlap the
// current chunk.  u, delta and z are read per lane with 16-byte loads.
#include <cstdint>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kTpWarps = 8;
constexpr int kTpK = 12;                   // steps per segment
constexpr int kTpT = kTpWarps * kTpK;      // steps per chunk
constexpr int kTpBcF = kTpT * 16;          // one staged B or C chunk (floats)
constexpr int kTpXS = kTpT + 4;            // padded row stride of staged u/delta
constexpr int kTpXF = 32 * kTpXS;          // one staged u or delta chunk (floats)

__device__ __forceinline__ void tp_cp4(void* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 4 : 0));
}
__device__ __forceinline__ void tp_cp16(void* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void tp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void tp_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

template <bool REV>
__global__ void __launch_bounds__(kTpWarps * 32, 2) m1_twopass_kernel(M1Params p,
                                                                    int tiles_per_group,
                                                                    int n_tiles) {
    extern __shared__ float4 smem4[];
    float* bcs = reinterpret_cast<float*>(smem4);      // [2 bufs][B, C][T][16]
    float* xs = bcs + 2 * 2 * kTpBcF;                   // [2 bufs][delta, u][32 rows][XS]
    float* aggH = xs + 2 * 2 * kTpXF;                   // [warp][16][32 lanes]
    float* aggS = aggH + kTpWarps * 16 * 32;            // [warp][32 lanes] sum dt
    float* carry = aggS + kTpWarps * 32;                // [2 bufs][16][32 lanes]

    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, tid = threadIdx.x;
    const int L = static_cast<int>(p.len), N = static_cast<int>(p.state);
    const int gsz = static_cast<int>(p.dim / p.groups);
    const int n_chunks = (L + kTpT - 1) / kTpT;

    int tile = blockIdx.x;
    if (tile >= n_tiles) return;

    // stage B/C of (tile, chunk) into buffer buf
    auto issue = [&](int tl, int ch, int buf, bool valid) {
        if (valid) {
            const int bg = tl / tiles_per_group;
            {
                // u, delta: 32 rows x T steps, time-ascending 4-vectors
                const int jt = tl - bg * tiles_per_group;
                const int rem = gsz - jt * 32;
                const int nr = rem < 32 ? rem : 32;
                for (int idx = tid; idx < 2 * 32 * (kTpT / 4); idx += kTpWarps * 32) {
                    const int a = idx / (32 * (kTpT / 4));
                    const int rr = (idx / (kTpT / 4)) & 31, m = idx % (kTpT / 4);
                    const int i0 = ch * kTpT + 4 * m;  // traversal index of slot 4m
                    const int t0 = REV ? L - i0 - 4 : i0;
                    const bool ok = rr < nr && t0 >= 0 && t0 < L;
                    const int64_t r = static_cast<int64_t>(bg) * gsz + jt * 32 + rr;
                    const float* src = a == 0 ? p.delta : p.u;
                    tp_cp16(xs + (buf * 2 + a) * kTpXF + rr * kTpXS + 4 * m,
                            ok ? src + r * L + t0 : p.u, ok);
                }
            }
            const float* Bg = p.B + static_cast<int64_t>(bg) * N * L;
            const float* Cg = p.C + static_cast<int64_t>(bg) * N * L;
            float* db = bcs + buf * 2 * kTpBcF;
            float* dc = db + kTpBcF;
            for (int idx = tid; idx < 16 * kTpT; idx += kTpWarps * 32) {
                const int n = idx / kTpT, j = idx - n * kTpT;
                const int it = ch * kTpT + j;
                const bool ok = it < L && n < N;
                const int off = ok ? n * L + (REV ? L - 1 - it : it) : 0;
                tp_cp4(db + j * 16 + n, Bg + off, ok);
                tp_cp4(dc + j * 16 + n, Cg + off, ok);
            }
        }
        tp_commit();
    };

    issue(tile, 0, 0, true);
    int buf = 0;
    while (true) {
        const int bg = tile / tiles_per_group, jt = tile - bg * tiles_per_group;
        const int rem = gsz - jt * 32;
        const int n_rows = rem < 32 ? rem : 32;
        const bool active = lane < n_rows;
        const int64_t row = static_cast<int64_t>(bg) * gsz + jt * 32 + (active ? lane : 0);
        const int64_t d = row % p.dim;
        float al[16];
#pragma unroll
        for (int n = 0; n < 16; ++n) al[n] = (active && n < N) ? p.A[d * N + n] * kLog2e : 0.f;
        const float bias = p.delta_bias ? p.delta_bias[d] : 0.f;
        const float dsk = p.d_skip ? p.d_skip[d] : 0.f;
        const float* zrow = p.z ? p.z + row * L : nullptr;
        float* orow = p.out + row * L;
        if (w == 0) {
#pragma unroll
            for (int n = 0; n < 16; ++n)
                carry[(buf * 16 + n) * 32 + lane] =
                    (p.h0 && active && n < N) ? p.h0[row * N + n] : 0.f;
        }

        for (int ch = 0; ch < n_chunks; ++ch, buf ^= 1) {
            const bool last_chunk = ch + 1 == n_chunks;
            const int ntile = last_chunk ? tile + static_cast<int>(gridDim.x) : tile;
            tp_wait_all();
            __syncthreads();  // chunk's B/C visible; previous chunk fully done
            issue(ntile, last_chunk ? 0 : ch + 1, buf ^ 1, ntile < n_tiles);
            const float* sB = bcs + buf * 2 * kTpBcF;
            const float* sC = sB + kTpBcF;
            const int i0 = ch * kTpT + w * kTpK;  // traversal index of step 0
            const float* xd = xs + (buf * 2 + 0) * kTpXF + lane * kTpXS;
            const float* xu = xs + (buf * 2 + 1) * kTpXF + lane * kTpXS;
            // dt, dt*u of traversal steps i0+k4 .. i0+k4+3 from the staged rows
            // (4-vectors hold times ascending: reverse reads them backward)
            auto load_du = [&](int k4, float (&dv)[4], float (&uv)[4]) {
                const int slot = w * kTpK + k4;
                const float4 d4 = *reinterpret_cast<const float4*>(xd + slot);
                const float4 u4 = *reinterpret_cast<const float4*>(xu + slot);
                const float da[4] = {d4.x, d4.y, d4.z, d4.w}, ua[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int it = i0 + k4 + e;
                    const bool ok = active && it < L;
                    float v = da[REV ? 3 - e : e] + bias;
                    if (p.delta_softplus) v = softplus_fast(v);
                    dv[e] = ok ? v : 0.f;
                    uv[e] = ua[REV ? 3 - e : e];
                }
            };

            // ---- pass 1: end state of the segment from zero, and sum dt
            float h[16];
#pragma unroll
            for (int n = 0; n < 16; ++n) h[n] = 0.f;
            float sdt = 0.f;
#pragma unroll 2
            for (int k4 = 0; k4 < kTpK; k4 += 4) {
                float dv[4], uv[4];
                load_du(k4, dv, uv);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float dt = dv[e], du = dt * uv[e];
                    sdt += dt;
                    const float* bj = sB + (w * kTpK + k4 + e) * 16;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const float4 b4 = *reinterpret_cast<const float4*>(bj + 4 * q4);
                        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int n = 4 * q4 + v;
                            h[n] = fmaf(ex2_approx(dt * al[n]), h[n], du * bb[v]);
                        }
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < 16; ++n) aggH[(w * 16 + n) * 32 + lane] = h[n];
            aggS[w * 32 + lane] = sdt;
            __syncthreads();
            // ---- fold: carry, then segments 0..w-1
#pragma unroll
            for (int n = 0; n < 16; ++n) h[n] = carry[(buf * 16 + n) * 32 + lane];
            for (int j = 0; j < w; ++j) {
                const float s = aggS[j * 32 + lane];
#pragma unroll
                for (int n = 0; n < 16; ++n)
                    h[n] = fmaf(ex2_approx(s * al[n]), h[n], aggH[(j * 16 + n) * 32 + lane]);
            }
            // ---- pass 2: re-sweep from the incoming state, write y
#pragma unroll 2
            for (int k4 = 0; k4 < kTpK; k4 += 4) {
                float dv[4], uv[4], zv[4];
                load_du(k4, dv, uv);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int it = i0 + k4 + e;
                    const bool ok = active && it < L;
                    zv[e] = (ok && zrow) ? __ldcs(zrow + (REV ? L - 1 - it : it)) : 0.f;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float dt = dv[e], du = dt * uv[e];
                    const float* bj = sB + (w * kTpK + k4 + e) * 16;
                    const float* cj = sC + (w * kTpK + k4 + e) * 16;
                    float y0 = 0.f, y1 = 0.f;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const float4 b4 = *reinterpret_cast<const float4*>(bj + 4 * q4);
                        const float4 c4 = *reinterpret_cast<const float4*>(cj + 4 * q4);
                        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                        const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const int n = 4 * q4 + v;
                            h[n] = fmaf(ex2_approx(dt * al[n]), h[n], du * bb[v]);
                            if (v & 1) y1 = fmaf(cc[v], h[n], y1);
                            else y0 = fmaf(cc[v], h[n], y0);
                        }
                    }
                    const int it = i0 + k4 + e;
                    if (active && it < L) {
                        float y = y0 + y1 + dsk * uv[e];
                        if (zrow) y *= silu_fast(zv[e]);
                        __stcs(orow + (REV ? L - 1 - it : it), y);
                    }
                }
            }
            // the outgoing carry goes to the other buffer: slower warps may
            // still be reading this chunk's incoming carry
            if (w == kTpWarps - 1) {
#pragma unroll
                for (int n = 0; n < 16; ++n) carry[((buf ^ 1) * 16 + n) * 32 + lane] = h[n];
            }
            if (last_chunk) {
                __syncthreads();
                if (w == 0 && active && p.last_state) {
#pragma unroll
                    for (int n = 0; n < 16; ++n)
                        if (n < N) p.last_state[row * N + n] = carry[((buf ^ 1) * 16 + n) * 32 + lane];
                }
            }
        }
        tile += gridDim.x;
        if (tile >= n_tiles) break;
        __syncthreads();  // last_state read of carry done before the next tile resets it
    }
    tp_wait_all();
}

}  // namespace

bool m1_twopass_applicable(const M1Params& p) {
    return p.state <= 16 && p.len % 4 == 0 && m1_pointers_aligned16(p) && p.len <= (INT32_MAX / 4) && p.state * p.len <= INT32_MAX;
}

cudaError_t m1_twopass_launch(const M1Params& p, cudaStream_t stream) {
    const int64_t gsz = p.dim / p.groups;
    const int64_t tiles_per_group = (gsz + 31) / 32;
    const int64_t n_tiles = p.batch * p.groups * tiles_per_group;
    if (n_tiles > INT32_MAX) return cudaErrorInvalidValue;
    const size_t smem =
        sizeof(float) * (2 * 2 * kTpBcF + 2 * 2 * kTpXF + kTpWarps * 16 * 32 + kTpWarps * 32 + 2 * 16 * 32);
    auto kern = p.reverse ? m1_twopass_kernel<true> : m1_twopass_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTpWarps * 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t cap = static_cast<int64_t>(sms) * per_sm;
    kern<<<dim3(static_cast<unsigned>(n_tiles < cap ? n_tiles : cap)), kTpWarps * 32, smem,
           stream>>>(p, static_cast<int>(tiles_per_group), static_cast<int>(n_tiles));
    note_launch();
    return cudaGetLastError();
}

}  // namespace b200scan
