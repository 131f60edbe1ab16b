// Mamba-3 RoPE angle pre-pass on the GPU.
//
// theta[b, t, h, p] = sum_{s <= t} tanh(angle[b, s, h, p]) * pi * dt[b, h, s]
// cos/sin[b, t, h, p] = cos/sin(theta) for p < n_angles, and (1, 0) -- the
// identity rotation -- for n_angles <= p < dqk/2.  Same contract as the
// reference's python/arm_scan/mamba3.py:41-89 (angles_to_cos_sin), whose
// prefix sum runs in torch; here it is a two-phase chunked scan:
//   phase 1: per (batch*head, chunk of kAgChunk steps, pair) the chunk's sum
//            of increments -> workspace;
//   phase 2: each (batch*head, chunk, pair) adds the sums of the earlier
//            chunks, then walks its chunk writing cos/sin.
// Reads of angles are coalesced over pairs (the innermost axis).
#include <climits>
#include <cstdint>

#include "common.cuh"
#include "m3_angles.h"

namespace b200scan {

namespace {

constexpr int kAgChunk = 128;
constexpr float kPi = 3.14159265358979323846f;

// Loads of a group of kAgUnroll steps are all issued before any of its
// arithmetic (and, in phase 2, before its stores), so each group costs one
// memory round trip.
constexpr int kAgUnroll = 8;

__device__ __forceinline__ int64_t angle_phys(const AngleParams& a, int64_t t) {
    if (!a.col_major) return t;
    const int64_t rows = a.len / a.grid_w;
    return (t % rows) * a.grid_w + t / rows;
}

// HG heads per thread (HG > 1 only for head-shared angles): the angle row
// and its tanh are loaded and computed once for HG heads, whose chains run
// side by side; per head the arithmetic and its order are those of HG = 1.
template <int HG>
__global__ void angle_chunk_sums(AngleParams a, float* ws) {
    // threadIdx.y: one of blockDim.y (batch*head) groups sharing the CTA
    const int64_t bh0 = (static_cast<int64_t>(blockIdx.y) * blockDim.y + threadIdx.y) * HG;
    if (bh0 >= a.batch * a.heads) return;
    const int c = blockIdx.x;
    const int p = threadIdx.x;
    if (p >= a.n_angles) return;
    const int64_t b = bh0 / a.heads, h0 = bh0 % a.heads;
    const int64_t t0 = static_cast<int64_t>(c) * kAgChunk;
    const int64_t t1 = t0 + kAgChunk < a.len ? t0 + kAgChunk : a.len;
    const float* ang = a.angles_shared ? a.angles + (b * a.len) * a.n_angles + p
                                       : a.angles + ((b * a.len) * a.heads + h0) * a.n_angles + p;
    const int64_t ang_step = a.angles_shared ? a.n_angles : a.heads * a.n_angles;
    const float* dt = a.dt + (b * a.heads + h0) * a.len;
    float s[HG];
#pragma unroll
    for (int k = 0; k < HG; ++k) s[k] = 0.f;
    for (int64_t t = t0; t < t1; t += kAgUnroll) {
        float av[kAgUnroll], dv[HG][kAgUnroll];
#pragma unroll
        for (int u = 0; u < kAgUnroll; ++u) {
            const bool in = t + u < t1;
            const int64_t pt = in ? angle_phys(a, t + u) : 0;
            av[u] = in ? __ldg(ang + pt * ang_step) : 0.f;
#pragma unroll
            for (int k = 0; k < HG; ++k) dv[k][u] = in ? __ldg(dt + k * a.len + pt) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kAgUnroll; ++u) {
            const float tv = tanhf(av[u]) * kPi;
#pragma unroll
            for (int k = 0; k < HG; ++k) s[k] = fmaf(tv, dv[k][u], s[k]);
        }
    }
    const int nc = gridDim.x;
#pragma unroll
    for (int k = 0; k < HG; ++k) ws[((bh0 + k) * nc + c) * a.n_angles + p] = s[k];
}

template <int HG>
__global__ void angle_chunk_write(AngleParams a, const float* ws) {
    // threadIdx.y: one of blockDim.y (batch*head) groups sharing the CTA
    const int64_t bh0 = (static_cast<int64_t>(blockIdx.y) * blockDim.y + threadIdx.y) * HG;
    if (bh0 >= a.batch * a.heads) return;
    const int c = blockIdx.x;
    const int p = threadIdx.x;
    if (p >= a.half) return;
    const int64_t b = bh0 / a.heads, h0 = bh0 % a.heads;
    const int64_t t0 = static_cast<int64_t>(c) * kAgChunk;
    const int64_t t1 = t0 + kAgChunk < a.len ? t0 + kAgChunk : a.len;
    const int64_t out_step = a.heads * a.half;
    float* cs_out = a.cos + ((b * a.len) * a.heads + h0) * a.half + p;
    float* sn_out = a.sin + ((b * a.len) * a.heads + h0) * a.half + p;
    if (p >= a.n_angles) {
        for (int64_t t = t0; t < t1; ++t)
#pragma unroll
            for (int k = 0; k < HG; ++k) {
                cs_out[t * out_step + k * a.half] = 1.f;
                sn_out[t * out_step + k * a.half] = 0.f;
            }
        return;
    }
    const int nc = gridDim.x;
    float theta[HG];
#pragma unroll
    for (int k = 0; k < HG; ++k) {
        theta[k] = 0.f;
        for (int j = 0; j < c; ++j) theta[k] += __ldg(ws + ((bh0 + k) * nc + j) * a.n_angles + p);
    }
    const float* ang = a.angles_shared ? a.angles + (b * a.len) * a.n_angles + p
                                       : a.angles + ((b * a.len) * a.heads + h0) * a.n_angles + p;
    const int64_t ang_step = a.angles_shared ? a.n_angles : a.heads * a.n_angles;
    const float* dt = a.dt + (b * a.heads + h0) * a.len;
    for (int64_t t = t0; t < t1; t += kAgUnroll) {
        float av[kAgUnroll], dv[HG][kAgUnroll];
#pragma unroll
        for (int u = 0; u < kAgUnroll; ++u) {
            const bool in = t + u < t1;
            const int64_t pt = in ? angle_phys(a, t + u) : 0;
            av[u] = in ? __ldg(ang + pt * ang_step) : 0.f;
#pragma unroll
            for (int k = 0; k < HG; ++k) dv[k][u] = in ? __ldg(dt + k * a.len + pt) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kAgUnroll; ++u) {
            if (t + u >= t1) break;
            const float tv = tanhf(av[u]) * kPi;
#pragma unroll
            for (int k = 0; k < HG; ++k) {
                theta[k] = fmaf(tv, dv[k][u], theta[k]);
                float sn, cs;
                sincosf(theta[k], &sn, &cs);
                cs_out[(t + u) * out_step + k * a.half] = cs;
                sn_out[(t + u) * out_step + k * a.half] = sn;
            }
        }
    }
}

}  // namespace

size_t angle_workspace_bytes(int64_t batch, int64_t heads, int64_t len, int64_t n_angles) {
    const int64_t chunks = (len + kAgChunk - 1) / kAgChunk;
    return static_cast<size_t>(batch * heads * chunks * n_angles) * sizeof(float);
}

cudaError_t angle_launch(const AngleParams& a, float* ws, cudaStream_t stream) {
    const int64_t chunks = (a.len + kAgChunk - 1) / kAgChunk;
    if (chunks > INT32_MAX || a.batch * a.heads > 65535) return cudaErrorInvalidValue;
    // head-shared angles: 4 heads per thread when the head count allows
    const bool g4 = a.angles_shared && a.heads % 4 == 0;
    const int hg = g4 ? 4 : 1;
    const int t1 = static_cast<int>((a.n_angles + 31) / 32 * 32);
    const int t2 = static_cast<int>((a.half + 31) / 32 * 32);
    // at least 2 warps per CTA (one warp per CTA would cap an SM at its CTA
    // slots, half its warps)
    const int by = t2 < 64 ? 64 / t2 : 1;
    const int64_t groups = a.batch * a.heads / hg;
    const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>((groups + by - 1) / by));
    if (a.n_angles > 0) {  // no rotated pairs: the write pass alone gives (1, 0)
        if (g4)
            angle_chunk_sums<4><<<grid, dim3(t1, by), 0, stream>>>(a, ws);
        else
            angle_chunk_sums<1><<<grid, dim3(t1, by), 0, stream>>>(a, ws);
        note_launch();
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (g4)
        angle_chunk_write<4><<<grid, dim3(t2, by), 0, stream>>>(a, ws);
    else
        angle_chunk_write<1><<<grid, dim3(t2, by), 0, stream>>>(a, ws);
    note_launch();
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Its chunk sums live in this fixed device array
// instead of a caller workspace; every GPU that loads the library holds it
// (4 MiB) until the process exits.  Host code must not pass the symbol itself
// to a kernel: on the host it only names a stand-in, so its device address is
// looked up with cudaGetSymbolAddress, with the calling device current, on
// every call.  The lookup is cheap, and looking it up each time means the
// address is always the one of the current context (a cached address would
// go stale after cudaDeviceReset or under another context on the device).
namespace {

static __device__ __align__(256) float g_angle_scratch[kAngleNoAllocMaxFloats];

}  // namespace

cudaError_t angle_noalloc_launch(const AngleParams& a, cudaStream_t stream, bool* too_big) {
    const size_t floats = angle_workspace_bytes(a.batch, a.heads, a.len, a.n_angles) / sizeof(float);
    *too_big = floats > static_cast<size_t>(kAngleNoAllocMaxFloats);
    if (*too_big) return cudaSuccess;
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_angle_scratch);
    if (e != cudaSuccess) return e;
    // Nothing needs clearing: phase 1 writes every chunk sum phase 2 reads.
    return angle_launch(a, static_cast<float*>(ptr), stream);
}

}  // namespace b200scan
