// Mamba-1 selective scan on sm_100a.
//
// Recurrence (reference kernel/arm-scan-core/src/scalar.rs:11-89), per
// (batch b, channel d), state n, traversal step i (time t = i, or L-1-i when
// reverse):
//   dt   = softplus(delta[t] + bias[d])           (or delta + bias)
//   h_n  = exp(dt * A[d,n]) * h_n + dt * u[t] * B[g(d), n, t]
//   y[t] = sum_n C[g(d), n, t] * h_n  (+ D[d] * u[t])  (* silu(z[t]))
//
// Chunked kernel layout.  One CTA of 256 threads owns DC consecutive
// (batch, channel) rows; thread (c, s) = (tid % DC, tid / DC) owns row c and
// a segment of K consecutive traversal steps.  The CTA walks the sequence in
// macro-chunks of T = (256/DC) * K steps.  For every group of 4 states:
//   1. each thread sweeps its K steps from a zero state, keeping h, the
//      running decay product P_n = prod exp(dt*A_n), its partial output, and
//      Q[k][n] = C[t,n] * P_n (registers);
//   2. the per-segment aggregates (P_n, h_n) go to shared memory; one thread
//      per (row, state) folds them in segment order starting from the carry of
//      the previous macro-chunk, leaving each segment's incoming state h_in;
//   3. each thread adds sum_n Q[k][n] * h_in[n] to its outputs.
// So every exp(dt*A) is evaluated exactly once; the carry between segments is
// the exact linear-recurrence composition (h -> P*h + h_loc).
//
// Memory: u, delta, z, out are read/written once as 16-byte vectors along the
// time axis (each thread touches whole 32-byte sectors); B and C rows are
// shared by all rows of a batch and stay L2-resident.  Rows of a CTA may span
// two batches or two B/C groups: every thread resolves its own B/C row.
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kThreads = 256;

template <int K, bool VEC, bool REV>
__device__ __forceinline__ void load_seg(const float* row, int64_t i0, int64_t L,
                                         bool active, float (&v)[K]) {
#pragma unroll
    for (int m = 0; m < K / 4; ++m) {
        // time of element 0 of this 4-vector
        const int64_t t0 = REV ? L - i0 - 4 * m - 4 : i0 + 4 * m;
        float e[4];
        if (VEC) {
            float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
            if (active && t0 >= 0 && t0 < L) q = __ldcs(reinterpret_cast<const float4*>(row + t0));
            e[0] = q.x; e[1] = q.y; e[2] = q.z; e[3] = q.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t t = t0 + j;
                e[j] = (active && t >= 0 && t < L) ? __ldcs(row + t) : 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[4 * m + (REV ? 3 - j : j)] = e[j];
    }
}

// B/C: 4 consecutive times of one state row, cached (shared across rows).
template <bool VEC>
__device__ __forceinline__ float4 load_bc4(const float* row, int64_t t0, int64_t L, bool ok) {
    if (VEC) {
        if (ok && t0 >= 0 && t0 < L) return __ldg(reinterpret_cast<const float4*>(row + t0));
        return make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int64_t t = t0 + j;
        e[j] = (ok && t >= 0 && t < L) ? __ldg(row + t) : 0.f;
    }
    return make_float4(e[0], e[1], e[2], e[3]);
}

template <int K, bool VEC, bool REV>
__device__ __forceinline__ void store_seg(float* row, int64_t i0, int64_t L, bool active,
                                          const float (&v)[K]) {
    if (!active) return;
#pragma unroll
    for (int m = 0; m < K / 4; ++m) {
        const int64_t t0 = REV ? L - i0 - 4 * m - 4 : i0 + 4 * m;
        float e[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) e[j] = v[4 * m + (REV ? 3 - j : j)];
        if (VEC) {
            if (t0 >= 0 && t0 < L)
                __stcs(reinterpret_cast<float4*>(row + t0), make_float4(e[0], e[1], e[2], e[3]));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t t = t0 + j;
                if (t >= 0 && t < L) __stcs(row + t, e[j]);
            }
        }
    }
}

__device__ __forceinline__ float f4_get(const float4& q, int j) {
    return j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
}

template <int DC, int K, bool VEC, bool REV>
__global__ void __launch_bounds__(kThreads, 1) m1_chunked_kernel(M1Params p) {
    constexpr int S = kThreads / DC;  // segments per macro-chunk
    constexpr int T = S * K;          // steps per macro-chunk
    extern __shared__ float4 smem4[];
    float4* aggP = smem4;                                        // [S][DC]
    float4* aggH = smem4 + S * DC;                               // [S][DC]
    float* carry = reinterpret_cast<float*>(smem4 + 2 * S * DC); // [DC][Npad]

    const int tid = threadIdx.x, c = tid % DC, s = tid / DC;
    const int64_t BD = p.batch * p.dim, L = p.len, N = p.state;
    const int Npad = static_cast<int>((N + 3) & ~int64_t(3));
    const int64_t ch0 = static_cast<int64_t>(blockIdx.x) * DC;
    const int64_t ch = ch0 + c;
    const bool active = ch < BD;
    const int64_t chc = active ? ch : 0;
    const int64_t bi = chc / p.dim, d = chc % p.dim;
    const int64_t gsz = p.dim / p.groups;
    const float* urow = p.u + chc * L;
    const float* drow = p.delta + chc * L;
    const float* zrow = p.z ? p.z + chc * L : nullptr;
    float* orow = p.out + chc * L;
    const int64_t bc_off = (bi * p.groups + d / gsz) * N * L;
    const float* Bbase = p.B + bc_off;
    const float* Cbase = p.C + bc_off;
    const float bias = p.delta_bias ? p.delta_bias[d] : 0.f;
    const float dsk = p.d_skip ? p.d_skip[d] : 0.f;

    for (int i = tid; i < DC * Npad; i += kThreads) {
        const int cc = i / Npad, n = i % Npad;
        const int64_t chh = ch0 + cc;
        carry[i] = (p.h0 && chh < BD && n < N) ? p.h0[chh * N + n] : 0.f;
    }
    __syncthreads();

    const int64_t n_macro = (L + T - 1) / T;
    const int n_groups = Npad / 4;
    for (int64_t mc = 0; mc < n_macro; ++mc) {
        const int64_t i0 = mc * T + static_cast<int64_t>(s) * K;  // traversal index
        float dt[K], dtu[K], y[K];
        load_seg<K, VEC, REV>(drow, i0, L, active, dt);
        load_seg<K, VEC, REV>(urow, i0, L, active, dtu);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const bool ok = active && (i0 + k < L);
            float v = dt[k] + bias;
            if (p.delta_softplus) v = softplus_f(v);
            v = ok ? v : 0.f;  // masked steps are the identity: a = 1, b = 0
            y[k] = dsk * dtu[k];
            dt[k] = v;
            dtu[k] = v * dtu[k];
        }

        for (int g = 0; g < n_groups; ++g) {
            const int n0 = 4 * g;
            float al[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                al[j] = (active && n0 + j < N) ? p.A[d * N + n0 + j] * kLog2e : 0.f;
            float h[4] = {0.f, 0.f, 0.f, 0.f};
            float P[4] = {1.f, 1.f, 1.f, 1.f};
            float Q[K][4];
#pragma unroll
            for (int m = 0; m < K / 4; ++m) {
                const int64_t t0 = REV ? L - i0 - 4 * m - 4 : i0 + 4 * m;
                float4 bv[4], cv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const bool okn = active && (n0 + j < N);
                    bv[j] = load_bc4<VEC>(Bbase + (n0 + j) * L, t0, L, okn);
                    cv[j] = load_bc4<VEC>(Cbase + (n0 + j) * L, t0, L, okn);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const int k = 4 * m + kk;
                    const int e = REV ? 3 - kk : kk;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float a = ex2_approx(dt[k] * al[j]);
                        const float bj = f4_get(bv[j], e), cj = f4_get(cv[j], e);
                        h[j] = fmaf(a, h[j], dtu[k] * bj);
                        y[k] = fmaf(cj, h[j], y[k]);
                        P[j] *= a;
                        Q[k][j] = cj * P[j];
                    }
                }
            }
            aggP[s * DC + c] = make_float4(P[0], P[1], P[2], P[3]);
            aggH[s * DC + c] = make_float4(h[0], h[1], h[2], h[3]);
            __syncthreads();
            if (tid < 4 * DC) {
                // fold the S segment aggregates of (row tid/4, state n0 + tid%4)
                float* aP = reinterpret_cast<float*>(aggP);
                float* aH = reinterpret_cast<float*>(aggH);
                float* cr = carry + (tid >> 2) * Npad + n0 + (tid & 3);
                float hc = *cr;
#pragma unroll
                for (int j = 0; j < S; ++j) {
                    const float pj = aP[j * 4 * DC + tid], hj = aH[j * 4 * DC + tid];
                    aH[j * 4 * DC + tid] = hc;
                    hc = fmaf(pj, hc, hj);
                }
                *cr = hc;
            }
            __syncthreads();
            const float4 hin = aggH[s * DC + c];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                y[k] = fmaf(Q[k][0], hin.x, y[k]);
                y[k] = fmaf(Q[k][1], hin.y, y[k]);
                y[k] = fmaf(Q[k][2], hin.z, y[k]);
                y[k] = fmaf(Q[k][3], hin.w, y[k]);
            }
        }

        if (zrow) {
            float zv[K];
            load_seg<K, VEC, REV>(zrow, i0, L, active, zv);
#pragma unroll
            for (int k = 0; k < K; ++k) y[k] *= silu_f(zv[k]);
        }
        store_seg<K, VEC, REV>(orow, i0, L, active, y);
    }

    if (p.last_state) {
        for (int i = tid; i < DC * Npad; i += kThreads) {
            const int cc = i / Npad, n = i % Npad;
            const int64_t chh = ch0 + cc;
            if (chh < BD && n < N) p.last_state[chh * N + n] = carry[i];
        }
    }
}

// Straightforward device restatement of scalar.rs:11-89: one warp per row,
// lanes over states, sequential in time, accurate expf.  Selected with
// backend = 1; used as an independent on-device cross-check.
__global__ void m1_sequential_kernel(M1Params p) {
    const int lane = threadIdx.x & 31;
    const int64_t ch = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t BD = p.batch * p.dim, L = p.len, N = p.state;
    if (ch >= BD) return;
    const int64_t bi = ch / p.dim, d = ch % p.dim;
    const int64_t gsz = p.dim / p.groups;
    const int64_t bc_off = (bi * p.groups + d / gsz) * N * L;
    const float bias = p.delta_bias ? p.delta_bias[d] : 0.f;
    constexpr int kMaxPerLane = 8;  // N <= 256
    float h[kMaxPerLane];
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int64_t n = lane + 32 * j;
        h[j] = (p.h0 && n < N) ? p.h0[ch * N + n] : 0.f;
    }
    for (int64_t i = 0; i < L; ++i) {
        const int64_t t = p.reverse ? L - 1 - i : i;
        float dt = p.delta[ch * L + t] + bias;
        if (p.delta_softplus) dt = softplus_f(dt);
        const float ut = p.u[ch * L + t];
        const float dtu = dt * ut;
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int64_t n = lane + 32 * j;
            if (n < N) {
                const int64_t bc = bc_off + n * L + t;
                h[j] = expf(dt * p.A[d * N + n]) * h[j] + dtu * p.B[bc];
                y = fmaf(p.C[bc], h[j], y);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (lane == 0) {
            if (p.d_skip) y += p.d_skip[d] * ut;
            if (p.z) y *= silu_f(p.z[ch * L + t]);
            p.out[ch * L + t] = y;
        }
    }
    if (p.last_state) {
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int64_t n = lane + 32 * j;
            if (n < N) p.last_state[ch * N + n] = h[j];
        }
    }
}

template <int DC, int K>
cudaError_t launch_chunked(const M1Params& p, cudaStream_t stream) {
    constexpr int S = kThreads / DC;
    const int64_t BD = p.batch * p.dim;
    const int64_t Npad = (p.state + 3) & ~int64_t(3);
    const size_t smem = sizeof(float4) * 2 * S * DC + sizeof(float) * DC * Npad;
    const dim3 grid(static_cast<unsigned>((BD + DC - 1) / DC));
    const bool vec = (p.len % 4 == 0) && m1_pointers_aligned16(p);
    void (*kern)(M1Params);
    if (vec) kern = p.reverse ? m1_chunked_kernel<DC, K, true, true> : m1_chunked_kernel<DC, K, true, false>;
    else kern = p.reverse ? m1_chunked_kernel<DC, K, false, true> : m1_chunked_kernel<DC, K, false, false>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, kThreads, smem, stream>>>(p);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

bool m1_pointers_aligned16(const M1Params& p) {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return al(p.u) && al(p.delta) && al(p.B) && al(p.C) && al(p.out) && (!p.z || al(p.z));
}

int m1_pick_channels_per_cta(int64_t rows) {
    // Widest row tile that still gives >= 2 CTAs per SM on 148 SMs: a wide
    // tile reuses each B/C vector across more rows, a narrow one spreads a
    // short problem over more SMs.
    const int64_t target = 2 * 148;
    if ((rows + 31) / 32 >= target) return 32;
    if ((rows + 15) / 16 >= target) return 16;
    if ((rows + 7) / 8 >= target) return 8;
    return 4;
}

// ---------------------------------------------------------------------------
// Time-split scan for few rows and long sequences (one long sequence has only
// batch*dim rows, too few tiles for the GPU).  The sequence is cut into S
// equal segments, scanned as S times as many rows:
//   1. state-only tile-kernel pass of every segment from a zero state -> h_end;
//   2. per (row, segment) sum of dt over the segment (exact segment decay
//      exp(A * sum dt) per state);
//   3. fold, in traversal order: h_in(s) = exp(A sum dt(prev)) h_in(prev) +
//      h_end(prev), seeded by h0; the final h is last_state;
//   4. full tile-kernel pass of every segment from its h_in.
namespace {

__global__ void m1_seg_dtsum_kernel(M1Params p, int64_t S, int64_t Ls, float* dtsum) {
    // one CTA per (row, segment); dtsum[(b * S + s) * D + d]
    const int64_t bsd = blockIdx.x;  // logical row b' * D + d
    const int64_t bb = bsd / p.dim, d = bsd % p.dim;
    const int64_t b = bb / S, s = bb % S;
    const float* dl = p.delta + (b * p.dim + d) * p.len + s * Ls;
    const float bias = p.delta_bias ? p.delta_bias[d] : 0.f;
    float acc = 0.f;
    for (int64_t t = threadIdx.x; t < Ls; t += blockDim.x) {
        float v = __ldg(dl + t) + bias;
        if (p.delta_softplus) v = softplus_fast(v);  // as the tile kernel's per-step dt
        acc += v;
    }
    __shared__ float red[32];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) dtsum[bsd] = v;
    }
}

__global__ void m1_seg_fold_kernel(M1Params p, int64_t S, const float* hend, const float* dtsum,
                                   float* hin) {
    // one thread per (b, d, n); segments in traversal order
    const int64_t N = p.state, D = p.dim;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= p.batch * D * N) return;
    const int64_t n = i % N, d = (i / N) % D, b = i / (N * D);
    const float a = p.A[d * N + n];
    float h = p.h0 ? p.h0[i] : 0.f;
    for (int64_t k = 0; k < S; ++k) {
        const int64_t s = p.reverse ? S - 1 - k : k;
        const int64_t row = (b * S + s) * D + d;
        hin[row * N + n] = h;
        h = fmaf(expf(a * dtsum[row]), h, hend[row * N + n]);
    }
    if (p.last_state) p.last_state[i] = h;
}

}  // namespace

int m1_timesplit_segments(const M1Params& p) {
    if (kernel_override(kKnobM1Kernel) == 4) {
        const int s = kernel_override(kKnobM1Segments);
        if (s > 1 && p.len % s == 0 && (p.len / s) % 4 == 0) return s;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t tiles = (p.batch * p.dim + 15) / 16;
    // The split runs every exp twice (state pass + rescan), and the tile
    // kernel's throughput per SM is the limit, so it pays only when fewer
    // than half of the SMs would otherwise have a tile (measured: 96 tiles,
    // i.e. one sequence of 1536 channels, gains nothing).
    if (p.state > 16 || 2 * tiles >= sms || p.len < 16384) return 1;
    // about three waves of the two-CTA-per-SM persistent grid
    for (int s = 16; s >= 2; s >>= 1)
        if (tiles * s <= 6 * sms && p.len % s == 0 && (p.len / s) % 4 == 0 && p.len / s >= 2048)
            return s;
    return 1;
}

cudaError_t m1_timesplit_launch(const M1Params& p, int S, cudaStream_t stream) {
    const int64_t Ls = p.len / S, rows = p.batch * p.dim * S;
    const size_t st_bytes = static_cast<size_t>(rows * p.state) * sizeof(float);
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, 2 * st_bytes + static_cast<size_t>(rows) * sizeof(float), pool,
                                stream);
    if (e != cudaSuccess) return e;
    float* hend = static_cast<float*>(raw);
    float* hin = hend + rows * p.state;
    float* dtsum = hin + rows * p.state;
    M1Params q = p;
    q.batch = p.batch * S;
    q.len = Ls;
    q.seg_count = S;
    q.len_full = p.len;
    q.h0 = nullptr;
    q.out = nullptr;  // state only
    q.last_state = hend;
    e = m1_tile_launch(q, 1, stream);
    if (e == cudaSuccess) {
        m1_seg_dtsum_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(p, S, Ls, dtsum);
        note_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        const int64_t n = p.batch * p.dim * p.state;
        m1_seg_fold_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(p, S, hend,
                                                                                     dtsum, hin);
        note_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        q.out = p.out;
        q.h0 = hin;
        q.last_state = nullptr;
        e = m1_tile_launch(q, 1, stream);
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

cudaError_t m1_final_state_launch(const M1Params& p, cudaStream_t stream) {
    M1Params q = p;
    q.out = nullptr;
    q.z = nullptr;
    q.d_skip = nullptr;
    const int S = m1_lane_segments(q);
    if (S > 0) return m1_lane_launch(q, S, stream);
    const bool tile_ok = q.state <= 16 && q.len <= (INT32_MAX / 4) && q.state * q.len <= INT32_MAX;
    return tile_ok ? m1_tile_launch(q, 1, stream) : cudaErrorNotSupported;
}

// Dispatch: backend 1 is the sequential cross-check kernel; otherwise the
// lane kernel where it applies (d_state <= 16, length a multiple of 4,
// 16-byte aligned tensors), the row-tile kernel (with a time split for long
// sequences of few rows) for the other lengths with d_state <= 16, and the
// block-chunked kernel for d_state > 16.
cudaError_t m1_scan_launch(const M1Params& p, int backend, cudaStream_t stream) {
    if (backend == kBackendSequential) {
        const int64_t BD = p.batch * p.dim;
        const int warps_per_block = 4;
        const dim3 grid(static_cast<unsigned>((BD + warps_per_block - 1) / warps_per_block));
        m1_sequential_kernel<<<grid, 32 * warps_per_block, 0, stream>>>(p);
        note_launch();
        return cudaGetLastError();
    }
    const int force = kernel_override(kKnobM1Kernel);
    if (force == 0 || force == 1)
        if (const int S = m1_lane_segments(p)) return m1_lane_launch(p, S, stream);
    const bool tile_ok = p.state <= 16 && p.len <= (INT32_MAX / 4) && p.state * p.len <= INT32_MAX;
    if (tile_ok && force != 3) {
        const int S = m1_timesplit_segments(p);
        if (S > 1 && force != 2) return m1_timesplit_launch(p, S, stream);
        return m1_tile_launch(p, 1, stream);
    }
    switch (m1_pick_channels_per_cta(p.batch * p.dim)) {
        case 32: return launch_chunked<32, 16>(p, stream);
        case 16: return launch_chunked<16, 16>(p, stream);
        case 8: return launch_chunked<8, 16>(p, stream);
        default: return launch_chunked<4, 16>(p, stream);
    }
}

// Whether a bidirectional call takes the shared-first-pass form of the lane
// kernel (wherever that kernel applies and the backend is not the
// sequential cross-check).
static int bidir_shared_segments(const M1Params& fwd, int backend) {
    if (backend == kBackendSequential || kernel_override(kKnobM1BidirShared) == 1) return 0;
    const int force = kernel_override(kKnobM1Kernel);
    if (force != 0 && force != 1) return 0;
    return m1_lane_bidir_segments(fwd);
}

cudaError_t m1_bidir_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                            cudaStream_t stream) {
    if (const int S = bidir_shared_segments(fwd, backend)) return m1_lane_bidir_launch(fwd, bwd, S, stream);
    cudaError_t e = m1_scan_launch(fwd, backend, stream);
    if (e != cudaSuccess) return e;
    return m1_scan_launch(bwd, backend, stream);
}

cudaError_t m1_bidir_states_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                   cudaStream_t stream) {
    M1Params f = fwd, r = bwd;
    f.out = r.out = nullptr;
    f.z = r.z = nullptr;
    f.d_skip = r.d_skip = nullptr;
    if (const int S = bidir_shared_segments(f, backend)) return m1_lane_bidir_launch(f, r, S, stream);
    const cudaError_t e = m1_final_state_launch(f, stream);
    return e != cudaSuccess ? e : m1_final_state_launch(r, stream);
}

namespace {
// Sum over the sequence of dt = softplus(delta + bias) per row, one warp per
// row (the segment-summary fallback where the lane kernel does not apply).
__global__ void m1_dt_sum_kernel(M1Params p, float* out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= p.batch * p.dim) return;
    const float bias = p.delta_bias ? p.delta_bias[row % p.dim] : 0.f;
    const float* d = p.delta + row * p.len;
    float s = 0.f;
    for (int64_t t = lane; t < p.len; t += 32) {
        float v = d[t] + bias;
        if (p.delta_softplus) v = softplus_f(v);
        s += v;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[row] = s;
}
}  // namespace

cudaError_t m1_segment_summary_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                      cudaStream_t stream) {
    M1Params f = fwd, r = bwd;
    f.out = r.out = nullptr;
    f.z = r.z = nullptr;
    f.d_skip = r.d_skip = nullptr;
    r.dt_sum = nullptr;
    if (const int S = bidir_shared_segments(f, backend)) return m1_lane_bidir_launch(f, r, S, stream);
    f.dt_sum = nullptr;
    cudaError_t e = m1_bidir_states_launch(f, r, backend, stream);
    if (e != cudaSuccess) return e;
    const int64_t rows = fwd.batch * fwd.dim;
    m1_dt_sum_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(fwd, fwd.dt_sum);
    note_launch();
    return cudaGetLastError();
}

namespace {
__global__ void m1_add_kernel(float* __restrict__ out, const float* __restrict__ other, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] += other[i];
}
}  // namespace

cudaError_t m1_bidir_sum_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                cudaStream_t stream) {
    // fwd.out receives the sum; bwd.out is ignored
    if (const int S = bidir_shared_segments(fwd, backend)) {
        M1Params r = bwd;
        r.out = fwd.out;
        r.out_acc = 1;
        return m1_lane_bidir_launch(fwd, r, S, stream);
    }
    const int64_t n = fwd.batch * fwd.dim * fwd.len;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    void* tmp = nullptr;
    e = cudaMallocFromPoolAsync(&tmp, static_cast<size_t>(n) * sizeof(float), pool, stream);
    if (e != cudaSuccess) return e;
    M1Params r = bwd;
    r.out = static_cast<float*>(tmp);
    e = m1_bidir_launch(fwd, r, backend, stream);
    if (e == cudaSuccess) {
        m1_add_kernel<<<148 * 8, 256, 0, stream>>>(fwd.out, r.out, n);
        note_launch();
        e = cudaGetLastError();
    }
    const cudaError_t ef = cudaFreeAsync(tmp, stream);
    return e != cudaSuccess ? e : ef;
}

}  // namespace b200scan
