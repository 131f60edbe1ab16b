// Mamba-1 selective scan, fold-free two-pass segmented form.
//
// Same recurrence as m1_tile.cu (reference kernel/arm-scan-core/src/
// scalar.rs:11-89): dt = softplus(delta + bias), h = exp(dt A) h + dt u B,
// y = C.h + D u, times silu(z).  The sequence is cut into S equal segments;
// a thread owns one (row, segment) and walks its steps in order with all
// d_state <= 16 states in registers, so there is no per-chunk fold:
//
//   pass 1: each (row, segment) but the last from a zero state -> h_end,
//           sum of dt; the first segment instead runs the full scan from
//           h0 (its incoming state is known), writing y and its true end;
//   carry:  h_in(s) = exp(A sum dt(prev)) h_in(prev) + h_end(prev) in
//           traversal order, starting from the first segment's end;
//   pass 2: each (row, segment) but the first from h_in, writing y; the
//           last segment writes last_state.
//
// Every exp but those of the first and last segments is computed twice
// (2 (S - 1) / S per element), in exchange for no barriers in the sweeps
// and far fewer instructions per (step, state) than the fold's aggregate
// bookkeeping.  With out == nullptr (final state only) pass 1 covers every
// segment from zero and the carry ends in last_state.  A CTA is 128 rows of one (batch, group)
// and one segment; B and C of the segment are staged in chunks of 64 steps
// by cp.async into a transposed [step][state] slab (one LDS.128 = 4 states
// of a step, broadcast to every row), double-buffered.  u, delta, z are
// read per thread 4 steps at a time, one block ahead.
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kS2Rows = 128;   // threads (rows) per CTA
constexpr int kS2Chunk = 64;   // steps of B/C per staged chunk
// default share of exps on the FMA pipe (see m1_seg2_kernel): pass 2 (kSeg2Poly)
// and pass 1 (kSeg2Poly1, the MUFU-bound one); the two passes' decays then
// differ by the approximations' error (~1e-7 relative), not by design
constexpr int kSeg2Poly = 0;
constexpr int kSeg2Poly1 = 0;
constexpr int kS2Stride = 20;  // floats per staged step (16 states + pad: fewer bank conflicts)

__device__ __forceinline__ void cpa4(float* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 4 : 0));
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cpa_wait1() { asm volatile("cp.async.wait_group 1;\n" ::); }
__device__ __forceinline__ void cpa_wait0() { asm volatile("cp.async.wait_group 0;\n" ::); }

struct Seg2Ws {
    float* hend;   // [S][rows][16]  pass 1 end states (zero start)
    float* hin;    // [S][rows][16]  incoming states
    float* dtsum;  // [S][rows]
};

// 4 consecutive traversal steps of a row, in traversal order.
template <bool REV>
__device__ __forceinline__ float4 ld_steps(const float* row, int64_t L, int64_t it) {
    if (!REV) return __ldg(reinterpret_cast<const float4*>(row + it));
    const float4 v = __ldg(reinterpret_cast<const float4*>(row + (L - 4 - it)));
    return make_float4(v.w, v.z, v.y, v.x);
}

// Sweep modes of one (row block, segment).
enum Seg2Mode {
    kSeg2State = 0,  // from zero: end state + sum of dt
    kSeg2Rescan = 1, // from h_in: y (and last_state on the last segment)
    kSeg2First = 2,  // from h0: y, and the true end state into hend
};

using Seg2Slab = float[2][2][kS2Chunk * kS2Stride];  // [buf][B, C][step][state]

// POLY: 0 every exp on MUFU; 1 states 12-15 (25%), 2 states 8-15 (50%) on the
// FMA pipe (exp2_poly2).
template <int MODE, bool REV, int POLY>
__device__ __forceinline__ void m1_seg2_sweep(const M1Params& p, const Seg2Ws& ws, int S, int64_t Ls,
                                              int s, Seg2Slab& sb) {
    constexpr bool FULL = MODE != kSeg2State;
    const int N = static_cast<int>(p.state);
    const int64_t L = p.len, D = p.dim, G = p.groups, gsz = D / G;
    const int64_t rows_all = p.batch * D;
    const int blocks_per_group = static_cast<int>((gsz + kS2Rows - 1) / kS2Rows);
    const int64_t bg = blockIdx.x / blocks_per_group;  // (batch, group)
    const int jb = blockIdx.x % blocks_per_group;
    const int64_t b = bg / G, g = bg % G;
    const int64_t dd = g * gsz + static_cast<int64_t>(jb) * kS2Rows + threadIdx.x;  // channel
    const bool active = static_cast<int64_t>(jb) * kS2Rows + threadIdx.x < gsz;
    const int64_t row = b * D + (active ? dd : g * gsz);
    const int64_t it0 = static_cast<int64_t>(s) * Ls;  // first traversal step of the segment

    // this row's A * log2 e, bias, D
    float2 a2[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int n0 = 2 * q;
        const float* A = p.A + (row % D) * N;
        a2[q] = make_float2(n0 < N ? A[n0] * kLog2e : 0.f, n0 + 1 < N ? A[n0 + 1] * kLog2e : 0.f);
    }
    const float bias = p.delta_bias ? p.delta_bias[row % D] : 0.f;
    const float dsk = p.d_skip ? p.d_skip[row % D] : 0.f;
    float2 h[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        h[q] = make_float2(0.f, 0.f);
        if (MODE == kSeg2Rescan) {
            const float* hi = ws.hin + (static_cast<int64_t>(s) * rows_all + row) * 16;
            h[q] = make_float2(2 * q < N ? hi[2 * q] : 0.f, 2 * q + 1 < N ? hi[2 * q + 1] : 0.f);
        } else if (MODE == kSeg2First && p.h0) {
            const float* hi = p.h0 + row * N;
            h[q] = make_float2(2 * q < N ? hi[2 * q] : 0.f, 2 * q + 1 < N ? hi[2 * q + 1] : 0.f);
        }
    }

    const float* Bg = p.B + bg * N * L;
    const float* Cg = p.C + bg * N * L;
    // stage chunk c of the segment into buffer buf: element (step j, state n)
    auto stage = [&](int c, int buf) {
        for (int idx = threadIdx.x; idx < kS2Chunk * 16; idx += kS2Rows) {
            const int n = idx / kS2Chunk, j = idx % kS2Chunk;  // coalesced over steps
            const int64_t it = it0 + static_cast<int64_t>(c) * kS2Chunk + j;
            const bool ok = n < N && it < L;
            const int64_t t = ok ? (REV ? L - 1 - it : it) : 0;
            cpa4(&sb[buf][0][j * kS2Stride + n], Bg + (ok ? n * L + t : 0), ok);
            if (FULL) cpa4(&sb[buf][1][j * kS2Stride + n], Cg + (ok ? n * L + t : 0), ok);
        }
        cpa_commit();
    };

    const float* drow = p.delta + row * L;
    const float* urow = p.u + row * L;
    const float* zrow = (FULL && p.z) ? p.z + row * L : nullptr;
    float* orow = FULL ? p.out + row * L : nullptr;
    const int n_chunks = static_cast<int>((Ls + kS2Chunk - 1) / kS2Chunk);
    float dtsum = 0.f;

    stage(0, 0);
    float4 nd = ld_steps<REV>(drow, L, it0), nu = ld_steps<REV>(urow, L, it0);
    float4 nz = zrow ? ld_steps<REV>(zrow, L, it0) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < n_chunks; ++c) {
        const int buf = c & 1;
        if (c + 1 < n_chunks) {
            stage(c + 1, buf ^ 1);
            cpa_wait1();
        } else {
            cpa_wait0();
        }
        __syncthreads();
        const float* sB = sb[buf][0];
        const float* sC = sb[buf][1];
#pragma unroll 1
        for (int j4 = 0; j4 < kS2Chunk; j4 += 4) {
            const int64_t it = it0 + static_cast<int64_t>(c) * kS2Chunk + j4;
            const float4 d4 = nd, u4 = nu, z4 = nz;
            if (j4 + 4 < kS2Chunk || c + 1 < n_chunks) {
                nd = ld_steps<REV>(drow, L, it + 4);
                nu = ld_steps<REV>(urow, L, it + 4);
                if (zrow) nz = ld_steps<REV>(zrow, L, it + 4);
            }
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
            const float zv[4] = {z4.x, z4.y, z4.z, z4.w};
            float yv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float dt = dv[k] + bias;
                if (p.delta_softplus) dt = softplus_fast(dt);
                dtsum += dt;
                const float dtu = dt * uv[k];
                const float2 dt2 = make_float2(dt, dt), du2 = make_float2(dtu, dtu);
                const float* bk = sB + (j4 + k) * kS2Stride;
                const float* ck = sC + (j4 + k) * kS2Stride;
                float2 y2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 bb = *reinterpret_cast<const float4*>(bk + 4 * q4);
                    const float2 x0 = fmul2(dt2, a2[2 * q4]), x1 = fmul2(dt2, a2[2 * q4 + 1]);
                    const bool poly = (POLY == 1 && q4 == 3) || (POLY == 2 && q4 >= 2);
                    const float2 e0 = poly ? exp2_poly2(x0) : make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
                    const float2 e1 = poly ? exp2_poly2(x1) : make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
                    h[2 * q4] = ffma2(e0, h[2 * q4], fmul2(du2, make_float2(bb.x, bb.y)));
                    h[2 * q4 + 1] = ffma2(e1, h[2 * q4 + 1], fmul2(du2, make_float2(bb.z, bb.w)));
                    if (FULL) {
                        const float4 cc = *reinterpret_cast<const float4*>(ck + 4 * q4);
                        y2 = ffma2(make_float2(cc.x, cc.y), h[2 * q4], y2);
                        y2 = ffma2(make_float2(cc.z, cc.w), h[2 * q4 + 1], y2);
                    }
                }
                if (FULL) {
                    float y = y2.x + y2.y + dsk * uv[k];
                    if (zrow) y *= silu_fast(zv[k]);
                    yv[k] = y;
                }
            }
            if (FULL && active && it < L) {
                if (!REV)
                    __stcs(reinterpret_cast<float4*>(orow + it), make_float4(yv[0], yv[1], yv[2], yv[3]));
                else
                    __stcs(reinterpret_cast<float4*>(orow + (L - 4 - it)),
                           make_float4(yv[3], yv[2], yv[1], yv[0]));
            }
        }
        __syncthreads();  // buffer buf is restaged two chunks later
    }
    if (MODE != kSeg2Rescan && active) {
        float* he = ws.hend + (static_cast<int64_t>(s) * rows_all + row) * 16;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            he[2 * q] = h[q].x;
            he[2 * q + 1] = h[q].y;
        }
        ws.dtsum[static_cast<int64_t>(s) * rows_all + row] = dtsum;
    }
    if (FULL && s == S - 1 && p.last_state && active) {
        float* ls = p.last_state + row * N;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (2 * q < N) ls[2 * q] = h[q].x;
            if (2 * q + 1 < N) ls[2 * q + 1] = h[q].y;
        }
    }
}

// Pass 1.  FIRST: segment 0 (blockIdx.y == 0) runs the full scan from h0 and
// the others (1 .. S-2) the state-only sweep; otherwise every segment is
// state-only.
template <bool FIRST, bool REV, int POLY>
__global__ void __launch_bounds__(kS2Rows, 5) m1_seg2_pass1(M1Params p, Seg2Ws ws, int S, int64_t Ls) {
    __shared__ __align__(16) Seg2Slab sb;
    const int s = blockIdx.y;
    if (FIRST && s == 0)
        m1_seg2_sweep<kSeg2First, REV, POLY>(p, ws, S, Ls, 0, sb);
    else
        m1_seg2_sweep<kSeg2State, REV, POLY>(p, ws, S, Ls, s, sb);
}

// Pass 2: segments 1 .. S-1 from their incoming states.
template <bool REV, int POLY>
__global__ void __launch_bounds__(kS2Rows) m1_seg2_pass2(M1Params p, Seg2Ws ws, int S, int64_t Ls) {
    __shared__ __align__(16) Seg2Slab sb;
    m1_seg2_sweep<kSeg2Rescan, REV, POLY>(p, ws, S, Ls, blockIdx.y + 1, sb);
}

// FIRST: segment 0's hend is already its true end state (pass 1 ran it from
// h0), the carry fills h_in of segments 1 .. S-1 and pass 2 writes
// last_state.  Otherwise every hend is from zero, the carry starts at h0 and
// ends in last_state.
template <bool FIRST>
__global__ void m1_seg2_carry_kernel(M1Params p, Seg2Ws ws, int S) {
    const int64_t rows_all = p.batch * p.dim, N = p.state;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows_all * N) return;
    const int64_t row = i / N, n = i % N;
    const float a = p.A[(row % p.dim) * N + n] * kLog2e;
    float h = FIRST ? __ldg(ws.hend + row * 16 + n) : (p.h0 ? p.h0[i] : 0.f);
    for (int k = FIRST ? 1 : 0; k < S; ++k) {  // segments are already in traversal order
        const int64_t sr = static_cast<int64_t>(k) * rows_all + row;
        ws.hin[sr * 16 + n] = h;
        if (FIRST && k == S - 1) break;
        const float ds = __ldg(ws.dtsum + sr), he = __ldg(ws.hend + sr * 16 + n);
        h = fmaf(ex2_approx(a * ds), h, he);
    }
    if (!FIRST && p.last_state) p.last_state[i] = h;
}

}  // namespace

int m1_seg2_segments(const M1Params& p) {
    if (p.state > 16 || p.len % kS2Chunk != 0) return 0;
    if (!m1_pointers_aligned16(p)) return 0;
    if (const char* v = getenv("B200SCAN_M1_SEG2_S")) {  // tuning override
        const int s = atoi(v);
        return (s >= 1 && p.len % s == 0 && (p.len / s) % kS2Chunk == 0) ? s : 0;
    }
    const int64_t rows = p.batch * p.dim;
    // enough (row, segment) threads to fill the GPU several times over, with
    // segments of at least two staged chunks
    int S = 1;
    while (rows * S < 148 * 1024 && p.len % (2 * S) == 0 && p.len / (2 * S) >= 2 * kS2Chunk &&
           (p.len / (2 * S)) % kS2Chunk == 0)
        S *= 2;
    return S;
}

cudaError_t m1_seg2_launch(const M1Params& p, int S, cudaStream_t stream) {
    const int64_t rows = p.batch * p.dim, Ls = p.len / S;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    const size_t st = static_cast<size_t>(S) * rows * 16;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, (2 * st + static_cast<size_t>(S) * rows) * sizeof(float), pool,
                                stream);
    if (e != cudaSuccess) return e;
    Seg2Ws ws;
    ws.hend = static_cast<float*>(raw);
    ws.hin = ws.hend + st;
    ws.dtsum = ws.hin + st;
    const int64_t gsz = p.dim / p.groups;
    const dim3 grid(static_cast<unsigned>(((gsz + kS2Rows - 1) / kS2Rows) * p.batch * p.groups),
                    static_cast<unsigned>(S));
    int poly = kSeg2Poly, poly1 = kSeg2Poly1;
    if (const char* v = getenv("B200SCAN_M1_SEG2_POLY")) poly = atoi(v);
    if (const char* v = getenv("B200SCAN_M1_SEG2_POLY1")) poly1 = atoi(v);
    const bool first = p.out != nullptr;  // out == nullptr: final state only
#define SEG2_PICK(K, PL, ...)                                                                    \
    (PL == 2 ? (p.reverse ? K<__VA_ARGS__ true, 2> : K<__VA_ARGS__ false, 2>)                    \
             : PL == 1 ? (p.reverse ? K<__VA_ARGS__ true, 1> : K<__VA_ARGS__ false, 1>)          \
                       : (p.reverse ? K<__VA_ARGS__ true, 0> : K<__VA_ARGS__ false, 0>))
    auto k1 = first ? SEG2_PICK(m1_seg2_pass1, poly1, true,) : SEG2_PICK(m1_seg2_pass1, poly1, false,);
    auto k2 = SEG2_PICK(m1_seg2_pass2, poly, );
#undef SEG2_PICK
    // pass 1 covers segments 0 .. S-2 when the first one runs in full (all of
    // them for S == 1), every segment otherwise
    const unsigned s1 = first ? static_cast<unsigned>(S > 1 ? S - 1 : 1) : static_cast<unsigned>(S);
    k1<<<dim3(grid.x, s1), kS2Rows, 0, stream>>>(p, ws, S, Ls);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess && (S > 1 || !first)) {
        const int64_t n = rows * p.state;
        const unsigned cg = static_cast<unsigned>((n + 255) / 256);
        if (first)
            m1_seg2_carry_kernel<true><<<cg, 256, 0, stream>>>(p, ws, S);
        else
            m1_seg2_carry_kernel<false><<<cg, 256, 0, stream>>>(p, ws, S);
        note_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && first && S > 1) {
        k2<<<dim3(grid.x, static_cast<unsigned>(S - 1)), kS2Rows, 0, stream>>>(p, ws, S, Ls);
        note_launch();
        e = cudaGetLastError();
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

}  // namespace b200scan
