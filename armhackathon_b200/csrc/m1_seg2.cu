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

constexpr int kS2Rows = 128;   // rows per CTA
constexpr int kS2Chunk = 64;   // steps of B/C per staged chunk
// rows per thread: 2 (half the shared-memory loads per row, 64 threads and
// ~165 registers) measured 13% slower at the prefill shape than 1
#ifndef B200SCAN_SEG2_RPT
#define B200SCAN_SEG2_RPT 1
#endif
constexpr int kS2Rpt = B200SCAN_SEG2_RPT;
// pass 1 asks the compiler for 5 resident CTAs per SM (96 registers; its
// first-segment branch otherwise takes 100 and 4 CTAs).  Pass 2 carries no
// minimum: with an explicit minimum of 1 the compiler spends 196 registers
// (2 CTAs per SM), without one 86.
#ifndef B200SCAN_SEG2_MINB1
#define B200SCAN_SEG2_MINB1 5
#endif
constexpr int kS2MinBlocks1 = B200SCAN_SEG2_MINB1;
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
    kSeg2Bidir = 3,  // from zero, walking forward: the end state and, for the
                     // reverse traversal of the same inputs, the segment's
                     // aggregate from zero (see m1_seg2_pass1_bidir)
};

using Seg2Slab = float[2][2][kS2Chunk * kS2Stride];  // [buf][B, C][step][state]

// One CTA sweeps kS2Rows rows of one (batch, group) over one segment with
// kS2Rows / RPT threads: a thread owns RPT rows (threadIdx.x + r * threads),
// so each shared-memory load of B/C (the same 4 states of a step for every
// row) feeds RPT rows' updates.
// POLY: 0 every exp on MUFU; 1 states 12-15 (25%), 2 states 8-15 (50%) on the
// FMA pipe (exp2_poly2).
template <int MODE, bool REV, int POLY, int RPT>
__device__ __forceinline__ void m1_seg2_sweep(const M1Params& p, const Seg2Ws& ws, int S, int64_t Ls,
                                              int s, Seg2Slab& sb, const Seg2Ws* wsb = nullptr) {
    constexpr bool FULL = MODE != kSeg2State && MODE != kSeg2Bidir;
    constexpr bool BID = MODE == kSeg2Bidir;
    constexpr int T = kS2Rows / RPT;  // threads
    const int N = static_cast<int>(p.state);
    const int64_t L = p.len, D = p.dim, G = p.groups, gsz = D / G;
    const int64_t rows_all = p.batch * D;
    const int blocks_per_group = static_cast<int>((gsz + kS2Rows - 1) / kS2Rows);
    const int64_t bg = blockIdx.x / blocks_per_group;  // (batch, group)
    const int jb = blockIdx.x % blocks_per_group;
    const int64_t b = bg / G, g = bg % G;
    const int64_t it0 = static_cast<int64_t>(s) * Ls;  // first traversal step of the segment

    int64_t row[RPT];
    bool active[RPT];
    float2 a2[RPT][8], h[RPT][8];  // this row's A * log2 e; state
    // BID: running product of the decays since the segment start, and the
    // reverse traversal's aggregate sum_t P_<t * dt_t u_t B_t
    float2 pr[RPT][8], hb[RPT][8];
    float bias[RPT], dsk[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int64_t local = static_cast<int64_t>(jb) * kS2Rows + r * T + threadIdx.x;
        active[r] = local < gsz;
        row[r] = b * D + g * gsz + (active[r] ? local : 0);
        const int64_t ch = row[r] % D;
        const float* A = p.A + ch * N;
#pragma unroll
        for (int q = 0; q < 8; ++q)
            a2[r][q] = make_float2(2 * q < N ? A[2 * q] * kLog2e : 0.f,
                                   2 * q + 1 < N ? A[2 * q + 1] * kLog2e : 0.f);
        bias[r] = p.delta_bias ? p.delta_bias[ch] : 0.f;
        dsk[r] = p.d_skip ? p.d_skip[ch] : 0.f;
    }

    // everything above reads only the op's inputs; under a programmatic
    // dependent launch the incoming states are the first thing that needs
    // the carry kernel finished (a no-op otherwise)
    if (MODE == kSeg2Rescan) griddep_wait();
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const float* hi = MODE == kSeg2Rescan ? ws.hin + (static_cast<int64_t>(s) * rows_all + row[r]) * 16
                          : (MODE == kSeg2First && p.h0) ? p.h0 + row[r] * N
                                                        : nullptr;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            h[r][q] = hi ? make_float2(2 * q < N ? hi[2 * q] : 0.f, 2 * q + 1 < N ? hi[2 * q + 1] : 0.f)
                         : make_float2(0.f, 0.f);
            pr[r][q] = make_float2(1.f, 1.f);
            hb[r][q] = make_float2(0.f, 0.f);
        }
    }

    const float* Bg = p.B + bg * N * L;
    const float* Cg = p.C + bg * N * L;
    // stage chunk c of the segment into buffer buf: element (step j, state n)
    auto stage = [&](int c, int buf) {
        for (int idx = threadIdx.x; idx < kS2Chunk * 16; idx += T) {
            const int n = idx / kS2Chunk, j = idx % kS2Chunk;  // coalesced over steps
            const int64_t it = it0 + static_cast<int64_t>(c) * kS2Chunk + j;
            const bool ok = n < N && it < L;
            const int64_t t = ok ? (REV ? L - 1 - it : it) : 0;
            cpa4(&sb[buf][0][j * kS2Stride + n], Bg + (ok ? n * L + t : 0), ok);
            if (FULL) cpa4(&sb[buf][1][j * kS2Stride + n], Cg + (ok ? n * L + t : 0), ok);
        }
        cpa_commit();
    };

    const bool has_z = FULL && p.z;
    const int n_chunks = static_cast<int>((Ls + kS2Chunk - 1) / kS2Chunk);
    float dtsum[RPT];
    float4 nd[RPT], nu[RPT], nz[RPT];
    stage(0, 0);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        dtsum[r] = 0.f;
        nd[r] = ld_steps<REV>(p.delta + row[r] * L, L, it0);
        nu[r] = ld_steps<REV>(p.u + row[r] * L, L, it0);
        nz[r] = has_z ? ld_steps<REV>(p.z + row[r] * L, L, it0) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
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
            float dv[RPT][4], uv[RPT][4], zv[RPT][4], yv[RPT][4];
            const bool more = j4 + 4 < kS2Chunk || c + 1 < n_chunks;
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                dv[r][0] = nd[r].x, dv[r][1] = nd[r].y, dv[r][2] = nd[r].z, dv[r][3] = nd[r].w;
                uv[r][0] = nu[r].x, uv[r][1] = nu[r].y, uv[r][2] = nu[r].z, uv[r][3] = nu[r].w;
                zv[r][0] = nz[r].x, zv[r][1] = nz[r].y, zv[r][2] = nz[r].z, zv[r][3] = nz[r].w;
                if (more) {
                    nd[r] = ld_steps<REV>(p.delta + row[r] * L, L, it + 4);
                    nu[r] = ld_steps<REV>(p.u + row[r] * L, L, it + 4);
                    if (has_z) nz[r] = ld_steps<REV>(p.z + row[r] * L, L, it + 4);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float2 dt2[RPT], du2[RPT], y2[RPT];
#pragma unroll
                for (int r = 0; r < RPT; ++r) {
                    float dt = dv[r][k] + bias[r];
                    if (p.delta_softplus) dt = softplus_fast(dt);
                    dtsum[r] += dt;
                    const float dtu = dt * uv[r][k];
                    dt2[r] = make_float2(dt, dt);
                    du2[r] = make_float2(dtu, dtu);
                    y2[r] = make_float2(0.f, 0.f);
                }
                const float* bk = sB + (j4 + k) * kS2Stride;
                const float* ck = sC + (j4 + k) * kS2Stride;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 bb = *reinterpret_cast<const float4*>(bk + 4 * q4);
                    float4 cc;
                    if (FULL) cc = *reinterpret_cast<const float4*>(ck + 4 * q4);
                    const bool poly = (POLY == 1 && q4 == 3) || (POLY == 2 && q4 >= 2);
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        const float2 x0 = fmul2(dt2[r], a2[r][2 * q4]), x1 = fmul2(dt2[r], a2[r][2 * q4 + 1]);
                        const float2 e0 = poly ? exp2_poly2(x0) : make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
                        const float2 e1 = poly ? exp2_poly2(x1) : make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
                        const float2 bu0 = fmul2(du2[r], make_float2(bb.x, bb.y));
                        const float2 bu1 = fmul2(du2[r], make_float2(bb.z, bb.w));
                        h[r][2 * q4] = ffma2(e0, h[r][2 * q4], bu0);
                        h[r][2 * q4 + 1] = ffma2(e1, h[r][2 * q4 + 1], bu1);
                        if (BID) {
                            hb[r][2 * q4] = ffma2(pr[r][2 * q4], bu0, hb[r][2 * q4]);
                            hb[r][2 * q4 + 1] = ffma2(pr[r][2 * q4 + 1], bu1, hb[r][2 * q4 + 1]);
                            pr[r][2 * q4] = fmul2(pr[r][2 * q4], e0);
                            pr[r][2 * q4 + 1] = fmul2(pr[r][2 * q4 + 1], e1);
                        }
                        if (FULL) {
                            y2[r] = ffma2(make_float2(cc.x, cc.y), h[r][2 * q4], y2[r]);
                            y2[r] = ffma2(make_float2(cc.z, cc.w), h[r][2 * q4 + 1], y2[r]);
                        }
                    }
                }
                if (FULL) {
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        float y = y2[r].x + y2[r].y + dsk[r] * uv[r][k];
                        if (has_z) y *= silu_fast(zv[r][k]);
                        yv[r][k] = y;
                    }
                }
            }
            if (FULL && it < L) {
#pragma unroll
                for (int r = 0; r < RPT; ++r) {
                    if (!active[r]) continue;
                    float* orow = p.out + row[r] * L;
                    float4* o4 = reinterpret_cast<float4*>(orow + (REV ? L - 4 - it : it));
                    float4 y4 = REV ? make_float4(yv[r][3], yv[r][2], yv[r][1], yv[r][0])
                                    : make_float4(yv[r][0], yv[r][1], yv[r][2], yv[r][3]);
                    if (p.out_acc) {  // summing into an earlier traversal's output
                        const float4 o = __ldcs(o4);
                        y4 = make_float4(o.x + y4.x, o.y + y4.y, o.z + y4.z, o.w + y4.w);
                    }
                    __stcs(o4, y4);
                }
            }
        }
        __syncthreads();  // buffer buf is restaged two chunks later
    }
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        if (!active[r]) continue;
        if (MODE != kSeg2Rescan) {
            float* he = ws.hend + (static_cast<int64_t>(s) * rows_all + row[r]) * 16;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                he[2 * q] = h[r][q].x;
                he[2 * q + 1] = h[r][q].y;
            }
            ws.dtsum[static_cast<int64_t>(s) * rows_all + row[r]] = dtsum[r];
        }
        if (BID) {
            // the reverse traversal visits this segment as its (S - 1 - s)-th
            const int64_t sr = static_cast<int64_t>(S - 1 - s) * rows_all + row[r];
            float* he = wsb->hend + sr * 16;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                he[2 * q] = hb[r][q].x;
                he[2 * q + 1] = hb[r][q].y;
            }
            wsb->dtsum[sr] = dtsum[r];
        }
        if (FULL && s == S - 1 && p.last_state) {
            float* ls = p.last_state + row[r] * N;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (2 * q < N) ls[2 * q] = h[r][q].x;
                if (2 * q + 1 < N) ls[2 * q + 1] = h[r][q].y;
            }
        }
    }
}

// Pass 1.  FIRST: segment 0 (blockIdx.y == 0) runs the full scan from h0 and
// the others (1 .. S-2) the state-only sweep; otherwise every segment is
// state-only.
template <bool FIRST, bool REV, int POLY>
__global__ void __launch_bounds__(kS2Rows / kS2Rpt, kS2MinBlocks1) m1_seg2_pass1(M1Params p, Seg2Ws ws, int S, int64_t Ls) {
    __shared__ __align__(16) Seg2Slab sb;
    griddep_launch_dependents();  // the carry kernel may be scheduled into the tail wave
    const int s = blockIdx.y;
    if (FIRST && s == 0)
        m1_seg2_sweep<kSeg2First, REV, POLY, kS2Rpt>(p, ws, S, Ls, 0, sb);
    else
        m1_seg2_sweep<kSeg2State, REV, POLY, kS2Rpt>(p, ws, S, Ls, s, sb);
}

// Pass 1 of both traversals of the same inputs (bidirectional scan), one
// forward walk per segment with every exp computed once: the forward end
// state from zero as kSeg2State, and the reverse traversal's aggregate of the
// segment from zero, sum_t (prod_{r<t} exp(dt_r A)) dt_t u_t B_t (the running
// product needs multiplies only), written at the reverse traversal's segment
// index into wsb.
template <int POLY>
__global__ void __launch_bounds__(kS2Rows / kS2Rpt, 4)  // 32 more live registers: 4 CTAs
    m1_seg2_pass1_bidir(M1Params p, Seg2Ws ws, Seg2Ws wsb, int S, int64_t Ls) {
    __shared__ __align__(16) Seg2Slab sb;
    griddep_launch_dependents();
    m1_seg2_sweep<kSeg2Bidir, false, POLY, kS2Rpt>(p, ws, S, Ls, blockIdx.y, sb, &wsb);
}

// Pass 2: segments s_off .. S-1 from their incoming states.
template <bool REV, int POLY>
__global__ void __launch_bounds__(kS2Rows / kS2Rpt) m1_seg2_pass2(M1Params p, Seg2Ws ws, int S, int64_t Ls,
                                                                  int s_off) {
    __shared__ __align__(16) Seg2Slab sb;
    m1_seg2_sweep<kSeg2Rescan, REV, POLY, kS2Rpt>(p, ws, S, Ls, blockIdx.y + s_off, sb);
}

// FIRST: segment 0's hend is already its true end state (pass 1 ran it from
// h0), the carry fills h_in of segments 1 .. S-1 and pass 2 writes
// last_state.  Otherwise every hend is from zero, the carry starts at h0 and
// ends in last_state.
template <bool FIRST>
__global__ void m1_seg2_carry_kernel(M1Params p, Seg2Ws ws, int S) {
    const int64_t rows_all = p.batch * p.dim, N = p.state;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    griddep_launch_dependents();  // pass 2 may start its prologue
    griddep_wait();               // pass 1's end states
    if (i >= rows_all * N) return;
    const int64_t row = i / N, n = i % N;
    const float a = p.A[(row % p.dim) * N + n] * kLog2e;
    float h = FIRST ? __ldg(ws.hend + row * 16 + n) : (p.h0 ? p.h0[i] : 0.f);
    // segments are already in traversal order; each group of 8 has all its
    // loads in flight before the serial combine
    const int k_end = FIRST ? S - 1 : S;  // segments whose (dtsum, hend) fold in
    for (int k0 = FIRST ? 1 : 0; k0 < k_end; k0 += 8) {
        float ds[8], he[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int64_t sr = static_cast<int64_t>(k0 + u) * rows_all + row;
            ds[u] = k0 + u < k_end ? __ldg(ws.dtsum + sr) : 0.f;
            he[u] = k0 + u < k_end ? __ldg(ws.hend + sr * 16 + n) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (k0 + u >= k_end) break;
            ws.hin[(static_cast<int64_t>(k0 + u) * rows_all + row) * 16 + n] = h;
            h = fmaf(ex2_approx(a * ds[u]), h, he[u]);
        }
    }
    if (FIRST && S > 1) ws.hin[(static_cast<int64_t>(S - 1) * rows_all + row) * 16 + n] = h;
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
    k1<<<dim3(grid.x, s1), kS2Rows / kS2Rpt, 0, stream>>>(p, ws, S, Ls);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess && (S > 1 || !first)) {
        const int64_t n = rows * p.state;
        const unsigned cg = static_cast<unsigned>((n + 255) / 256);
        e = first ? launch_pdl(m1_seg2_carry_kernel<true>, dim3(cg), dim3(256), stream, p, ws, S)
                  : launch_pdl(m1_seg2_carry_kernel<false>, dim3(cg), dim3(256), stream, p, ws, S);
        note_launch();
    }
    if (e == cudaSuccess && first && S > 1) {
        e = launch_pdl(k2, dim3(grid.x, static_cast<unsigned>(S - 1)), dim3(kS2Rows / kS2Rpt), stream, p,
                       ws, S, Ls, 1);
        note_launch();
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

// Both traversals of the same inputs: fwd (reverse 0) and bwd (reverse 1)
// share every input but out / last_state (and out_acc).  One shared pass 1,
// a carry per direction, a pass 2 per direction over every segment: three
// exps per (step, state) instead of 2 x 2(S-1)/S.  bwd.out == fwd.out with
// bwd.out_acc sums the two outputs in place (bwd's pass 2 runs after fwd's).
// fwd.out == nullptr: final states only (pass 1 and the carries).  Each
// direction's carry starts at its own h0.
cudaError_t m1_seg2_bidir_launch(const M1Params& fwd, const M1Params& bwd, int S,
                                 cudaStream_t stream) {
    const int64_t rows = fwd.batch * fwd.dim, Ls = fwd.len / S;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    const size_t st = static_cast<size_t>(S) * rows * 16, per = 2 * st + static_cast<size_t>(S) * rows;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, 2 * per * sizeof(float), pool, stream);
    if (e != cudaSuccess) return e;
    Seg2Ws wf, wb;
    wf.hend = static_cast<float*>(raw);
    wf.hin = wf.hend + st;
    wf.dtsum = wf.hin + st;
    wb.hend = wf.hend + per;
    wb.hin = wb.hend + st;
    wb.dtsum = wb.hin + st;
    const int64_t gsz = fwd.dim / fwd.groups;
    const unsigned gx = static_cast<unsigned>(((gsz + kS2Rows - 1) / kS2Rows) * fwd.batch * fwd.groups);
    const dim3 grid(gx, static_cast<unsigned>(S)), block(kS2Rows / kS2Rpt);
    m1_seg2_pass1_bidir<0><<<grid, block, 0, stream>>>(fwd, wf, wb, S, Ls);
    note_launch();
    e = cudaGetLastError();
    const int64_t n = rows * fwd.state;
    const dim3 cg(static_cast<unsigned>((n + 255) / 256));
    // the carries end in last_state; pass 2 leaves it alone
    M1Params f2 = fwd, b2 = bwd;
    f2.last_state = nullptr;
    b2.last_state = nullptr;
    if (e == cudaSuccess) e = launch_pdl(m1_seg2_carry_kernel<false>, cg, dim3(256), stream, fwd, wf, S);
    if (e == cudaSuccess) note_launch();
    if (e == cudaSuccess) e = launch_pdl(m1_seg2_carry_kernel<false>, cg, dim3(256), stream, bwd, wb, S);
    if (e == cudaSuccess) note_launch();
    if (fwd.out) {
        if (e == cudaSuccess) e = launch_pdl(m1_seg2_pass2<false, 0>, grid, block, stream, f2, wf, S, Ls, 0);
        if (e == cudaSuccess) note_launch();
        if (e == cudaSuccess) e = launch_pdl(m1_seg2_pass2<true, 0>, grid, block, stream, b2, wb, S, Ls, 0);
        if (e == cudaSuccess) note_launch();
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

}  // namespace b200scan
