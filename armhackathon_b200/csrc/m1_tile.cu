// Mamba-1 selective scan, pipelined row-tile kernel (default path for
// d_state <= 16, the Mamba-1 configuration).
//
// Same algorithm as the chunked kernel in m1_scan.cu (segment sweep from a
// zero state, fold of the per-segment (P, h) aggregates in segment order,
// output fix-up sum_n C*P*h_in), restructured around the measured limits of
// that kernel (few resident warps, global latency exposed every macro-chunk):
//
//  * Tiles never straddle a (batch, B/C group): a tile is DC rows of one
//    group, so the CTA stages ONE copy of B/C per macro-chunk.
//  * Every global read of a macro-chunk is issued with cp.async one
//    macro-chunk ahead into double-buffered shared memory: u and delta into
//    per-thread padded slots (16-byte copies), B and C scattered by 4-byte
//    copies into a transposed [step][state] slab so that a step's 4 states
//    come from one LDS.128 and state pairs are register-adjacent.
//  * Two states per fma.rn.f32x2 / mul.rn.f32x2 in the sweep and fix-up.
//  * <= 128 registers and ~100 KB of shared memory: two CTAs per SM, and a
//    persistent grid-stride loop over (tile, macro-chunk) units keeps the
//    pipeline primed across tile boundaries.
#include <cstdint>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kTileThreads = 256;
constexpr int kBcStride = 20;  // words per staged step (16 states + pad)

__device__ __forceinline__ void cp_async4(void* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 4 : 0));
}
__device__ __forceinline__ void cp_async16(void* smem, const float* gmem, bool pred) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem),
                 "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

template <int DC, int K>
struct TileLayout {
    static constexpr int S = kTileThreads / DC;  // segments per macro-chunk
    static constexpr int T = S * K;              // steps per macro-chunk
    static constexpr int XS = K + 4;             // padded per-thread slot (floats)
    static constexpr int X_F = 2 * 2 * kTileThreads * XS;       // [buf][delta,u][thr][XS]
    static constexpr int BC_ROWS_F = T * kBcStride + S * 4;     // one staged array
    static constexpr int BC_F = 2 * 2 * BC_ROWS_F;              // [buf][B,C]
    static constexpr int AGG_F = 2 * S * (4 * DC + 4);          // aggP, aggH (padded)
    static constexpr int CARRY_F = DC * 16;
    static constexpr int ROWP_F = DC * 16 + 2 * DC;  // A*log2e [DC][16], bias, D
    static constexpr size_t bytes() {
        return sizeof(float) * static_cast<size_t>(X_F + BC_F + AGG_F + CARRY_F + ROWP_F);
    }
    // word offset of traversal step j inside a staged slab: one 4-word pad per
    // segment keeps the two segments a warp reads on different banks
    __device__ static int row(int j) { return j * kBcStride + (j / K) * 4; }
};

// Rows, pointers and row parameters of one tile (DC rows of one group).
struct TileInfo {
    int64_t row0;   // first row (batch*dim index) of the tile
    int64_t bc0;    // element offset of the group's B/C rows
    int n_rows;     // rows of the tile that exist (<= DC)
};

template <int DC, int K, bool VEC, bool REV, int POLY, int MINB = 2>
__global__ void __launch_bounds__(kTileThreads, MINB) m1_tile_kernel(M1Params p, int tiles_per_group,
                                                                     int n_tiles) {
    using LY = TileLayout<DC, K>;
    constexpr int S = LY::S, T = LY::T, XS = LY::XS;
    constexpr int AGG_STRIDE = 4 * DC + 4;  // floats per segment in aggP/aggH
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* xs = sm;                                  // [2][2][256][XS]
    float* bcs = xs + LY::X_F;                       // [2][2][BC_ROWS_F]
    float* aggP = bcs + LY::BC_F;                    // [S][AGG_STRIDE]
    float* aggH = aggP + S * AGG_STRIDE;             // [S][AGG_STRIDE]
    float* carry = aggH + S * AGG_STRIDE;            // [DC][16]
    float* a_s = carry + LY::CARRY_F;                // [DC][16] A*log2e
    float* bias_s = a_s + DC * 16;                   // [DC]
    float* dsk_s = bias_s + DC;                      // [DC]

    const int tid = threadIdx.x, c = tid % DC, s = tid / DC;
    const int L = static_cast<int>(p.len), N = static_cast<int>(p.state);
    // element offsets of a logical row / (batch, group) under the segmented view
    const int64_t SEG = p.seg_count > 1 ? p.seg_count : 1;
    const int64_t LP = p.len_full > 0 ? p.len_full : p.len;
    auto phys_row = [&](int64_t row) {
        const int64_t bb = row / p.dim, d = row - bb * p.dim;
        return ((bb / SEG) * p.dim + d) * LP + (bb % SEG) * L;
    };
    const int n_groups = (N + 3) / 4;
    const int gsz = static_cast<int>(p.dim / p.groups);
    const int n_macro = (L + T - 1) / T;

    auto tile_info = [&](int tile) {
        TileInfo ti;
        const int bg = tile / tiles_per_group, jt = tile - bg * tiles_per_group;
        ti.row0 = static_cast<int64_t>(bg) * gsz + static_cast<int64_t>(jt) * DC;
        {
            const int64_t bb = bg / p.groups, g = bg - bb * p.groups;
            ti.bc0 = ((bb / SEG) * p.groups + g) * N * LP + (bb % SEG) * L;
        }
        const int rem = gsz - jt * DC;
        ti.n_rows = rem < DC ? rem : DC;
        return ti;
    };

    // Issue the copies of (tile ti, chunk mc) into buffer buf, one commit group.
    auto issue = [&](const TileInfo& ti, int mc, int buf, bool valid) {
        if (valid) {
            const bool act = c < ti.n_rows;
            const int64_t row = ti.row0 + (act ? c : 0);
            const int i0 = mc * T + s * K;
            const int64_t base = phys_row(row);
            const float* srcs[2] = {p.delta + base, p.u + base};
#pragma unroll
            for (int a = 0; a < 2; ++a) {
                float* dst = xs + ((buf * 2 + a) * kTileThreads + tid) * XS;
                if (VEC) {
#pragma unroll
                    for (int m = 0; m < K / 4; ++m) {
                        const int t0 = REV ? L - i0 - 4 * m - 4 : i0 + 4 * m;
                        const bool ok = act && t0 >= 0 && t0 < L;
                        cp_async16(dst + 4 * m, srcs[a] + (ok ? t0 : 0), ok);
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < K; ++k) {
                        const int it = i0 + k;
                        const bool ok = act && it < L;
                        cp_async4(dst + k, srcs[a] + (ok ? (REV ? L - 1 - it : it) : 0), ok);
                    }
                }
            }
            // B, C of the tile's group for the whole chunk, transposed
            const float* Bg = p.B + ti.bc0;
            const float* Cg = p.C + ti.bc0;
            float* db = bcs + (buf * 2) * LY::BC_ROWS_F;
            float* dc = db + LY::BC_ROWS_F;
#pragma unroll 4
            for (int idx = tid; idx < n_groups * 4 * T; idx += kTileThreads) {
                const int n = idx / T, j = idx - (idx / T) * T;
                const int it = mc * T + j;
                const bool ok = it < L && n < N;
                const int64_t off = ok ? n * LP + (REV ? L - 1 - it : it) : 0;
                const int w = LY::row(j) + n;
                cp_async4(db + w, Bg + off, ok);
                cp_async4(dc + w, Cg + off, ok);
            }
        }
        cp_async_commit();
    };

    int tile = blockIdx.x;
    if (tile >= n_tiles) return;
    TileInfo cur = tile_info(tile);
    issue(cur, 0, 0, true);
    int buf = 0;
    while (true) {
        for (int mc = 0; mc < n_macro; ++mc, buf ^= 1) {
            // the unit after this one: next chunk, or chunk 0 of the next tile
            const bool last_chunk = mc + 1 == n_macro;
            const int ntile = last_chunk ? tile + static_cast<int>(gridDim.x) : tile;
            const bool has_next = ntile < n_tiles;
            const TileInfo nxt = last_chunk ? (has_next ? tile_info(ntile) : cur) : cur;

            const bool active = c < cur.n_rows;
            const int64_t row = cur.row0 + (active ? c : 0);
            const int i0 = mc * T + s * K;

            cp_async_wait_all();
            __syncthreads();  // chunk visible to all; everyone is done with the previous one
            if (mc == 0) {
                for (int i = tid; i < DC * 16; i += kTileThreads) {
                    const int cc = i / 16, n = i % 16;
                    const bool ok = cc < cur.n_rows && n < N;
                    const int64_t r = cur.row0 + (cc < cur.n_rows ? cc : 0);
                    const int64_t dd = r % p.dim;
                    carry[i] = (p.h0 && ok) ? p.h0[r * N + n] : 0.f;
                    a_s[i] = ok ? p.A[dd * N + n] * kLog2e : 0.f;
                    if (n == 0) {
                        bias_s[cc] = p.delta_bias ? p.delta_bias[dd] : 0.f;
                        dsk_s[cc] = p.d_skip ? p.d_skip[dd] : 0.f;
                    }
                }
                __syncthreads();
            }
            issue(nxt, last_chunk ? 0 : mc + 1, buf ^ 1, has_next || !last_chunk);

            // z for the epilogue, straight from global (consumed at the end)
            float zv[K];
            if (p.z && p.out) {
                const float* zr = p.z + phys_row(row);
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const int it = i0 + k;
                    zv[k] = (active && it < L) ? __ldcs(zr + (REV ? L - 1 - it : it)) : 0.f;
                }
            }
            const float bias = bias_s[c];
            const float dsk = dsk_s[c];
            const float* xd = xs + ((buf * 2 + 0) * kTileThreads + tid) * XS;
            const float* xu = xs + ((buf * 2 + 1) * kTileThreads + tid) * XS;
            float dt[K], dtu[K];
            float2 y2[K];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int sl = (VEC && REV) ? (k & ~3) + 3 - (k & 3) : k;
                const bool ok = active && (i0 + k < L);
                float vv = xd[sl] + bias;
                if (p.delta_softplus) vv = softplus_fast(vv);
                vv = ok ? vv : 0.f;  // masked steps are the identity: a = 1, b = 0
                const float uu = xu[sl];
                y2[k] = make_float2(dsk * uu, 0.f);
                dt[k] = vv;
                dtu[k] = vv * uu;
            }
            const float* sbB = bcs + (buf * 2) * LY::BC_ROWS_F;
            const float* sbC = sbB + LY::BC_ROWS_F;

            for (int g = 0; g < n_groups; ++g) {
                const int n0 = 4 * g;
                const float4 al = *reinterpret_cast<const float4*>(a_s + c * 16 + n0);
                const float2 al01 = make_float2(al.x, al.y), al23 = make_float2(al.z, al.w);
                float2 h01 = make_float2(0.f, 0.f), h23 = h01;
                float2 P01 = make_float2(1.f, 1.f), P23 = P01;
                float2 Q01[K], Q23[K];
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const int w = LY::row(s * K + k) + n0;
                    const float4 bv = *reinterpret_cast<const float4*>(sbB + w);
                    const float4 cv = *reinterpret_cast<const float4*>(sbC + w);
                    const float2 dt2 = make_float2(dt[k], dt[k]);
                    const float2 du2 = make_float2(dtu[k], dtu[k]);
                    const float2 x01 = fmul2(dt2, al01), x23 = fmul2(dt2, al23);
                    // POLY 1: states 2,3 of odd steps on the FMA pipe (25% of
                    // the exps); POLY 2: states 2,3 of every step (50%)
                    const float2 a01 = make_float2(ex2_approx(x01.x), ex2_approx(x01.y));
                    const float2 a23 = (POLY == 2 || (POLY == 1 && (k & 1)))
                                           ? exp2_poly2(x23)
                                           : make_float2(ex2_approx(x23.x), ex2_approx(x23.y));
                    const float2 c01 = make_float2(cv.x, cv.y), c23 = make_float2(cv.z, cv.w);
                    h01 = ffma2(a01, h01, fmul2(du2, make_float2(bv.x, bv.y)));
                    h23 = ffma2(a23, h23, fmul2(du2, make_float2(bv.z, bv.w)));
                    y2[k] = ffma2(c01, h01, y2[k]);
                    y2[k] = ffma2(c23, h23, y2[k]);
                    P01 = fmul2(P01, a01);
                    P23 = fmul2(P23, a23);
                    Q01[k] = fmul2(c01, P01);
                    Q23[k] = fmul2(c23, P23);
                }
                *reinterpret_cast<float4*>(aggP + s * AGG_STRIDE + 4 * c) =
                    make_float4(P01.x, P01.y, P23.x, P23.y);
                *reinterpret_cast<float4*>(aggH + s * AGG_STRIDE + 4 * c) =
                    make_float4(h01.x, h01.y, h23.x, h23.y);
                __syncthreads();
                {
                    // Fold the S segment aggregates of every (row, state) pair in
                    // segment order, seeded by the pair's carry, on all 256
                    // threads: pair = tid / PARTS, part q = tid % PARTS covers
                    // segments 4q..4q+3.
                    constexpr int PARTS = S / 4;
                    const int pair = tid / PARTS, q = tid % PARTS;
                    float pj[4], hj[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        pj[j] = aggP[(4 * q + j) * AGG_STRIDE + pair];
                        hj[j] = aggH[(4 * q + j) * AGG_STRIDE + pair];
                    }
                    float Pq = pj[0], Hq = hj[0];
#pragma unroll
                    for (int j = 1; j < 4; ++j) {
                        Hq = fmaf(pj[j], Hq, hj[j]);
                        Pq *= pj[j];
                    }
#pragma unroll
                    for (int dd = 1; dd < PARTS; dd <<= 1) {
                        const float pp = __shfl_up_sync(0xffffffffu, Pq, dd, PARTS);
                        const float hp = __shfl_up_sync(0xffffffffu, Hq, dd, PARTS);
                        if (q >= dd) {
                            Hq = fmaf(Pq, hp, Hq);
                            Pq *= pp;
                        }
                    }
                    float Pe = __shfl_up_sync(0xffffffffu, Pq, 1, PARTS);
                    float He = __shfl_up_sync(0xffffffffu, Hq, 1, PARTS);
                    if (q == 0) {
                        Pe = 1.f;
                        He = 0.f;
                    }
                    float* cr = carry + (pair >> 2) * 16 + n0 + (pair & 3);
                    float h = fmaf(Pe, *cr, He);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        aggH[(4 * q + j) * AGG_STRIDE + pair] = h;
                        h = fmaf(pj[j], h, hj[j]);
                    }
                    if (q == PARTS - 1) *cr = h;
                }
                __syncthreads();
                const float4 hin = *reinterpret_cast<const float4*>(aggH + s * AGG_STRIDE + 4 * c);
                const float2 hin01 = make_float2(hin.x, hin.y), hin23 = make_float2(hin.z, hin.w);
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    y2[k] = ffma2(Q01[k], hin01, y2[k]);
                    y2[k] = ffma2(Q23[k], hin23, y2[k]);
                }
            }

            if (active && p.out) {
                float* orow = p.out + phys_row(row);
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const int it = i0 + k;
                    float y = y2[k].x + y2[k].y;
                    if (p.z) y *= silu_fast(zv[k]);
                    if (it < L) __stcs(orow + (REV ? L - 1 - it : it), y);
                }
            }
            if (last_chunk && p.last_state) {
                // carry is final: the last fold wrote it before the barrier above
                for (int i = tid; i < DC * 16; i += kTileThreads) {
                    const int cc = i / 16, n = i % 16;
                    if (cc < cur.n_rows && n < N) p.last_state[(cur.row0 + cc) * N + n] = carry[i];
                }
            }
        }
        tile += gridDim.x;
        if (tile >= n_tiles) break;
        cur = tile_info(tile);
    }
    cp_async_wait_all();
}

template <int DC, int K, int POLY = 0, int MINB = 2>
cudaError_t launch_tile(const M1Params& p, cudaStream_t stream) {
    using LY = TileLayout<DC, K>;
    const int64_t gsz = p.dim / p.groups;
    const int64_t tiles_per_group = (gsz + DC - 1) / DC;
    const int64_t n_tiles = p.batch * p.groups * tiles_per_group;
    const int64_t pitch = p.len_full > 0 ? p.len_full : p.len;
    if (n_tiles > INT32_MAX || p.len > (INT32_MAX / 4) || p.state * pitch > INT32_MAX)
        return cudaErrorInvalidValue;
    const size_t smem = LY::bytes();
    const bool vec = (p.len % 4 == 0) && (pitch % 4 == 0) && m1_pointers_aligned16(p);
    void (*kern)(M1Params, int, int);
    if (vec)
        kern = p.reverse ? m1_tile_kernel<DC, K, true, true, POLY, MINB>
                         : m1_tile_kernel<DC, K, true, false, POLY, MINB>;
    else
        kern = p.reverse ? m1_tile_kernel<DC, K, false, true, POLY, MINB>
                         : m1_tile_kernel<DC, K, false, false, POLY, MINB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTileThreads, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t cap = static_cast<int64_t>(sms) * per_sm;
    const int64_t grid = n_tiles < cap ? n_tiles : cap;
    kern<<<dim3(static_cast<unsigned>(grid)), kTileThreads, smem, stream>>>(
        p, static_cast<int>(tiles_per_group), static_cast<int>(n_tiles));
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t m1_tile_launch(const M1Params& p, int variant, cudaStream_t stream) {
    switch (variant) {
        case 1: return launch_tile<16, 8>(p, stream);
        case 2: return launch_tile<8, 8>(p, stream);
        case 3: return launch_tile<32, 8>(p, stream);
        case 4: return launch_tile<16, 4>(p, stream);
        case 9: return launch_tile<16, 8, 1>(p, stream);
        case 10: return launch_tile<16, 8, 2>(p, stream);
        case 11: return launch_tile<16, 4, 0, 3>(p, stream);  // three CTAs per SM
        default: return launch_tile<16, 8>(p, stream);
    }
}

}  // namespace b200scan
