// Mamba-1 selective scan, lanes over states, TMA-staged (default kernel for
// d_state <= 16).
//
// Recurrence (reference kernel/arm-scan-core/src/scalar.rs:11-89):
//   dt = softplus(delta + bias), h_n = exp(dt A_n) h_n + dt u B_n,
//   y = sum_n C_n h_n + D u, times silu(z); reverse walks the steps from the
// end (scalar.rs:59).
//
// Thread mapping.  Four lanes of a warp own one (batch, channel) row, lane q
// holding states q, q+4, q+8, q+12 in registers, so a warp covers 8 rows and
// every lane computes exactly one exp per (step, owned state).  The per-step
// row work (softplus of delta, dt*u, silu(z), D*u) is spread over the four
// lanes instead of repeated by each: lane q takes steps 4k+q of every
// 32-step tile, writes dt and dt*u back into the staged tile, and keeps
// silu(z) and D*u*silu(z) in registers.  After the recurrence over 4 steps
// every lane holds 4 partial outputs (its states' share of y at each step);
// a two-stage butterfly (xor 2, xor 1) reduce-scatters them so that lane q
// ends with the full y of step 4k+q, the step whose silu(z) it computed.
//
// Staging.  A CTA is 32 rows of one (batch, B/C group) and one time segment:
// four compute warps and one producer warp.  The producer streams 32-step
// tiles of delta, u, z ([32 rows][32 steps]) and B, C ([N states][32 steps])
// through a 4-deep shared-memory ring with 2D TMA loads
// (cp.async.bulk.tensor, 128-byte swizzle so that the rows of a warp's
// 16-byte loads fall in distinct banks), full/empty mbarriers between the
// producer and the compute warps.  Outputs are written back from the staged
// z slot as coalesced 16-byte stores.  Every mbarrier wait is bounded; on
// expiry the kernel sets a device status flag and stops.
//
// Time segments.  When rows are too few to fill the GPU, the sequence is cut
// into S segments, as in a two-pass segmented scan: pass 1 computes each
// segment's end state from zero (and the first segment's outputs from h0),
// a carry kernel chains h_in(s) = exp(A sum dt(prev)) h_in(prev) +
// h_end(prev), and pass 2 rescans segments 1..S-1 from h_in.  The segment
// count is chosen from a wave model of the launch (see lane_pick_segments).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "m1_scan.h"

namespace b200scan {

namespace {

constexpr int kLT = 32;        // steps per tile
constexpr int kLRows = 32;     // rows per CTA
// Ring depth: 4 stages (3 CTAs per SM, 128 registers) for the unsplit sweep,
// whose row count caps the CTAs anyway; 3 stages (4 CTAs per SM) for the
// split and bidirectional passes, which have CTAs to spare and gain from the
// extra warps.
constexpr int kLStagesWide = 4, kLStagesDense = 3;
constexpr int kLWarps = 4;     // compute warps
constexpr int kLThreads = (kLWarps + 1) * 32;
constexpr uint32_t kXBytes = kLRows * kLT * 4;  // one [32 rows][32 steps] fp32 tile
constexpr uint32_t kBCBytes = 16 * kLT * 4;     // one [16 states][32 steps] tile
constexpr uint32_t kStageBytes = 3 * kXBytes + 2 * kBCBytes;
constexpr uint32_t smem_bytes(int stages) { return stages * kStageBytes + 1024 /* alignment */ + 256 /* barriers */; }
constexpr int min_blocks(int stages) { return stages == kLStagesWide ? 3 : 4; }
constexpr uint32_t kWaitLimit = 1u << 24;
// Owned states (bit i: state q + 4i) whose decays run on the FMA pipe
// (exp2_poly2) instead of the MUFU unit, to balance the two pipes.
#ifndef B200SCAN_LANE_POLY_MASK
#define B200SCAN_LANE_POLY_MASK 0
#endif
constexpr int kLanePolyMask = B200SCAN_LANE_POLY_MASK;

__device__ int g_m1_status;  // 0 ok, 1 a staging wait expired

enum LaneMode {
    kLaneState = 0,   // from zero: end state + sum of dt
    kLaneRescan = 1,  // from h_in: y (and last_state on the last segment)
    kLaneFirst = 2,   // from h0: y, and the true end state into hend
    kLaneBidir = 3,   // from zero, forward: the end state and the reverse
                      // traversal's aggregate of the segment (see pass1_bidir)
};

struct LaneWs {
    float* hend;   // [S][rows][16]
    float* hin;    // [S][rows][16]
    float* dtsum;  // [S][rows]
};

struct LaneMaps {
    CUtensorMap delta, u, z, B, C;
};

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mb_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// bounded wait for the phase of the given parity; false on expiry
__device__ __forceinline__ bool mb_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t b = smem_u32(bar);
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(b), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiles are [rows][32] fp32 written by TMA with 128-byte swizzle: 16-byte
// chunk c of row r sits at chunk c ^ (r % 8).  With a row's base address
// (128-byte aligned) and its key (r % 8) << 4, chunk c is at
// base | ((c << 4) ^ key): one logic op per access for a constant c.
__device__ __forceinline__ uint32_t chunk_addr(uint32_t base, uint32_t key, int c) {
    return base | ((static_cast<uint32_t>(c) << 4) ^ key);
}
// Shared-memory loads are plain (non-volatile) asm so that the compiler may
// schedule them early; every address is derived from a base passed through
// order_after(), a volatile no-op with a memory clobber placed after the
// barrier that makes the data visible, so no load can move above it.
__device__ __forceinline__ uint32_t order_after(uint32_t base) {
    asm volatile("mov.b32 %0, %0;" : "+r"(base)::"memory");
    return base;
}
__device__ __forceinline__ float4 lds4(uint32_t a) {
    float4 v;
    asm("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds1(uint32_t a) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts1(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// ---- the sweep --------------------------------------------------------------
// One CTA: rows [row0, row0 + 32) of one (batch, group), segment s.
template <int MODE, bool REV, int kLStages>
__device__ __forceinline__ void lane_sweep(const M1Params& p, const LaneMaps& maps, const LaneWs& ws,
                                           const LaneWs* wsb, int S, int64_t Ls, int s, char* smem,
                                           uint64_t* full, uint64_t* empty) {
    constexpr bool FULL = MODE == kLaneRescan || MODE == kLaneFirst;
    constexpr bool BID = MODE == kLaneBidir;
    const int N = static_cast<int>(p.state);
    const int64_t L = p.len, D = p.dim, G = p.groups, gsz = D / G;
    const int64_t rows_all = p.batch * D;
    const int blocks_per_group = static_cast<int>((gsz + kLRows - 1) / kLRows);
    const int64_t bg = blockIdx.x / blocks_per_group;
    const int jb = blockIdx.x % blocks_per_group;
    const int64_t b = bg / G, g = bg % G;
    const int64_t row0 = b * D + g * gsz + static_cast<int64_t>(jb) * kLRows;
    const int64_t it0 = static_cast<int64_t>(s) * Ls;
    const int64_t ie = it0 + Ls < L ? it0 + Ls : L;
    const int n_tiles = static_cast<int>((ie - it0 + kLT - 1) / kLT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool has_z = FULL && p.z;

    if (warp == kLWarps) {  // ---- producer warp
        if (lane == 0) {
            tma_prefetch_desc(&maps.delta);
            tma_prefetch_desc(&maps.u);
            tma_prefetch_desc(&maps.B);
            if (has_z) tma_prefetch_desc(&maps.z);
            if (FULL) tma_prefetch_desc(&maps.C);
            const uint32_t bc = static_cast<uint32_t>(N) * kLT * 4;
            const uint32_t bytes = 2 * kXBytes + bc + (has_z ? kXBytes : 0) + (FULL ? bc : 0);
            for (int c = 0; c < n_tiles; ++c) {
                const int slot = c % kLStages;
                if (c >= kLStages && !mb_wait(&empty[slot], ((c / kLStages) - 1) & 1)) {
                    atomicExch(&g_m1_status, 1);
                    break;
                }
                char* st = smem + slot * kStageBytes;
                const int64_t j0 = it0 + static_cast<int64_t>(c) * kLT;
                const int x = static_cast<int>(REV ? L - j0 - kLT : j0);
                const int yr = static_cast<int>(row0);
                const int yb = static_cast<int>(bg * N);
                mb_expect_tx(&full[slot], bytes);
                tma_load_2d(st, &maps.delta, x, yr, &full[slot]);
                tma_load_2d(st + kXBytes, &maps.u, x, yr, &full[slot]);
                if (has_z) tma_load_2d(st + 2 * kXBytes, &maps.z, x, yr, &full[slot]);
                tma_load_2d(st + 3 * kXBytes, &maps.B, x, yb, &full[slot]);
                if (FULL) tma_load_2d(st + 3 * kXBytes + kBCBytes, &maps.C, x, yb, &full[slot]);
            }
        }
        return;
    }

    // ---- compute warps: lane (r, q) owns row r (0..31) and states q + 4i
    const int r = warp * 8 + (lane >> 2), q = lane & 3;
    const int64_t row = row0 + r;
    const bool active = static_cast<int64_t>(jb) * kLRows + r < gsz && row < rows_all;
    const int64_t ch = active ? row % D : 0;
    float2 a2[4];  // (A_n, A_n) * log2(e) for the owned states n = q + 4i
    {
        const float* A = p.A + ch * N;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v = q + 4 * i < N ? A[q + 4 * i] * kLog2e : 0.f;
            a2[i] = make_float2(v, v);
        }
    }
    const float bias = p.delta_bias ? p.delta_bias[ch] : 0.f;
    const float dsk = (FULL && p.d_skip) ? p.d_skip[ch] : 0.f;

    if (MODE == kLaneRescan) griddep_wait();  // h_in comes from the carry kernel
    float h[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) {
        const float* hi = MODE == kLaneRescan ? ws.hin + (static_cast<int64_t>(s) * rows_all + row) * 16
                          : (MODE == kLaneFirst && p.h0) ? p.h0 + row * N
                                                        : nullptr;
        if (hi) {
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = q + 4 * i < N ? hi[q + 4 * i] : 0.f;
        }
    }
    float pr[4] = {1.f, 1.f, 1.f, 1.f};  // BID: running decay product
    float hb[4] = {0.f, 0.f, 0.f, 0.f};  // BID: reverse aggregate
    float dtsum = 0.f;

    for (int c = 0; c < n_tiles; ++c) {
        const int slot = c % kLStages;
        const bool ok = mb_wait(&full[slot], (c / kLStages) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicExch(&g_m1_status, 1);
            return;
        }
        // this lane's row in the delta (-> dt), u, z (-> silu(z) -> y) tiles,
        // and its states' rows in the B, C tiles
        const uint32_t st = order_after(smem_u32(smem) + slot * kStageBytes);
        uint32_t rd = st + r * 128, ru = rd + kXBytes, rz = rd + 2 * kXBytes;
        const uint32_t rkey = (r & 7) << 4;
        uint32_t bB = st + 3 * kXBytes + q * 128, bC = bB + kBCBytes;
        const uint32_t bkey = q << 4;  // states q + 4i: key q (i even), q + 4 (i odd)
        const int64_t j0 = it0 + static_cast<int64_t>(c) * kLT;
        const int cnt = static_cast<int>(ie - j0 < kLT ? ie - j0 : kLT);

        // phase A: lane q takes the steps at memory positions 4c + q of the
        // tile (c = 0..7): dt over delta, silu(z) over z; u stays
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int m = 4 * c + q;
            const int j = REV ? kLT - 1 - m : m;  // traversal index within the tile
            const uint32_t off = chunk_addr(q * 4, rkey, c);  // (c ^ key) * 16 + q * 4
            float dt = 0.f;
            if (j < cnt) {
                dt = lds1(rd + off) + bias;
                if (p.delta_softplus) dt = softplus_fast(dt);
            }
            dtsum += dt;
            sts1(rd + off, dt);
            if (has_z) sts1(rz + off, silu_fast(lds1(rz + off)));
        }
        __syncwarp();
        rd = order_after(rd);
        ru = order_after(ru);
        rz = order_after(rz);

        // phase B: the recurrence, one 16-byte chunk (4 steps) at a time;
        // pairs are formed along time in memory order, (e0, e1), (e2, e3),
        // so that the packed products read their operands straight from the
        // 16-byte loads; the state chain walks e0..e3 (e3..e0 in reverse)
        // The decays of chunk k + 1 are computed while chunk k's chains run:
        // the exps do not depend on the state, so issuing them one chunk
        // ahead keeps MUFU work ready whenever a chain waits.
        struct Chunk {
            float e[4][4];   // decays [state][memory element]
            float2 dul, duh; // dt * u, (e0, e1) and (e2, e3)
        };
        auto decays = [&](int c, Chunk& ck) {
            const float4 dt4 = lds4(chunk_addr(rd, rkey, c)), u4 = lds4(chunk_addr(ru, rkey, c));
            const float2 dtl = make_float2(dt4.x, dt4.y), dth = make_float2(dt4.z, dt4.w);
            ck.dul = fmul2(dtl, make_float2(u4.x, u4.y));
            ck.duh = fmul2(dth, make_float2(u4.z, u4.w));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 xl = fmul2(dtl, a2[i]), xh = fmul2(dth, a2[i]);
                if ((kLanePolyMask >> i) & 1) {
                    const float2 el = exp2_poly2(xl), eh = exp2_poly2(xh);
                    ck.e[i][0] = el.x, ck.e[i][1] = el.y, ck.e[i][2] = eh.x, ck.e[i][3] = eh.y;
                } else {
                    ck.e[i][0] = ex2_approx(xl.x), ck.e[i][1] = ex2_approx(xl.y);
                    ck.e[i][2] = ex2_approx(xh.x), ck.e[i][3] = ex2_approx(xh.y);
                }
            }
        };
        Chunk cur, nxt;
        decays(REV ? 7 : 0, cur);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = REV ? 7 - k : k;
            if (k + 1 < 8) decays(REV ? 6 - k : k + 1, nxt);
            float2 yl = make_float2(0.f, 0.f), yh = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t nkey = bkey ^ ((i & 1) << 6), noff = i * 512;
                const float4 b4 = lds4(chunk_addr(bB + noff, nkey, c));
                const float2 bl = fmul2(cur.dul, make_float2(b4.x, b4.y));
                const float2 bh = fmul2(cur.duh, make_float2(b4.z, b4.w));
                const float bu[4] = {bl.x, bl.y, bh.x, bh.y};
                float hs[4];
                float hc = h[i];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int ei = REV ? 3 - t : t;
                    hc = fmaf(cur.e[i][ei], hc, bu[ei]);
                    hs[ei] = hc;
                    if (BID) {
                        hb[i] = fmaf(pr[i], bu[ei], hb[i]);
                        pr[i] *= cur.e[i][ei];
                    }
                }
                h[i] = hc;
                if (FULL) {
                    const float4 c4 = lds4(chunk_addr(bC + noff, nkey, c));
                    yl = ffma2(make_float2(c4.x, c4.y), make_float2(hs[0], hs[1]), yl);
                    yh = ffma2(make_float2(c4.z, c4.w), make_float2(hs[2], hs[3]), yh);
                }
            }
            if (k + 1 < 8) cur = nxt;
            if (FULL) {
                // reduce-scatter over the row's 4 lanes: lane q gets memory
                // element q of the chunk
                const bool hi = q & 2, lo = q & 1;
                const float s0 = hi ? yl.x : yh.x, s1 = hi ? yl.y : yh.y;
                const float k0 = hi ? yh.x : yl.x, k1 = hi ? yh.y : yl.y;
                const float v0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 2);
                const float v1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 2);
                const float sl = lo ? v0 : v1, kp = lo ? v1 : v0;
                const float y = kp + __shfl_xor_sync(0xffffffffu, sl, 1);
                const uint32_t off = chunk_addr(q * 4, rkey, c);
                float yo = fmaf(dsk, lds1(ru + off), y);
                if (has_z) yo *= lds1(rz + off);
                sts1(rz + off, yo);
            }
        }

        if (FULL) {
            // phase C: the warp's 8 rows x 32 steps of y, as 16-byte stores
            __syncwarp();
            const uint32_t sy = order_after(st + 2 * kXBytes);
            const int64_t ms = REV ? L - j0 - kLT : j0;  // memory step of tile position 0
#pragma unroll
            for (int rep = 0; rep < 2; ++rep) {
                const int idx = rep * 32 + lane;
                const int rr = warp * 8 + (idx >> 3), cc = idx & 7;
                const int64_t orow = row0 + rr;
                const bool valid = REV ? (4 * cc >= kLT - cnt) : (4 * cc < cnt);
                const bool ract = static_cast<int64_t>(jb) * kLRows + rr < gsz && orow < rows_all;
                if (valid && ract) {
                    float4 y4 = lds4(chunk_addr(sy + rr * 128, (rr & 7) << 4, cc));
                    float4* o4 = reinterpret_cast<float4*>(p.out + orow * L + ms + 4 * cc);
                    if (p.out_acc) {
                        const float4 o = __ldcs(o4);
                        y4 = make_float4(o.x + y4.x, o.y + y4.y, o.z + y4.z, o.w + y4.w);
                    }
                    __stcs(o4, y4);
                }
            }
        }
        // release the slot: the generic-proxy writes above come before the
        // next TMA writes into it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mb_arrive(&empty[slot]);
    }

    // segment summaries
    dtsum += __shfl_xor_sync(0xffffffffu, dtsum, 1);
    dtsum += __shfl_xor_sync(0xffffffffu, dtsum, 2);
    if (!active) return;
    const float* hv = h;
    // segment end states for the carry (an unsplit scan with outputs has no
    // workspace and no carry)
    if (MODE != kLaneRescan && ws.hend) {
        float* he = ws.hend + (static_cast<int64_t>(s) * rows_all + row) * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) he[q + 4 * i] = hv[i];
        if (q == 0) ws.dtsum[static_cast<int64_t>(s) * rows_all + row] = dtsum;
    }
    if (BID) {
        // the reverse traversal visits this segment as its (S - 1 - s)-th
        const int64_t sr = static_cast<int64_t>(S - 1 - s) * rows_all + row;
        const float* bv = hb;
        float* he = wsb->hend + sr * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) he[q + 4 * i] = bv[i];
        if (q == 0) wsb->dtsum[sr] = dtsum;
    }
    if (FULL && s == S - 1 && p.last_state) {
        float* ls = p.last_state + row * N;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (q + 4 * i < N) ls[q + 4 * i] = hv[i];
    }
}

// Shared set-up of every pass: aligned ring, barriers, zeroed B/C rows >= N.
template <int kLStages>
__device__ __forceinline__ char* lane_setup(uint64_t*& full, uint64_t*& empty, int N) {
    extern __shared__ unsigned char lane_smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(lane_smem_raw) + 1023) & ~uintptr_t(1023));
    full = reinterpret_cast<uint64_t*>(smem + kLStages * kStageBytes);
    empty = full + kLStages;
    if (N < 16) {  // TMA writes rows 0..N-1 of the B/C tiles; the rest stay zero
        for (int i = threadIdx.x; i < kLStages * 2 * (16 - N) * kLT; i += blockDim.x) {
            const int per = (16 - N) * kLT;
            const int st = i / (2 * per), rem = i % (2 * per), w = rem / per, e = rem % per;
            reinterpret_cast<float*>(smem + st * kStageBytes + 3 * kXBytes + w * kBCBytes)[N * kLT + e] = 0.f;
        }
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kLStages; ++i) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], kLWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    return smem;
}

// Pass 1.  FIRST 2: segment 0 runs the full scan from h0, segments 1..S-2
// the state-only sweep; FIRST 1: the full scan of an unsplit sequence (its
// own kernel, so that its registers are not those of both sweeps); FIRST 0:
// every segment state-only.
template <int FIRST, bool REV, int ST>
__global__ void __launch_bounds__(kLThreads, min_blocks(ST))
    m1_lane_pass1(M1Params p, const __grid_constant__ LaneMaps maps, LaneWs ws, int S, int64_t Ls) {
    uint64_t *full, *empty;
    char* smem = lane_setup<ST>(full, empty, static_cast<int>(p.state));
    griddep_launch_dependents();
    if (FIRST == 1 || (FIRST == 2 && blockIdx.y == 0))
        lane_sweep<kLaneFirst, REV, ST>(p, maps, ws, nullptr, S, Ls, 0, smem, full, empty);
    else
        lane_sweep<kLaneState, REV, ST>(p, maps, ws, nullptr, S, Ls, blockIdx.y, smem, full, empty);
}

// Pass 1 of both traversals of the same inputs: one forward walk per segment
// with every exp computed once gives the forward end state from zero and the
// reverse traversal's aggregate of the segment from zero,
// sum_t (prod_{r<t} exp(dt_r A)) dt_t u_t B_t (the running product needs
// multiplies only), written at the reverse traversal's segment index.
template <int ST>
__global__ void __launch_bounds__(kLThreads, min_blocks(ST))
    m1_lane_pass1_bidir(M1Params p, const __grid_constant__ LaneMaps maps, LaneWs ws, LaneWs wsb, int S,
                        int64_t Ls) {
    uint64_t *full, *empty;
    char* smem = lane_setup<ST>(full, empty, static_cast<int>(p.state));
    griddep_launch_dependents();
    lane_sweep<kLaneBidir, false, ST>(p, maps, ws, &wsb, S, Ls, blockIdx.y, smem, full, empty);
}

// Pass 2: segments s_off .. from their incoming states.
template <bool REV, int ST>
__global__ void __launch_bounds__(kLThreads, min_blocks(ST))
    m1_lane_pass2(M1Params p, const __grid_constant__ LaneMaps maps, LaneWs ws, int S, int64_t Ls, int s_off) {
    uint64_t *full, *empty;
    char* smem = lane_setup<ST>(full, empty, static_cast<int>(p.state));
    lane_sweep<kLaneRescan, REV, ST>(p, maps, ws, nullptr, S, Ls, blockIdx.y + s_off, smem, full, empty);
}

// Carry across segments in traversal order.  FIRST: segment 0's hend is its
// true end state, the carry fills h_in of segments 1..S-1; otherwise every
// hend is from zero, the carry starts at h0 and ends in last_state.
template <bool FIRST>
__global__ void m1_lane_carry(M1Params p, LaneWs ws, int S) {
    const int64_t rows_all = p.batch * p.dim, N = p.state;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    griddep_launch_dependents();
    griddep_wait();
    if (i >= rows_all * N) return;
    const int64_t row = i / N, n = i % N;
    const float a = p.A[(row % p.dim) * N + n] * kLog2e;
    float h = FIRST ? __ldg(ws.hend + row * 16 + n) : (p.h0 ? p.h0[i] : 0.f);
    float dts = 0.f;  // the whole sequence's sum of dt (segment summaries)
    const int k_end = FIRST ? S - 1 : S;
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
            dts += ds[u];
        }
    }
    if (FIRST && S > 1) ws.hin[(static_cast<int64_t>(S - 1) * rows_all + row) * 16 + n] = h;
    if (!FIRST && p.last_state) p.last_state[i] = h;
    if (!FIRST && p.dt_sum && n == 0) p.dt_sum[row] = dts;
}

// ---- host side --------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 2D map over a row-major (rows, len) fp32 matrix, box (box_rows, 32 steps).
cudaError_t make_map(CUtensorMap* m, const float* base, int64_t len, int64_t rows, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(len), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(len) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kLT), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_maps(const M1Params& p, LaneMaps* m) {
    std::memset(m, 0, sizeof(*m));
    const int64_t rows = p.batch * p.dim, bcrows = p.batch * p.groups * p.state;
    cudaError_t e = make_map(&m->delta, p.delta, p.len, rows, kLRows);
    if (e == cudaSuccess) e = make_map(&m->u, p.u, p.len, rows, kLRows);
    if (e == cudaSuccess && p.z) e = make_map(&m->z, p.z, p.len, rows, kLRows);
    if (e == cudaSuccess) e = make_map(&m->B, p.B, p.len, bcrows, static_cast<int>(p.state));
    if (e == cudaSuccess && p.C) e = make_map(&m->C, p.C, p.len, bcrows, static_cast<int>(p.state));
    return e;
}

// Tensor maps of the last few distinct calls (per host thread): encoding
// five maps costs microseconds of host time, which a small op (one batch
// row) would otherwise spend on every call.
struct MapKey {
    const void *u, *delta, *z, *B, *C;
    int64_t batch, dim, len, state, groups;
    bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
cudaError_t make_maps(const M1Params& p, LaneMaps* m) {
    struct Entry {
        MapKey key;
        int dev;
        LaneMaps maps;
    };
    thread_local Entry cache[8];
    thread_local int next = 0, used = 0;
    MapKey k;
    std::memset(&k, 0, sizeof(k));
    k.u = p.u;
    k.delta = p.delta;
    k.z = p.z;
    k.B = p.B;
    k.C = p.C;
    k.batch = p.batch;
    k.dim = p.dim;
    k.len = p.len;
    k.state = p.state;
    k.groups = p.groups;
    int dev = 0;
    cudaGetDevice(&dev);
    for (int i = 0; i < used; ++i)
        if (cache[i].dev == dev && cache[i].key == k) {
            *m = cache[i].maps;
            return cudaSuccess;
        }
    const cudaError_t e = encode_maps(p, m);
    if (e != cudaSuccess) return e;
    cache[next].key = k;
    cache[next].dev = dev;
    cache[next].maps = *m;
    next = (next + 1) % 8;
    if (used < 8) ++used;
    return cudaSuccess;
}

// Raises the kernel's dynamic shared-memory limit, once per (kernel, device).
template <class K>
cudaError_t allow_smem(K kern, uint32_t bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    const void* key = reinterpret_cast<const void*>(kern);
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == key && d.second == dev) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) done.emplace_back(key, dev);
    return e;
}

// Concurrent CTAs of the lane kernels per device (SMs x resident CTAs per SM).
// Concurrent CTAs per device (SMs x resident CTAs per SM) of the wide
// (unsplit sweep) or the dense (split / bidirectional) configuration.
int lane_slots(bool dense) {
    static int cache[64][2] = {{0}};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[dev][dense]) return cache[dev][dense];
    int sms = 148, per = dense ? 4 : 3;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dense) {
        auto k = m1_lane_pass2<false, kLStagesDense>;
        if (allow_smem(k, smem_bytes(kLStagesDense)) == cudaSuccess)
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, kLThreads, smem_bytes(kLStagesDense));
    } else {
        auto k = m1_lane_pass1<1, false, kLStagesWide>;
        if (allow_smem(k, smem_bytes(kLStagesWide)) == cudaSuccess)
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, kLThreads, smem_bytes(kLStagesWide));
    }
    if (per < 1) per = 1;
    const int v = sms * per;
    if (dev >= 0 && dev < 64) cache[dev][dense] = v;
    return v;
}

// Segment count: the cheapest S under a wave model.  Each pass costs
// (steps per segment) x (waves of CTAs it needs); a split scan makes two
// passes (pass 1 over S-1 segments, pass 2 over S-1), an unsplit one a
// single pass.  passes_all: the bidirectional (3 passes over all S
// segments) and final-state-only (1 pass over all S) forms.
int lane_pick_segments(const M1Params& p, int passes_all) {
    const int64_t gsz = p.dim / p.groups;
    const int64_t rb = ((gsz + kLRows - 1) / kLRows) * p.batch * p.groups;
    int best = 1;
    double best_cost = -1;
    for (int S = 1; S <= 1024; S *= 2) {
        if (p.len % S != 0 || (p.len / S) % 4 != 0) break;
        if (S > 1 && p.len / S < 128) break;
        const int64_t Ls = p.len / S;
        const int64_t ctas = passes_all ? rb * S : rb * (S > 1 ? S - 1 : 1);
        if (ctas > 65535 * 64) break;
        const int64_t slots = lane_slots(ctas > lane_slots(false));
        const int64_t waves = (ctas + slots - 1) / slots;
        const int passes = passes_all ? passes_all : (S > 1 ? 2 : 1);
        // a small fixed cost per pass (pipeline fill, launch) breaks ties;
        // the carries walk the segments serially (about two steps' time
        // each, measured), so many short segments cost their own
        const double cost = static_cast<double>(passes) * (Ls * waves + 64) + (S > 1 ? 2.0 * S : 0.0);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = S;
        }
    }
    return best;
}

bool lane_applicable(const M1Params& p) {
    if (p.state > 16 || p.state < 1 || p.len % 4 != 0 || p.len < 4) return false;
    if (!m1_pointers_aligned16(p)) return false;
    if (p.len > (int64_t(1) << 30) || p.batch * p.dim > (int64_t(1) << 30)) return false;
    if (p.batch * p.groups * p.state > (int64_t(1) << 30)) return false;
    if (p.dim % p.groups != 0) return false;
    return encode_fn() != nullptr;
}

struct LaneWsAlloc {
    void* raw = nullptr;
    cudaStream_t stream;
    explicit LaneWsAlloc(cudaStream_t s) : stream(s) {}
    cudaError_t get(size_t bytes) {
        cudaMemPool_t pool = nullptr;
        cudaError_t e = device_workspace_pool(&pool);
        if (e != cudaSuccess) return e;
        return cudaMallocFromPoolAsync(&raw, bytes, pool, stream);
    }
    cudaError_t release() { return raw ? cudaFreeAsync(raw, stream) : cudaSuccess; }
};

void carve(float* base, size_t S, size_t rows, LaneWs* ws) {
    const size_t st = S * rows * 16;
    ws->hend = base;
    ws->hin = base + st;
    ws->dtsum = base + 2 * st;
}

}  // namespace

// The kKnobM1Segments override, where it divides the sequence into
// segments of a multiple of 4 steps.
static int forced_segments(const M1Params& p) {
    const int s = kernel_override(kKnobM1Segments);
    return (s >= 1 && p.len % s == 0 && (p.len / s) % 4 == 0) ? s : 0;
}

int m1_lane_segments(const M1Params& p) {
    if (!lane_applicable(p)) return 0;
    if (const int s = forced_segments(p)) return s;
    if (p.segments > 0 && p.len % p.segments == 0 && (p.len / p.segments) % 4 == 0) return p.segments;
    return lane_pick_segments(p, p.out ? 0 : 1);
}

cudaError_t m1_lane_launch(const M1Params& p, int S, cudaStream_t stream) {
    const int64_t rows = p.batch * p.dim, Ls = p.len / S;
    LaneMaps maps;
    cudaError_t e = make_maps(p, &maps);
    if (e != cudaSuccess) return e;
    const bool first = p.out != nullptr;  // out == nullptr: final state only
    const int f = first ? (S == 1 ? 1 : 2) : 0;
    constexpr int W = kLStagesWide, Dn = kLStagesDense;
    const int64_t gsz = p.dim / p.groups;
    const unsigned gx = static_cast<unsigned>(((gsz + kLRows - 1) / kLRows) * p.batch * p.groups);
    // pass 1 covers segments 0 .. S-2 when the first runs in full (all of
    // them for S == 1), every segment otherwise
    const unsigned s1 = first ? static_cast<unsigned>(S > 1 ? S - 1 : 1) : static_cast<unsigned>(S);
    // the dense configuration where a pass has more CTAs than the wide one holds
    const bool dense = static_cast<int64_t>(gx) * s1 > lane_slots(false);
#define LANE_P1(F) (dense ? (p.reverse ? m1_lane_pass1<F, true, Dn> : m1_lane_pass1<F, false, Dn>) \
                          : (p.reverse ? m1_lane_pass1<F, true, W> : m1_lane_pass1<F, false, W>))
    auto k1 = f == 1 ? LANE_P1(1) : f == 2 ? LANE_P1(2) : LANE_P1(0);
#undef LANE_P1
    auto k2 = dense ? (p.reverse ? m1_lane_pass2<true, Dn> : m1_lane_pass2<false, Dn>)
                    : (p.reverse ? m1_lane_pass2<true, W> : m1_lane_pass2<false, W>);
    const uint32_t smem1 = smem_bytes(dense ? Dn : W), smem2 = smem1;
    if ((e = allow_smem(k1, smem1)) != cudaSuccess || (e = allow_smem(k2, smem2)) != cudaSuccess) return e;
    LaneWsAlloc alloc(stream);
    LaneWs ws = {nullptr, nullptr, nullptr};
    if (S > 1 || !first) {
        e = alloc.get((2 * static_cast<size_t>(S) * rows * 16 + static_cast<size_t>(S) * rows) * sizeof(float));
        if (e != cudaSuccess) return e;
        carve(static_cast<float*>(alloc.raw), S, rows, &ws);
    }
    k1<<<dim3(gx, s1), kLThreads, smem1, stream>>>(p, maps, ws, S, Ls);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess && (S > 1 || !first)) {
        const int64_t n = rows * p.state;
        const dim3 cg(static_cast<unsigned>((n + 255) / 256));
        e = first ? launch_pdl(m1_lane_carry<true>, cg, dim3(256), stream, p, ws, S)
                  : launch_pdl(m1_lane_carry<false>, cg, dim3(256), stream, p, ws, S);
        note_launch();
    }
    if (e == cudaSuccess && first && S > 1) {
        e = launch_pdl_smem(k2, dim3(gx, static_cast<unsigned>(S - 1)), dim3(kLThreads), smem2, stream, p, maps,
                       ws, S, Ls, 1);
        note_launch();
    }
    const cudaError_t ef = alloc.release();
    return e != cudaSuccess ? e : ef;
}

// Both traversals of the same inputs: fwd (reverse 0) and bwd (reverse 1)
// share every input but out / last_state (and out_acc).  One shared pass 1,
// a carry per direction, a pass 2 per direction over every segment: three
// exps per (step, state).  bwd.out == fwd.out with bwd.out_acc sums the two
// outputs in place (bwd's pass 2 runs after fwd's).  fwd.out == nullptr:
// final states only.  Each direction's carry starts at its own h0.
int m1_lane_bidir_segments(const M1Params& fwd) {
    if (!lane_applicable(fwd)) return 0;
    if (const int s = forced_segments(fwd)) return s;
    return lane_pick_segments(fwd, fwd.out ? 3 : 1);
}

// The bidirectional passes over a given workspace (both directions' segment
// aggregates, see lane_bidir_ws_floats).  first: the shared pass 1; then
// the carries (each direction from its own h0, ending in its last_state and,
// forward, dt_sum); finish: the two rescans (fwd.out != nullptr).  A
// sequence split over devices runs first + carries from zero (its summary),
// exchanges summaries, and later finish with the carries from the folded
// incoming states, reusing pass 1's aggregates from the same workspace.
static cudaError_t lane_bidir_run(const M1Params& fwd, const M1Params& bwd, int S, float* raw, bool first,
                                  bool finish, cudaStream_t stream) {
    const int64_t rows = fwd.batch * fwd.dim, Ls = fwd.len / S;
    LaneMaps maps;
    cudaError_t e = make_maps(fwd, &maps);
    if (e != cudaSuccess) return e;
    const int64_t gsz = fwd.dim / fwd.groups;
    const unsigned gx = static_cast<unsigned>(((gsz + kLRows - 1) / kLRows) * fwd.batch * fwd.groups);
    const bool dense = static_cast<int64_t>(gx) * S > lane_slots(false);
    constexpr int W = kLStagesWide, Dn = kLStagesDense;
    auto kb = dense ? m1_lane_pass1_bidir<Dn> : m1_lane_pass1_bidir<W>;
    auto kf = dense ? m1_lane_pass2<false, Dn> : m1_lane_pass2<false, W>;
    auto kr = dense ? m1_lane_pass2<true, Dn> : m1_lane_pass2<true, W>;
    const uint32_t smem = smem_bytes(dense ? Dn : W);
    if ((e = allow_smem(kb, smem)) != cudaSuccess || (e = allow_smem(kf, smem)) != cudaSuccess ||
        (e = allow_smem(kr, smem)) != cudaSuccess)
        return e;
    const size_t per = 2 * static_cast<size_t>(S) * rows * 16 + static_cast<size_t>(S) * rows;
    LaneWs wf, wb;
    carve(raw, S, rows, &wf);
    carve(raw + per, S, rows, &wb);
    const dim3 grid(gx, static_cast<unsigned>(S)), block(kLThreads);
    if (first) {
        kb<<<grid, block, smem, stream>>>(fwd, maps, wf, wb, S, Ls);
        note_launch();
        e = cudaGetLastError();
    }
    const int64_t n = rows * fwd.state;
    const dim3 cg(static_cast<unsigned>((n + 255) / 256));
    // the carries end in last_state; pass 2 leaves it alone
    M1Params f2 = fwd, b2 = bwd;
    f2.last_state = nullptr;
    b2.last_state = nullptr;
    if (e == cudaSuccess) e = launch_pdl(m1_lane_carry<false>, cg, dim3(256), stream, fwd, wf, S);
    if (e == cudaSuccess) note_launch();
    if (e == cudaSuccess) e = launch_pdl(m1_lane_carry<false>, cg, dim3(256), stream, bwd, wb, S);
    if (e == cudaSuccess) note_launch();
    if (finish && fwd.out) {
        if (e == cudaSuccess) e = launch_pdl_smem(kf, grid, block, smem, stream, f2, maps, wf, S, Ls, 0);
        if (e == cudaSuccess) note_launch();
        if (e == cudaSuccess) e = launch_pdl_smem(kr, grid, block, smem, stream, b2, maps, wb, S, Ls, 0);
        if (e == cudaSuccess) note_launch();
    }
    return e;
}

static size_t lane_bidir_ws_floats(int64_t rows, int S) {
    return 2 * (2 * static_cast<size_t>(S) * rows * 16 + static_cast<size_t>(S) * rows);
}

cudaError_t m1_lane_bidir_launch(const M1Params& fwd, const M1Params& bwd, int S, cudaStream_t stream) {
    LaneWsAlloc alloc(stream);
    cudaError_t e = alloc.get(lane_bidir_ws_floats(fwd.batch * fwd.dim, S) * sizeof(float));
    if (e != cudaSuccess) return e;
    e = lane_bidir_run(fwd, bwd, S, static_cast<float*>(alloc.raw), true, true, stream);
    const cudaError_t ef = alloc.release();
    return e != cudaSuccess ? e : ef;
}

// Two-phase form for sequence parallelism (caller's workspace).  The segment
// count depends on the shape and the device only, so both phases agree.
int m1_lane_bidir_plan(const M1Params& shape, size_t* ws_bytes) {
    M1Params q = shape;
    q.out = reinterpret_cast<float*>(uintptr_t(256));  // the plan of a call with outputs
    const bool ok = q.state <= 16 && q.state >= 1 && q.len % 4 == 0 && q.len >= 4 && q.dim % q.groups == 0 &&
                    q.len <= (int64_t(1) << 30) && q.batch * q.dim <= (int64_t(1) << 30) && encode_fn() != nullptr;
    if (!ok) {
        *ws_bytes = 0;
        return 0;
    }
    const int S = forced_segments(q) ? forced_segments(q) : lane_pick_segments(q, 3);
    *ws_bytes = lane_bidir_ws_floats(q.batch * q.dim, S) * sizeof(float);
    return S;
}

cudaError_t m1_lane_bidir_phase(const M1Params& fwd, const M1Params& bwd, void* workspace, size_t ws_bytes,
                                bool summary, cudaStream_t stream) {
    size_t need = 0;
    const int S = m1_lane_bidir_plan(fwd, &need);
    if (!S || !lane_applicable(fwd)) return cudaErrorNotSupported;
    if (ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u)) return cudaErrorInvalidValue;
    return lane_bidir_run(fwd, bwd, S, static_cast<float*>(workspace), summary, !summary, stream);
}

// ---- SS2D: the column-major traversals of an (h, w) grid, in place ---------
// The column-major ordering visits t = c*h + r, so its natural segments of h
// steps are the grid's columns.  A CTA owns 32 adjacent columns of 8
// channels of one batch entry (one thread per (channel, column), all of its
// states in registers) and sweeps the columns' steps in blocks of kColRB
// rows of the grid, staged by cp.async into double-buffered shared memory:
// each staged row of u, delta, B_n, C_n is 128 contiguous bytes of the grid,
// and B/C are staged once for the CTA's 8 channels.  The grid is read in
// place, with no transposed copy.  Three launches per ordering:
//  1. m1_col_pass1: per column, from zero, the forward end state, the
//     reverse end state (sum over r of prod_{r'<r} a_{r'} * b_r, from the
//     same sweep: one exp per (step, state)) and the sum of dt -- written as
//     the aggregates of forward segment c and of reverse segment w-1-c;
//  2. m1_lane_carry per direction (segments in traversal order);
//  3. m1_col_pass2: per column, the forward rescan from its incoming state
//     and then the reverse one, both adding y + D u into the output, the
//     second also applying the merge scale.
struct ColGrid {
    int64_t h, w;
    float scale;  // applied to the finished sum (1 for "sum", 0.25 for "mean")
    int64_t hs;   // grid rows per sub-segment (a multiple of kColRB)
    int k;        // sub-segments per column (1: a column is one segment)
};

constexpr int kColWarps = 8;
constexpr int kColRB = 8;  // grid rows per staged block
// one stage: B, C [kColRB][16][32], u, delta [kColWarps][kColRB][32] (floats)
constexpr int kColBC = kColRB * 16 * 32;
constexpr int kColX = kColWarps * kColRB * 32;
constexpr int kColStage = 2 * kColBC + 2 * kColX;
constexpr size_t kColSmem = 2 * kColStage * sizeof(float);

struct ColCta {
    int64_t bi, grp, c0, d0, c, d, row;
    int64_t r_lo, r_hi;  // grid rows of this CTA's sub-segment
    int j;               // its index within the column
    bool live;           // this thread's (channel, column) exists
};

__device__ __forceinline__ ColCta col_cta(const M1Params& p, const ColGrid& g) {
    ColCta t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    t.c0 = static_cast<int64_t>(blockIdx.x / g.k) * 32;
    t.j = static_cast<int>(blockIdx.x % g.k);
    t.r_lo = t.j * g.hs;
    t.r_hi = t.r_lo + g.hs < g.h ? t.r_lo + g.hs : g.h;
    t.d0 = static_cast<int64_t>(blockIdx.y) * kColWarps;
    t.bi = blockIdx.z;
    t.c = t.c0 + lane;
    t.d = t.d0 + warp;
    t.live = t.c < g.w && t.d < p.dim;
    t.row = t.bi * p.dim + (t.d < p.dim ? t.d : p.dim - 1);
    // a CTA's channels share one B/C group (channel blocks never straddle
    // a group: the launcher checks dim/groups % kColWarps == 0 or groups 1)
    t.grp = t.d0 / (p.dim / p.groups);
    return t;
}

__device__ __forceinline__ void cp_async_f(float* dst, const float* src, bool pred, int bytes) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(src), "r"(pred ? 16 : 0));
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(src), "r"(pred ? 4 : 0));
}

// Stage grid rows [r0, r0 + kColRB) of this CTA's columns: B (and C when
// WITH_C), u and delta.  VEC: 16-byte copies (w % 4 == 0, aligned tensors).
template <bool VEC, bool WITH_C>
__device__ __forceinline__ void col_stage(const M1Params& p, const ColGrid& g, const ColCta& t, int64_t r0,
                                          float* st) {
    constexpr int U = VEC ? 4 : 1;     // floats per copy
    constexpr int PER = 32 / U;        // copies per staged row
    const int64_t L = p.len, N = p.state;
    const float* Bg = p.B + (t.bi * p.groups + t.grp) * N * L + t.c0;
    const float* Cg = p.C + (t.bi * p.groups + t.grp) * N * L + t.c0;
    const int nbc = kColRB * static_cast<int>(N) * PER;
    for (int i = threadIdx.x; i < nbc; i += kColWarps * 32) {
        const int r = i / (static_cast<int>(N) * PER), n = (i / PER) % static_cast<int>(N), j = (i % PER) * U;
        const bool ok = r0 + r < t.r_hi && t.c0 + j < g.w;
        const int64_t o = ok ? n * L + (r0 + r) * g.w + j : 0;
        cp_async_f(st + (r * 16 + n) * 32 + j, Bg + o, ok, U * 4);
        if (WITH_C) cp_async_f(st + kColBC + (r * 16 + n) * 32 + j, Cg + o, ok, U * 4);
    }
    constexpr int nx = kColWarps * kColRB * PER;
    for (int i = threadIdx.x; i < nx; i += kColWarps * 32) {
        const int wv = i / (kColRB * PER), r = (i / PER) % kColRB, j = (i % PER) * U;
        const bool ok = r0 + r < t.r_hi && t.c0 + j < g.w && t.d0 + wv < p.dim;
        const int64_t o = ok ? ((t.bi * p.dim + t.d0 + wv) * L + (r0 + r) * g.w + t.c0 + j) : 0;
        const int so = (wv * kColRB + r) * 32 + j;
        cp_async_f(st + 2 * kColBC + so, p.u + o, ok, U * 4);
        cp_async_f(st + 2 * kColBC + kColX + so, p.delta + o, ok, U * 4);
    }
    asm volatile("cp.async.commit_group;\n" ::);
}

__device__ __forceinline__ void col_params(const M1Params& p, const ColCta& t, float (&a2)[16], float& bias,
                                           float& dsk) {
    const int64_t N = p.state, d = t.d < p.dim ? t.d : p.dim - 1;
#pragma unroll
    for (int n = 0; n < 16; ++n) a2[n] = n < N ? __ldg(p.A + d * N + n) * kLog2e : 0.f;
    bias = p.delta_bias ? __ldg(p.delta_bias + d) : 0.f;
    dsk = p.d_skip ? __ldg(p.d_skip + d) : 0.f;
}

// Sweep the CTA's columns over the grid rows, forward (REV false) or
// backward, calling blk(r0, rows, stage) for every staged block of rows.
template <bool VEC, bool WITH_C, bool REV, typename Blk>
__device__ __forceinline__ void col_sweep(const M1Params& p, const ColGrid& g, const ColCta& t, float* sm,
                                          Blk blk) {
    const int64_t nb = (t.r_hi - t.r_lo + kColRB - 1) / kColRB;
    auto block_r0 = [&](int64_t k) { return t.r_lo + (REV ? nb - 1 - k : k) * kColRB; };
    col_stage<VEC, WITH_C>(p, g, t, block_r0(0), sm);
    for (int64_t k = 0; k < nb; ++k) {
        float* st = sm + (k & 1) * kColStage;
        if (k + 1 < nb) {
            col_stage<VEC, WITH_C>(p, g, t, block_r0(k + 1), sm + ((k + 1) & 1) * kColStage);
            asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        }
        __syncthreads();
        const int64_t r0 = block_r0(k);
        const int rows = static_cast<int>(t.r_hi - r0 < kColRB ? t.r_hi - r0 : kColRB);
        blk(r0, rows, st);
        __syncthreads();  // the stage is refilled two blocks later
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kColWarps * 32, 2) m1_col_pass1(M1Params p, ColGrid g, LaneWs wf, LaneWs wb) {
    extern __shared__ __align__(16) float csm[];
    const ColCta t = col_cta(p, g);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t N = p.state, rows = p.batch * p.dim;
    float a2[16], bias, dsk;
    col_params(p, t, a2, bias, dsk);
    // states in pairs (n, n+1) for the packed fp32x2 instructions; a
    // missing odd partner keeps b = 0, so its state stays 0
    float2 hf[8], hr[8], pr[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        hf[k] = make_float2(0.f, 0.f);
        hr[k] = make_float2(0.f, 0.f);
        pr[k] = make_float2(1.f, 1.f);
    }
    float dts = 0.f;
    auto step = [&](int q, const float* st) {
        const int xo = (warp * kColRB + q) * 32 + lane;
        float dt = st[2 * kColBC + kColX + xo] + bias;
        if (p.delta_softplus) dt = softplus_fast(dt);
        const float du = dt * st[2 * kColBC + xo];
        dts += dt;
        const float2 dt2 = make_float2(dt, dt), du2 = make_float2(du, du);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (2 * k < N) {
                const float2 x = fmul2(dt2, make_float2(a2[2 * k], a2[2 * k + 1]));
                const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                const float* bp = st + (q * 16 + 2 * k) * 32 + lane;
                const float2 bu = fmul2(du2, make_float2(bp[0], 2 * k + 1 < N ? bp[32] : 0.f));
                hf[k] = ffma2(e, hf[k], bu);
                hr[k] = ffma2(pr[k], bu, hr[k]);
                pr[k] = fmul2(pr[k], e);
            }
        }
    };
    col_sweep<VEC, false, false>(p, g, t, csm, [&](int64_t, int rows, const float* st) {
        if (rows == kColRB) {
#pragma unroll
            for (int q = 0; q < kColRB; ++q) step(q, st);
        } else {
            for (int q = 0; q < rows; ++q) step(q, st);
        }
    });
    if (!t.live) return;
    // one segment per column: the carries' segment order (forward c,
    // reverse w-1-c); sub-segments: (column, sub-segment) for m1_col_fold
    const int64_t sf = g.k == 1 ? t.c : t.c * g.k + t.j;
    const int64_t sb = g.k == 1 ? g.w - 1 - t.c : sf;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (2 * k < N) {
            wf.hend[(sf * rows + t.row) * 16 + 2 * k] = hf[k].x;
            wb.hend[(sb * rows + t.row) * 16 + 2 * k] = hr[k].x;
        }
        if (2 * k + 1 < N) {
            wf.hend[(sf * rows + t.row) * 16 + 2 * k + 1] = hf[k].y;
            wb.hend[(sb * rows + t.row) * 16 + 2 * k + 1] = hr[k].y;
        }
    }
    wf.dtsum[sf * rows + t.row] = dts;
    wb.dtsum[sb * rows + t.row] = dts;
}

template <bool VEC, bool REV>
__device__ __forceinline__ void col_rescan(const M1Params& p, const ColGrid& g, const ColCta& t, float* sm,
                                           const float (&a2)[16], float bias, float dsk,
                                           const float (&hin)[16], float scale) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t L = p.len, N = p.state;
    // states in pairs (n, n+1) for the packed fp32x2 instructions; a
    // missing odd partner has h = b = c = 0
    float2 h[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
        h[k] = make_float2(hin[2 * k], hin[2 * k + 1]);
    float* out = p.out + t.row * L + t.c;
    auto step = [&](int q, const float* st) {
        const int xo = (warp * kColRB + q) * 32 + lane;
        float dt = st[2 * kColBC + kColX + xo] + bias;
        if (p.delta_softplus) dt = softplus_fast(dt);
        const float uu = st[2 * kColBC + xo];
        const float du = dt * uu;
        const float2 dt2 = make_float2(dt, dt), du2 = make_float2(du, du);
        float2 y = make_float2(dsk * uu, 0.f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (2 * k < N) {
                const bool odd = 2 * k + 1 < N;
                const float2 x = fmul2(dt2, make_float2(a2[2 * k], a2[2 * k + 1]));
                const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                const float* bp = st + (q * 16 + 2 * k) * 32 + lane;
                const float2 bu = fmul2(du2, make_float2(bp[0], odd ? bp[32] : 0.f));
                h[k] = ffma2(e, h[k], bu);
                y = ffma2(make_float2(bp[kColBC], odd ? bp[kColBC + 32] : 0.f), h[k], y);
            }
        }
        return y.x + y.y;
    };
    col_sweep<VEC, true, REV>(p, g, t, sm, [&](int64_t r0, int rows, const float* st) {
        if (rows == kColRB) {
            // the block's output values are requested before its steps run
            float ov[kColRB];
#pragma unroll
            for (int i = 0; i < kColRB; ++i) ov[i] = t.live ? out[(r0 + i) * g.w] : 0.f;
#pragma unroll
            for (int i = 0; i < kColRB; ++i) {
                const int q = REV ? kColRB - 1 - i : i;
                const float y = step(q, st);
                if (t.live) out[(r0 + q) * g.w] = (ov[q] + y) * scale;
            }
        } else {
            for (int i = 0; i < rows; ++i) {
                const int q = REV ? rows - 1 - i : i;
                const float y = step(q, st);
                if (t.live) {
                    float* o = out + (r0 + q) * g.w;
                    *o = (*o + y) * scale;
                }
            }
        }
    });
}

// Incoming state of this thread's sub-segment in one direction: the
// column's incoming state (from the carries) advanced over the sub-segments
// the traversal visits before this one (forward: j' < j; reverse: j' > j).
template <bool REV>
__device__ __forceinline__ void col_sub_hin(const M1Params& p, const ColGrid& g, const ColCta& t,
                                            const float (&a2)[16], const float* col_hin, const LaneWs& sub,
                                            float (&h)[16]) {
    const int64_t N = p.state, rows = p.batch * p.dim;
#pragma unroll
    for (int n = 0; n < 16; ++n) h[n] = (t.live && n < N) ? col_hin[n] : 0.f;
    if (g.k == 1 || !t.live) return;
    const int first = REV ? g.k - 1 : 0;
    for (int jj = first; jj != t.j; jj += REV ? -1 : 1) {
        const int64_t si = (t.c * g.k + jj) * rows + t.row;
        const float ds = sub.dtsum[si];
#pragma unroll
        for (int n = 0; n < 16; ++n)
            if (n < N) h[n] = fmaf(ex2_approx(a2[n] * ds), h[n], sub.hend[si * 16 + n]);
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kColWarps * 32, 2) m1_col_pass2(M1Params p, ColGrid g, LaneWs wf, LaneWs wb,
                                                                  LaneWs subf, LaneWs subr) {
    extern __shared__ __align__(16) float csm[];
    const ColCta t = col_cta(p, g);
    const int64_t rows = p.batch * p.dim;
    float a2[16], bias, dsk;
    col_params(p, t, a2, bias, dsk);
    const int64_t cc = t.c < g.w ? t.c : g.w - 1;
    float h0[16];
    col_sub_hin<false>(p, g, t, a2, wf.hin + (cc * rows + t.row) * 16, subf, h0);
    col_rescan<VEC, false>(p, g, t, csm, a2, bias, dsk, h0, 1.f);
    col_sub_hin<true>(p, g, t, a2, wb.hin + ((g.w - 1 - cc) * rows + t.row) * 16, subr, h0);
    col_rescan<VEC, true>(p, g, t, csm, a2, bias, dsk, h0, g.scale);
}

// Sub-segments -> column aggregates (time-split columns only): per (column,
// row, state) the forward fold over j = 0..k-1 and the reverse one over
// j = k-1..0 of the sub-segments' end states from zero, and the column's
// sum of dt, in the carries' segment order (forward c, reverse w-1-c).
__global__ void m1_col_fold(M1Params p, ColGrid g, LaneWs subf, LaneWs subr, LaneWs wf, LaneWs wb) {
    const int64_t rows = p.batch * p.dim, N = p.state;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= g.w * rows * N) return;
    const int64_t n = i % N, row = (i / N) % rows, c = i / (N * rows);
    const float a = __ldg(p.A + (row % p.dim) * N + n) * kLog2e;
    float hf = 0.f, hr = 0.f, dts = 0.f;
    for (int jj = 0; jj < g.k; ++jj) {
        const int64_t sf = (c * g.k + jj) * rows + row, sr = (c * g.k + (g.k - 1 - jj)) * rows + row;
        hf = fmaf(ex2_approx(a * subf.dtsum[sf]), hf, subf.hend[sf * 16 + n]);
        hr = fmaf(ex2_approx(a * subr.dtsum[sr]), hr, subr.hend[sr * 16 + n]);
        dts += subf.dtsum[sf];
    }
    wf.hend[(c * rows + row) * 16 + n] = hf;
    wb.hend[((g.w - 1 - c) * rows + row) * 16 + n] = hr;
    if (n == 0) {
        wf.dtsum[c * rows + row] = dts;
        wb.dtsum[(g.w - 1 - c) * rows + row] = dts;
    }
}

static int64_t sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    return sms;
}

cudaError_t m1_ss2d_cols_launch(const M1Params& p, int64_t h, int64_t w, float scale, cudaStream_t stream) {
    if (p.state > 16 || p.state < 1 || h < 1 || w < 1 || h * w != p.len || p.dim % p.groups != 0 ||
        p.batch > 65535 || (p.dim + kColWarps - 1) / kColWarps > 65535 || w > 0x7fffffff)
        return cudaErrorNotSupported;
    // a CTA's 8 channels must share one B/C group
    if (p.groups > 1 && (p.dim / p.groups) % kColWarps != 0) return cudaErrorNotSupported;
    const int64_t rows = p.batch * p.dim;
    const int S = static_cast<int>(w);
    // Split the columns in time when (columns / 32) x (channels / 8) x batch
    // CTAs would not give every SM two: about four CTAs per SM after the split.
    const int64_t base = ((w + 31) / 32) * ((p.dim + kColWarps - 1) / kColWarps) * p.batch;
    const int64_t sms = sm_count();
    int64_t k = 1;
    if (base < 2 * sms) {
        k = (4 * sms + base - 1) / base;
        const int64_t max_k = (h + kColRB - 1) / kColRB;
        k = k < max_k ? k : max_k;
    }
    const int64_t hs = ((((h + k - 1) / k) + kColRB - 1) / kColRB) * kColRB;
    k = (h + hs - 1) / hs;
    if (((w + 31) / 32) * k > 0x7fffffff) return cudaErrorNotSupported;
    const size_t per = 2 * static_cast<size_t>(S) * rows * 16 + static_cast<size_t>(S) * rows;
    // sub-segment aggregates: forward and reverse end states, one dt sum
    const size_t sub_n = static_cast<size_t>(S) * k * rows;
    const size_t sub = k > 1 ? 2 * sub_n * 16 + sub_n : 0;
    const bool vec = w % 4 == 0 && m1_pointers_aligned16(p);
    auto k1 = vec ? m1_col_pass1<true> : m1_col_pass1<false>;
    auto k2 = vec ? m1_col_pass2<true> : m1_col_pass2<false>;
    cudaError_t e;
    if ((e = allow_smem(k1, kColSmem)) != cudaSuccess || (e = allow_smem(k2, kColSmem)) != cudaSuccess) return e;
    LaneWsAlloc alloc(stream);
    if ((e = alloc.get((2 * per + sub) * sizeof(float))) != cudaSuccess) return e;
    float* raw = static_cast<float*>(alloc.raw);
    LaneWs wf, wb, subf{}, subr{};
    carve(raw, S, rows, &wf);
    carve(raw + per, S, rows, &wb);
    if (k > 1) {
        subf.hend = raw + 2 * per;
        subr.hend = subf.hend + sub_n * 16;
        subf.dtsum = subr.dtsum = subr.hend + sub_n * 16;
    }
    const ColGrid g{h, w, scale, hs, static_cast<int>(k)};
    const dim3 grid(static_cast<unsigned>(((w + 31) / 32) * k),
                    static_cast<unsigned>((p.dim + kColWarps - 1) / kColWarps), static_cast<unsigned>(p.batch));
    M1Params q = p;
    q.h0 = nullptr;
    q.last_state = nullptr;
    q.dt_sum = nullptr;
    if (k > 1)
        k1<<<grid, kColWarps * 32, kColSmem, stream>>>(q, g, subf, subr);
    else
        k1<<<grid, kColWarps * 32, kColSmem, stream>>>(q, g, wf, wb);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess && k > 1) {
        const int64_t nf = w * rows * q.state;
        m1_col_fold<<<static_cast<unsigned>((nf + 255) / 256), 256, 0, stream>>>(q, g, subf, subr, wf, wb);
        note_launch();
        e = cudaGetLastError();
    }
    const dim3 cg(static_cast<unsigned>((rows * q.state + 255) / 256));
    if (e == cudaSuccess) e = launch_pdl(m1_lane_carry<false>, cg, dim3(256), stream, q, wf, S);
    if (e == cudaSuccess) note_launch();
    if (e == cudaSuccess) e = launch_pdl(m1_lane_carry<false>, cg, dim3(256), stream, q, wb, S);
    if (e == cudaSuccess) note_launch();
    if (e == cudaSuccess) {
        k2<<<grid, kColWarps * 32, kColSmem, stream>>>(q, g, wf, wb, subf, subr);
        note_launch();
        e = cudaGetLastError();
    }
    const cudaError_t ef = alloc.release();
    return e != cudaSuccess ? e : ef;
}

int m1_lane_status_and_clear() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_m1_status, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_m1_status, &z, sizeof(int));
    return v;
}

}  // namespace b200scan
