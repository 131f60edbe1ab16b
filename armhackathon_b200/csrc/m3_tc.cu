// Mamba-3 SISO scan on the 5th-generation tensor cores (tcgen05), bf16
// operands with fp32 accumulation in tensor memory; selected with backend 3.
//
// Same chunked dual form as m3_chunk.cu (see its header for the algebra),
// with chunks of QC = 128 steps so every product is an M = 128 UMMA:
//   G     = Qr Kr^T                 M=128 (i) N=128 (j) K=dqk     -> TMEM cols [0,128)
//   W     = mask(l, scale, gamma) o G, rounded to bf16, back to shared memory
//   Y     = W X + (e^l o Qr) S^T     M=128 (i) N=dv    K=128, dqk -> TMEM cols [128,192)
//   dS^T  = (w o Kr)^T X             M=128 (n) N=dv    K=128      -> TMEM cols [192,256)
// One CTA of 4 warps per (batch, head); warp w owns TMEM lanes 32w..32w+31,
// i.e. rows i (for G, Y) and state rows n (for dS^T) of those lanes.  The
// state S^T (dqk x dv) stays fp32 in registers (thread n holds row n) and is
// rounded to bf16 only as the next chunk's MMA operand.  Operands use the
// canonical no-swizzle layouts: 8-row x 16-byte core matrices.
//
// Every wait on an mbarrier is bounded; on expiry the kernel records a
// timeout in g_tc_status, skips the remaining work and frees its tensor
// memory.  Requires dqk == 128, dv == 64, rank 1, len % 8 == 0 is NOT needed.
#include <cuda_bf16.h>

#include <cstdint>

#include "common.cuh"
#include "m3_scan.h"

namespace b200scan {

__device__ int g_tc_status;  // 0 ok, 1 an mbarrier wait timed out

namespace {

constexpr int kTcQ = 128;   // steps per chunk
constexpr int kTcN = 128;   // dqk
constexpr int kTcP = 64;    // dv
constexpr int kTcThreads = 128;
constexpr uint32_t kTmemCols = 256;

// ---- shared-memory operand layouts (bf16 elements, byte offsets) ----------
// K-major (rows r, K index k): core matrix (r/8, k/8) of 8x8 elements is 128
// contiguous bytes; SBO (next 8 rows) = 128 B, LBO (next 8 k) = rows/8 * 128 B.
__device__ __forceinline__ uint32_t kmaj_off(int r, int k, int rows) {
    return static_cast<uint32_t>(((k >> 3) * (rows >> 3) + (r >> 3)) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
// MN-major (MN index m, K index k): core matrix (m/8, k/8) = 8 K-rows of 8
// contiguous MN elements; SBO (next 8 m) = 128 B, LBO (next 8 k) = M/8 * 128 B.
__device__ __forceinline__ uint32_t mnmaj_off(int m, int k, int mdim) {
    return static_cast<uint32_t>(((k >> 3) * (mdim >> 3) + (m >> 3)) * 128 + (k & 7) * 16 + (m & 7) * 2);
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm100)
    return d;                              // base offset 0, no swizzle
}

// kind::f16 instruction descriptor: bf16 A/B, fp32 D, M x N, majors
__device__ __forceinline__ uint32_t instr_desc(int M, int N, bool a_mn, bool b_mn) {
    uint32_t d = 0;
    d |= 1u << 4;                 // D format f32
    d |= 1u << 7;                 // A format bf16
    d |= 1u << 10;                // B format bf16
    d |= (a_mn ? 1u : 0u) << 15;  // A major
    d |= (b_mn ? 1u : 0u) << 16;  // B major
    d |= static_cast<uint32_t>(N >> 3) << 17;
    d |= static_cast<uint32_t>(M >> 4) << 24;
    return d;
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(b)
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(count) : "memory");
}

// bounded wait for the phase with the given parity; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
    for (uint32_t it = 0; it < (1u << 24); ++it) {
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

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// shared memory map (bytes)
constexpr uint32_t kOffQ = 0;                         // Qr  K-major 128x128
constexpr uint32_t kOffQs = kOffQ + 128 * 128 * 2;    // e^l Qr K-major
constexpr uint32_t kOffK = kOffQs + 128 * 128 * 2;    // Kr  K-major (B of G)
constexpr uint32_t kOffKw = kOffK + 128 * 128 * 2;    // w Kr MN-major (A of dS^T: m=n, k=j)
constexpr uint32_t kOffW = kOffKw + 128 * 128 * 2;    // W   K-major (A of Y: r=i, k=j)
constexpr uint32_t kOffX = kOffW + 128 * 128 * 2;     // X   MN-major (B: m=p, k=j)
constexpr uint32_t kOffS = kOffX + 64 * 128 * 2;      // S^T MN-major (B: m=p, k=n)
constexpr uint32_t kOffGate = kOffS + 64 * 128 * 2;   // lcum, scale, gamma, w (fp32 x 128)
constexpr uint32_t kOffMisc = kOffGate + 4 * 128 * 4; // eQ, mbarrier, tmem base
constexpr uint32_t kTcSmem = kOffMisc + 64;

__global__ void __launch_bounds__(kTcThreads, 1) m3_tc_kernel(M3Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* lcum = reinterpret_cast<float*>(smem + kOffGate);
    float* scl = lcum + kTcQ;
    float* gam = scl + kTcQ;
    float* wdec = gam + kTcQ;
    float* eQ = reinterpret_cast<float*>(smem + kOffMisc);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffMisc + 16);
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc + 32);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t bh = blockIdx.x;
    const int64_t H = p.heads, L = p.len;
    const int64_t bi = bh / H, h = bh % H;
    const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
    const int64_t gate_base = (bi * H + h) * L;
    const int n_chunks = static_cast<int>((L + kTcQ - 1) / kTcQ);
    constexpr int half = kTcN / 2;

    if (warp == 0) {
        const uint32_t slot = static_cast<uint32_t>(__cvta_generic_to_shared(tmem_base_slot));
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_slot;
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tG = tmem, tY = tmem + 128, tS = tmem + 192;

    // fp32 state row n = tid of S^T (dqk x dv)
    float S[kTcP];
#pragma unroll
    for (int q = 0; q < kTcP; ++q) S[q] = 0.f;
    uint32_t phase = 0;
    bool ok_run = true;

    const uint32_t id_G = instr_desc(128, 128, false, false);
    const uint32_t id_Y = instr_desc(128, kTcP, false, true);
    const uint32_t id_S = instr_desc(128, kTcP, true, true);

    for (int ch = 0; ch < n_chunks; ++ch) {
        const int64_t it0 = static_cast<int64_t>(ch) * kTcQ;
        // ---- gates (warp 0): cumulative log decay, trapezoid weights
        if (warp == 0) {
            float lv[4], sc[4], gm[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = lane * 4 + e;  // contiguous steps per lane
                const int64_t it = it0 + j;
                lv[e] = sc[e] = gm[e] = 0.f;
                if (it < L) {
                    const int64_t t = p.reverse ? L - 1 - it : it;
                    const int64_t g = gate_base + t;
                    const float gamma = p.dt[g] * sigmoid_f(p.trap[g]);
                    float shifted = 0.f;
                    if (it + 1 < L) {
                        const int64_t nx = p.reverse ? g - 1 : g + 1;
                        shifted = p.dt[nx] * (1.f - sigmoid_f(p.trap[nx]));
                    }
                    lv[e] = p.adt[g];
                    sc[e] = gamma + shifted;
                    gm[e] = gamma;
                }
            }
            lv[1] += lv[0];
            lv[2] += lv[1];
            lv[3] += lv[2];
            float run = lv[3];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float v = __shfl_up_sync(0xffffffffu, run, o);
                if (lane >= o) run += v;
            }
            const float before = run - lv[3];
            const float last = __shfl_sync(0xffffffffu, run, 31);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = lane * 4 + e;
                const float l = before + lv[e];
                lcum[j] = l;
                scl[j] = sc[e];
                gam[j] = gm[e];
                wdec[j] = expf(last - l) * sc[e];
            }
            if (lane == 0) eQ[0] = expf(last);
        }
        __syncthreads();
        // ---- operands: rotated q/k rows, e^l q, w k, x (all bf16)
        for (int idx = tid; idx < kTcQ * half; idx += kTcThreads) {
            const int j = idx / half, pi = idx % half;
            const int64_t it = it0 + j;
            float q0 = 0.f, q1 = 0.f, k0 = 0.f, k1 = 0.f;
            if (it < L) {
                const int64_t t = p.reverse ? L - 1 - it : it;
                const int64_t qk = (bi * L + t) * kTcN;
                const float* qb = p.q_bias + h * kTcN;
                const float* kb = p.k_bias + h * kTcN;
                const int64_t cs = ((bi * L + t) * H + h) * half + pi;
                const float c = p.cos[cs], s = p.sin[cs];
                float a0 = p.q[qk + 2 * pi] + qb[2 * pi], a1 = p.q[qk + 2 * pi + 1] + qb[2 * pi + 1];
                q0 = a0 * c - a1 * s;
                q1 = a0 * s + a1 * c;
                a0 = p.k[qk + 2 * pi] + kb[2 * pi];
                a1 = p.k[qk + 2 * pi + 1] + kb[2 * pi + 1];
                k0 = a0 * c - a1 * s;
                k1 = a0 * s + a1 * c;
            }
            const float el = it < L ? expf(lcum[j]) : 0.f;
            const float w = wdec[j];
            const int n0 = 2 * pi, n1 = 2 * pi + 1;
            *reinterpret_cast<uint16_t*>(smem + kOffQ + kmaj_off(j, n0, 128)) = bf16_bits(q0);
            *reinterpret_cast<uint16_t*>(smem + kOffQ + kmaj_off(j, n1, 128)) = bf16_bits(q1);
            *reinterpret_cast<uint16_t*>(smem + kOffQs + kmaj_off(j, n0, 128)) = bf16_bits(el * q0);
            *reinterpret_cast<uint16_t*>(smem + kOffQs + kmaj_off(j, n1, 128)) = bf16_bits(el * q1);
            *reinterpret_cast<uint16_t*>(smem + kOffK + kmaj_off(j, n0, 128)) = bf16_bits(k0);
            *reinterpret_cast<uint16_t*>(smem + kOffK + kmaj_off(j, n1, 128)) = bf16_bits(k1);
            *reinterpret_cast<uint16_t*>(smem + kOffKw + mnmaj_off(n0, j, 128)) = bf16_bits(w * k0);
            *reinterpret_cast<uint16_t*>(smem + kOffKw + mnmaj_off(n1, j, 128)) = bf16_bits(w * k1);
        }
        for (int idx = tid; idx < kTcQ * kTcP; idx += kTcThreads) {
            const int j = idx / kTcP, pp = idx % kTcP;
            const int64_t it = it0 + j;
            float v = 0.f;
            if (it < L) {
                const int64_t t = p.reverse ? L - 1 - it : it;
                v = p.v[((bi * L + t) * H + h) * kTcP + pp];
            }
            *reinterpret_cast<uint16_t*>(smem + kOffX + mnmaj_off(pp, j, kTcP)) = bf16_bits(v);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- G = Qr Kr^T
        if (tid == 0) {
#pragma unroll
            for (int kb = 0; kb < kTcN / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kOffQ + kb * 2 * (128 / 8) * 128, (128 / 8) * 128, 128);
                const uint64_t b = smem_desc(sbase + kOffK + kb * 2 * (128 / 8) * 128, (128 / 8) * 128, 128);
                umma(tG, a, b, id_G, kb > 0);
            }
            umma_commit(bar);
        }
        if (__syncthreads_or(!mbar_wait(bar, phase))) {
            ok_run = false;
            if (tid == 0) atomicExch(&g_tc_status, 1);
            break;
        }
        phase ^= 1;
        tc_fence_after();
        // ---- W = mask o G -> bf16, row i = tid
        {
            const int i = tid;
            const float li = lcum[i], gi = gam[i];
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
                float g[32];
                tmem_ld32(tG + t_lane + cb * 32, g);
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int j = cb * 32 + c;
                    float m = 0.f;
                    if (j < i) m = expf(li - lcum[j]) * scl[j];
                    else if (j == i) m = gi;
                    *reinterpret_cast<uint16_t*>(smem + kOffW + kmaj_off(i, j, 128)) =
                        bf16_bits(m * g[c]);
                }
            }
        }
        // S^T (bf16) for Y's inter-chunk term, row n = tid
#pragma unroll
        for (int q = 0; q < kTcP; ++q)
            *reinterpret_cast<uint16_t*>(smem + kOffS + mnmaj_off(q, tid, kTcP)) = bf16_bits(S[q]);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- Y = W X + (e^l Qr) S^T ; dS^T = (w Kr)^T X
        if (tid == 0) {
            for (int kb = 0; kb < kTcQ / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kOffW + kb * 2 * (128 / 8) * 128, (128 / 8) * 128, 128);
                const uint64_t b = smem_desc(sbase + kOffX + kb * 2 * (kTcP / 8) * 128, (kTcP / 8) * 128, 128);
                umma(tY, a, b, id_Y, kb > 0);
            }
            if (ch > 0) {
                for (int kb = 0; kb < kTcN / 16; ++kb) {
                    const uint64_t a = smem_desc(sbase + kOffQs + kb * 2 * (128 / 8) * 128, (128 / 8) * 128, 128);
                    const uint64_t b = smem_desc(sbase + kOffS + kb * 2 * (kTcP / 8) * 128, (kTcP / 8) * 128, 128);
                    umma(tY, a, b, id_Y, 1);
                }
            }
            for (int kb = 0; kb < kTcQ / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kOffKw + kb * 2 * (128 / 8) * 128, (128 / 8) * 128, 128);
                const uint64_t b = smem_desc(sbase + kOffX + kb * 2 * (kTcP / 8) * 128, (kTcP / 8) * 128, 128);
                umma(tS, a, b, id_S, kb > 0);
            }
            umma_commit(bar);
        }
        if (__syncthreads_or(!mbar_wait(bar, phase))) {
            ok_run = false;
            if (tid == 0) atomicExch(&g_tc_status, 1);
            break;
        }
        phase ^= 1;
        tc_fence_after();
        // ---- epilogue: y row i = tid; state row n = tid
        {
            const int i = tid;
            const int64_t it = it0 + i;
            float y[64];
            tmem_ld32(tY + t_lane, *reinterpret_cast<float(*)[32]>(y));
            tmem_ld32(tY + t_lane + 32, *reinterpret_cast<float(*)[32]>(y + 32));
            if (it < L) {
                const int64_t t = p.reverse ? L - 1 - it : it;
                const int64_t voff = ((bi * L + t) * H + h) * kTcP;
                float* o = p.out + ((bi * H + h) * L + t) * kTcP;
#pragma unroll
                for (int q = 0; q < kTcP; q += 4) {
                    const float4 vv = *reinterpret_cast<const float4*>(p.v + voff + q);
                    float r4[4] = {fmaf(dsk, vv.x, y[q]), fmaf(dsk, vv.y, y[q + 1]),
                                   fmaf(dsk, vv.z, y[q + 2]), fmaf(dsk, vv.w, y[q + 3])};
                    if (p.z) {
                        const float4 zz = *reinterpret_cast<const float4*>(p.z + voff + q);
                        r4[0] *= silu_f(zz.x);
                        r4[1] *= silu_f(zz.y);
                        r4[2] *= silu_f(zz.z);
                        r4[3] *= silu_f(zz.w);
                    }
                    *reinterpret_cast<float4*>(o + q) = make_float4(r4[0], r4[1], r4[2], r4[3]);
                }
            }
            float ds[64];
            tmem_ld32(tS + t_lane, *reinterpret_cast<float(*)[32]>(ds));
            tmem_ld32(tS + t_lane + 32, *reinterpret_cast<float(*)[32]>(ds + 32));
            const float e = eQ[0];
#pragma unroll
            for (int q = 0; q < kTcP; ++q) S[q] = fmaf(e, S[q], ds[q]);
            if (p.last_bx && ch == n_chunks - 1) {
                // scale_T * k_T: rotated k of the final step, fp32 (recomputed)
                const int jl = static_cast<int>(L - 1 - it0);
                if (tid < half) {
                    const int64_t itl = it0 + jl;
                    const int64_t t = p.reverse ? L - 1 - itl : itl;
                    const int64_t qk = (bi * L + t) * kTcN;
                    const float* kb = p.k_bias + h * kTcN;
                    const int64_t cs = ((bi * L + t) * H + h) * half + tid;
                    const float c = p.cos[cs], s = p.sin[cs];
                    const float a0 = p.k[qk + 2 * tid] + kb[2 * tid];
                    const float a1 = p.k[qk + 2 * tid + 1] + kb[2 * tid + 1];
                    p.last_bx[bh * kTcN + 2 * tid] = scl[jl] * (a0 * c - a1 * s);
                    p.last_bx[bh * kTcN + 2 * tid + 1] = scl[jl] * (a0 * s + a1 * c);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (!ok_run) {
        // a wait expired: give the MMAs in flight a second bounded wait
        // before the tensor memory they write is released
        mbar_wait(bar, phase);
    } else if (p.last_state) {
#pragma unroll
        for (int q = 0; q < kTcP; ++q) p.last_state[(bh * kTcP + q) * kTcN + tid] = S[q];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

}  // namespace

bool m3_tc_applicable(const M3Params& p) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return p.psi == nullptr && p.rank == 1 && p.dqk == kTcN && p.dv == kTcP && al(p.v) &&
           al(p.z) && al(p.out);
}

cudaError_t m3_tc_launch(const M3Params& p, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(m3_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kTcSmem));
    if (e != cudaSuccess) return e;
    m3_tc_kernel<<<dim3(static_cast<unsigned>(p.batch * p.heads)), kTcThreads, kTcSmem, stream>>>(p);
    return cudaGetLastError();
}

int m3_tc_status_and_clear() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
    cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
    return v;
}

}  // namespace b200scan
