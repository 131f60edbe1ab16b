// Mamba-3 SISO scan on the 5th-generation tensor cores (tcgen05), bf16
// operands with fp32 accumulation in tensor memory; selected with backend 3.
//
// Same chunked dual form as m3_chunk.cu (see its header for the algebra),
// with chunks of QC = 128 steps so every product is an M = 128 UMMA, in
// three launches so every chunk of every (batch, head) runs in parallel:
//
//  A. m3_tc_dstate, one CTA per (batch*head, chunk):
//       dS^T = Kr^T (w o X)      M=128 (n) N=dv K=128 (steps) -> TMEM
//     to the workspace in fp32, with the chunk's total decay 2^{l2_last}.
//     (Kr's K-major core matrices are byte for byte the MN-major A operand
//     of dS^T; only the descriptor strides differ.)
//  B. m3_tc_state: per (batch*head, slice of the state), walks the chunks
//     S_in(c+1) = 2^{l2_last(c)} S_in(c) + dS(c) in fp32 and writes S_in(c)
//     as chunk c's bf16 operand image; the final state is last_state.
//  C. m3_tc_out, persistent, per (batch*head, chunk):
//       G = Qr Kr^T              M=128 (i) N=128 (j) K=dqk
//       Z = Qr S_in^T            M=128 (i) N=dv      K=dqk   (chunk > 0)
//       W = mask(l, scale, gamma) o G -> bf16, over Qr in shared memory
//       Y = W X                  M=128 (i) N=dv      K=128
//       y = (Y + 2^{l2_i} Z + D x) * silu(z)
// Operands use the canonical no-swizzle layouts (8-row x 16-byte core
// matrices); every operand is staged with 16-byte stores that fill whole
// 128-byte rows of banks.  The state stays fp32 end to end; only MMA
// operands are rounded to bf16.
//
// Every wait on an mbarrier is bounded; on expiry the kernel records a
// timeout in g_tc_status, skips the remaining work, waits (bounded) for the
// MMAs in flight and frees its tensor memory.  Requires dqk == 128,
// dv == 64, rank 1 and 16-byte aligned tensors.
#include <cuda_bf16.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "m1_scan.h"
#include "m3_angles.h"
#include "m3_scan.h"

namespace b200scan {

__device__ int g_tc_status;
  // 0 ok, 1 an mbarrier wait timed out

namespace {

constexpr int kTcQ = 128;   // steps per chunk
constexpr int kTcN = 128;   // dqk
constexpr int kTcP = 64;    // dv

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



// one cvt.rn.bf16x2.f32 (round to nearest even)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
}
__device__ __forceinline__ void ld8(const float* g, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(g);
    const float4 b = *reinterpret_cast<const float4*>(g + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void ldg8(const float* g, float (&f)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(g));
    const float4 b = __ldg(reinterpret_cast<const float4*>(g + 4));
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// bulk prefetch of [g, g + bytes) into L2 (16-byte aligned, multiple of 16)
__device__ __forceinline__ void prefetch_l2(const void* g, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(g), "r"(bytes) : "memory");
}

// bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from this GPU's global memory into shared memory, completing on `bar`
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
        "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
                 "r"(bytes)
                 : "memory");
}

// line prefetches into L2 (the load/store unit, not the bulk-copy engine)
// for short rows: one per 128 bytes of [g, g + bytes)
__device__ __forceinline__ void prefetch_lines(const void* g, uint32_t bytes) {
    const char* c = static_cast<const char*>(g);
    for (uint32_t o = 0; o < bytes; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(slot));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols));
}

// CTA-uniform bounded wait; false (and the status flag set) on expiry.
// Thread 0 polls; the others wait at the barrier without taking issue slots.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity) {
    const bool mine = threadIdx.x == 0 ? !mbar_wait(bar, parity) : false;
    const bool expired = __syncthreads_or(mine);
    if (expired && threadIdx.x == 0) atomicExch(&g_tc_status, 1);
    return !expired;
}

constexpr int kTcThreads2 = 256;
constexpr uint32_t kChunkImg = 128 * 128 * 2;  // bytes of one 128 x 128 bf16 operand
constexpr uint32_t kStImg = 128 * 64 * 2;      // bytes of one dqk x dv bf16 operand
constexpr uint32_t kChunkSt = 128 * 64 * 4;    // bytes of one fp32 dqk x dv state

// workspace of one launch
struct TcWs {
    float* st;        // [bh][chunk] dS^T, fp32, row n, column p
    uint8_t* simg;    // [bh][chunk] S_in^T, bf16 MN-major operand image (m = p, k = n)
    float* decay;     // [bh][chunk] e^{l_last}
};

// Gates of one chunk (warp 0): cumulative log2 decay l2 (lcum), trapezoid
// scale, gamma, state weight w_j = 2^(l2_last - l2_j) * scale_j, and
// (lane 0) the chunk's total decay.
__device__ __forceinline__ void tile_gates(const M3Params& p, int64_t bh, int64_t it0, float* lcum,
                                           float* scl, float* gam, float* wdec, float* decay) {
    constexpr float kLog2eF = 1.4426950408889634f;
    const int lane = threadIdx.x & 31;
    const int64_t L = p.len, gate_base = bh * L;
    float lv[4], sc[4], gm[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int64_t it = it0 + lane * 4 + e;
        lv[e] = sc[e] = gm[e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t g = gate_base + t;
            const float gamma = __ldg(p.dt + g) * sigmoid_f(__ldg(p.trap + g));
            float shifted = 0.f;
            if (it + 1 < L) {
                const int64_t nx = p.reverse ? g - 1 : g + 1;
                shifted = __ldg(p.dt + nx) * (1.f - sigmoid_f(__ldg(p.trap + nx)));
            }
            lv[e] = __ldg(p.adt + g) * kLog2eF;
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
        wdec[j] = ex2_approx(last - l) * sc[e];
    }
    if (decay && lane == 0) *decay = ex2_approx(last);
}

// X items: step j, 8 consecutive channels = one 16-byte chunk of an
// MN-major (m = p, k = j) operand.  Item r of this thread:
__device__ __forceinline__ void x_item(int r, int& j, int& pc) {
    const int item = threadIdx.x + r * kTcThreads2;
    const int hi = item >> 5;
    j = (hi >> 1) * 8 + (item & 7);
    pc = ((item >> 3) & 3) + 4 * (hi & 1);
}
constexpr int kXItems = 128 * 8 / kTcThreads2;

__device__ __forceinline__ void load_x(const M3Params& p, int64_t bi, int64_t h, int64_t it0,
                                       float (&xv)[kXItems][8]) {
    const int64_t L = p.len, H = p.heads;
#pragma unroll
    for (int r = 0; r < kXItems; ++r) {
        int j, pc;
        x_item(r, j, pc);
        const int64_t it = it0 + j;
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[r][e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            ldg8(p.v + ((bi * L + t) * H + h) * kTcP + pc * 8, xv[r]);
        }
    }
}

// Rotated k (and, with WITH_Q, rotated q) rows of one chunk into K-major
// 128 x 128 operand images.  One item = step j, 8 consecutive dims (4
// rotation pairs); a warp covers 8 steps x 4 dim-chunks, i.e. 128
// contiguous bytes of each input row.  Items 2m and 2m+1 share their dim
// chunk and are both loaded before either is stored.
template <bool WITH_Q>
__device__ __forceinline__ void stage_qk(const M3Params& p, int64_t bi, int64_t h, int64_t it0,
                                         uint8_t* img_q, uint8_t* img_k, const float* qb,
                                         const float* kb) {
    const int64_t L = p.len, H = p.heads;
    const int tid = threadIdx.x;
    for (int m = 0; m < 128 * 16 / kTcThreads2 / 2; ++m) {
        float qa[2][8], ka[2][8], cc[2][4], ss[2][4];
        int jj[2];
        int kc = 0;
        bool live[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int item = tid + (2 * m + u) * kTcThreads2;
            const int hi = item >> 5;
            jj[u] = (hi & 15) * 8 + (item & 7);
            kc = ((item >> 3) & 3) + 4 * (hi >> 4);
            const int64_t it = it0 + jj[u];
            live[u] = it < L;
            const int64_t t = live[u] ? (p.reverse ? L - 1 - it : it) : 0;
            const int64_t qk = (bi * L + t) * kTcN + kc * 8;
            const int64_t cs = ((bi * L + t) * H + h) * (kTcN / 2) + kc * 4;
            if (WITH_Q) ldg8(p.q + qk, qa[u]);
            ldg8(p.k + qk, ka[u]);
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cos + cs));
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sin + cs));
            cc[u][0] = c4.x; cc[u][1] = c4.y; cc[u][2] = c4.z; cc[u][3] = c4.w;
            ss[u][0] = s4.x; ss[u][1] = s4.y; ss[u][2] = s4.z; ss[u][3] = s4.w;
        }
        float qbb[8], kbb[8];
        if (WITH_Q) ld8(qb + kc * 8, qbb);
        ld8(kb + kc * 8, kbb);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float qr[8], kr[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (WITH_Q) {
                    const float a0 = qa[u][2 * e] + qbb[2 * e], a1 = qa[u][2 * e + 1] + qbb[2 * e + 1];
                    qr[2 * e] = a0 * cc[u][e] - a1 * ss[u][e];
                    qr[2 * e + 1] = a0 * ss[u][e] + a1 * cc[u][e];
                }
                const float a0 = ka[u][2 * e] + kbb[2 * e], a1 = ka[u][2 * e + 1] + kbb[2 * e + 1];
                kr[2 * e] = a0 * cc[u][e] - a1 * ss[u][e];
                kr[2 * e + 1] = a0 * ss[u][e] + a1 * cc[u][e];
            }
            if (!live[u]) {
#pragma unroll
                for (int e = 0; e < 8; ++e) qr[e] = kr[e] = 0.f;
            }
            const uint32_t ko = kmaj_off(jj[u], kc * 8, 128);
            if (WITH_Q) *reinterpret_cast<uint4*>(img_q + ko) = pack8(qr);
            *reinterpret_cast<uint4*>(img_k + ko) = pack8(kr);
        }
    }
}

// ---------------------------------------------------------------------------
// Kernel A: per (batch*head, chunk) the chunk's state contribution
// dS^T = Kr^T (w o X) (fp32, to the workspace), its total decay, and for the
// last chunk scale_T * k_T.
constexpr uint32_t kAK = 0;                        // Kr K-major; A of dS^T as MN-major
constexpr uint32_t kAXw = kAK + kChunkImg;         // w o X MN-major (B)
constexpr uint32_t kAGate = kAXw + 128 * 64 * 2;   // lcum, scale, gamma, w
constexpr uint32_t kAMisc = kAGate + 4 * 128 * 4;
constexpr uint32_t kASmem = kAMisc + 64;

__global__ void __launch_bounds__(kTcThreads2, 3) m3_tc_dstate(M3Params p, TcWs ws, int n_chunks) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* lcum = reinterpret_cast<float*>(smem + kAGate);
    float* scl = lcum + kTcQ;
    float* gam = scl + kTcQ;
    float* wdec = gam + kTcQ;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kAMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kAMisc + 16);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t H = p.heads, L = p.len, BH = p.batch * p.heads;
    const int64_t bh = blockIdx.x % BH;
    const int ch = static_cast<int>(blockIdx.x / BH);
    const int64_t bi = bh / H, h = bh % H;
    const int64_t bhc = bh * n_chunks + ch;
    const int64_t it0 = static_cast<int64_t>(ch) * kTcQ;

    if (warp == 0) tmem_alloc(tmem_slot, 64);
    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    float xv[kXItems][8];
    load_x(p, bi, h, it0, xv);
    if (warp == 0) tile_gates(p, bh, it0, lcum, scl, gam, wdec, ws.decay + bhc);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kXItems; ++r) {
        int j, pc;
        x_item(r, j, pc);
        const float w = wdec[j];
        float xw[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) xw[e] = w * xv[r][e];
        *reinterpret_cast<uint4*>(smem + kAXw + mnmaj_off(pc * 8, j, kTcP)) = pack8(xw);
    }
    stage_qk<false>(p, bi, h, it0, nullptr, smem + kAK, p.q_bias + h * kTcN, p.k_bias + h * kTcN);
    if (p.last_bx && ch == n_chunks - 1 && tid < kTcN / 2) {
        // scale_T * k_T: rotated k of the final step, fp32
        const int jl = static_cast<int>(L - 1 - it0);
        const int64_t t = p.reverse ? 0 : L - 1;
        const int64_t qk = (bi * L + t) * kTcN;
        const float* kb = p.k_bias + h * kTcN;
        const int64_t cs = ((bi * L + t) * H + h) * (kTcN / 2) + tid;
        const float c = p.cos[cs], s = p.sin[cs];
        const float a0 = p.k[qk + 2 * tid] + kb[2 * tid];
        const float a1 = p.k[qk + 2 * tid + 1] + kb[2 * tid + 1];
        p.last_bx[bh * kTcN + 2 * tid] = scl[jl] * (a0 * c - a1 * s);
        p.last_bx[bh * kTcN + 2 * tid + 1] = scl[jl] * (a0 * s + a1 * c);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) {
        const uint32_t id_S = instr_desc(128, kTcP, true, true);
        // A = Kr viewed MN-major (m = n, k = j): next 8 n = 2048 B (SBO),
        // next 8 j = 128 B (LBO); 16 steps of j = 256 B
        for (int kb = 0; kb < kTcQ / 16; ++kb) {
            const uint64_t a = smem_desc(sbase + kAK + kb * 2 * 128, 128, 16 * 128);
            const uint64_t b = smem_desc(sbase + kAXw + kb * 2 * 8 * 128, 8 * 128, 128);
            umma(tmem, a, b, id_S, kb > 0);
        }
        umma_commit(bar);
    }
    if (cta_wait(bar, 0)) {
        tc_fence_after();
        const int n = (warp & 3) * 32 + lane, hc = warp >> 2;
        float ds[32];
        tmem_ld32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + hc * 32, ds);
        float* st = ws.st + bhc * (kTcN * kTcP) + n * kTcP + hc * 32;
#pragma unroll
        for (int q = 0; q < 32; q += 4)
            *reinterpret_cast<float4*>(st + q) = make_float4(ds[q], ds[q + 1], ds[q + 2], ds[q + 3]);
    } else {
        mbar_wait(bar, 0);  // the MMA still in flight: bounded second wait
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

// ---------------------------------------------------------------------------
// Kernel B: S_in(0) = 0; S_in(c+1) = decay(c) S_in(c) + dS(c) in fp32.
// S_in(c) is written as chunk c's bf16 MN-major operand image; the final
// state goes to last_state.  A thread owns 4 consecutive (n, p) entries;
// slices of 1024 entries per CTA.
constexpr int kStSlices = (kTcN * kTcP) / (kTcThreads2 * 4);

__global__ void __launch_bounds__(kTcThreads2) m3_tc_state(M3Params p, TcWs ws, int n_chunks) {
    const int64_t bh = blockIdx.x;
    const int e0 = (blockIdx.y * kTcThreads2 + threadIdx.x) * 4;
    const int n = e0 / kTcP, p0 = e0 % kTcP;
    const uint32_t img_off = mnmaj_off(p0, n, kTcP);  // 4 consecutive p: 8 bytes
    float4 S = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* base = ws.st + bh * n_chunks * (kTcN * kTcP) + e0;
    uint8_t* img = ws.simg + bh * n_chunks * kStImg + img_off;
    const float* dec = ws.decay + bh * n_chunks;
    float4 nd = __ldg(reinterpret_cast<const float4*>(base));
    float nq = __ldg(dec);
    for (int c = 0; c < n_chunks; ++c) {
        const float4 d = nd;
        const float q = nq;
        if (c + 1 < n_chunks) {
            nd = __ldg(reinterpret_cast<const float4*>(base + static_cast<int64_t>(c + 1) * (kTcN * kTcP)));
            nq = __ldg(dec + c + 1);
        }
        if (c > 0)
            *reinterpret_cast<uint2*>(img + static_cast<int64_t>(c) * kStImg) =
                make_uint2(pack_bf16x2(S.x, S.y), pack_bf16x2(S.z, S.w));
        S.x = fmaf(q, S.x, d.x);
        S.y = fmaf(q, S.y, d.y);
        S.z = fmaf(q, S.z, d.z);
        S.w = fmaf(q, S.w, d.w);
    }
    if (p.last_state) {
        // state entries are (n, p) row-major; last_state is (p, n)
        const float sv[4] = {S.x, S.y, S.z, S.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) p.last_state[(bh * kTcP + p0 + e) * kTcN + n] = sv[e];
    }
}

// ---------------------------------------------------------------------------
// Kernel C, persistent (CTA b takes tiles b, b + gridDim.x, ...; tile =
// chunk * batch*heads + batch*head): the chunk's output
//   G = Qr Kr^T -> TMEM [0,128);  Z = Qr S_in^T -> TMEM [128,192) (chunk > 0)
//   W = mask o G -> bf16 over Qr;  Y = W X -> TMEM [0,64)
//   y = (Y + 2^{l2_i} Z + D x) * silu(z)
constexpr uint32_t kCQ = 0;                        // Qr K-major (A of G, Z); then W (A of Y)
constexpr uint32_t kCK = kCQ + kChunkImg;          // Kr K-major (B of G)
constexpr uint32_t kCX = kCK + kChunkImg;          // X MN-major (B of Y)
constexpr uint32_t kCS = kCX + 128 * 64 * 2;       // S_in^T MN-major (B of Z)
constexpr uint32_t kCGate = kCS + kStImg;          // lcum, scale, gamma, w
constexpr uint32_t kCMisc = kCGate + 4 * 128 * 4;
constexpr uint32_t kCSmem = kCMisc + 64;

__global__ void __launch_bounds__(kTcThreads2, 2) m3_tc_out(M3Params p, TcWs ws, int n_chunks) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* lcum = reinterpret_cast<float*>(smem + kCGate);  // log2 units
    float* scl = lcum + kTcQ;
    float* gam = scl + kTcQ;
    float* wdec = gam + kTcQ;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kCMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kCMisc + 16);
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t H = p.heads, L = p.len, BH = p.batch * p.heads;
    const int64_t n_tiles = BH * n_chunks;

    if (warp == 0) tmem_alloc(tmem_slot, 256);
    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int hc = warp >> 2;  // column half of this warp
    const uint32_t tG = tmem, tY = tmem, tZ = tmem + 128;
    uint32_t phase = 0;
    bool ok = true;

    for (int64_t tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        const int64_t bh = tile % BH;
        const int ch = static_cast<int>(tile / BH);
        const int64_t bi = bh / H, h = bh % H;
        const int64_t bhc = bh * n_chunks + ch;
        const int64_t it0 = static_cast<int64_t>(ch) * kTcQ;

        float xv[kXItems][8];
        load_x(p, bi, h, it0, xv);
        uint4 sv[kStImg / 16 / kTcThreads2];
        if (ch > 0) {
            const uint4* src = reinterpret_cast<const uint4*>(ws.simg + bhc * kStImg);
#pragma unroll
            for (int r = 0; r < static_cast<int>(kStImg / 16 / kTcThreads2); ++r)
                sv[r] = __ldg(src + tid + r * kTcThreads2);
        }
        if (warp == 0) tile_gates(p, bh, it0, lcum, scl, gam, wdec, nullptr);
#pragma unroll
        for (int r = 0; r < kXItems; ++r) {
            int j, pc;
            x_item(r, j, pc);
            *reinterpret_cast<uint4*>(smem + kCX + mnmaj_off(pc * 8, j, kTcP)) = pack8(xv[r]);
        }
        if (ch > 0) {
            uint4* dst = reinterpret_cast<uint4*>(smem + kCS);
#pragma unroll
            for (int r = 0; r < static_cast<int>(kStImg / 16 / kTcThreads2); ++r)
                dst[tid + r * kTcThreads2] = sv[r];
        }
        stage_qk<true>(p, bi, h, it0, smem + kCQ, smem + kCK, p.q_bias + h * kTcN, p.k_bias + h * kTcN);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();

        if (tid == 0) {
            const uint32_t id_G = instr_desc(128, 128, false, false);
#pragma unroll
            for (int kb = 0; kb < kTcN / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kCQ + kb * 2 * 16 * 128, 16 * 128, 128);
                const uint64_t b = smem_desc(sbase + kCK + kb * 2 * 16 * 128, 16 * 128, 128);
                umma(tG, a, b, id_G, kb > 0);
            }
            if (ch > 0) {
                const uint32_t id_Z = instr_desc(128, kTcP, false, true);
#pragma unroll
                for (int kb = 0; kb < kTcN / 16; ++kb) {
                    const uint64_t a = smem_desc(sbase + kCQ + kb * 2 * 16 * 128, 16 * 128, 128);
                    const uint64_t b = smem_desc(sbase + kCS + kb * 2 * 8 * 128, 8 * 128, 128);
                    umma(tZ, a, b, id_Z, kb > 0);
                }
            }
            umma_commit(bar);
        }
        ok = cta_wait(bar, phase);
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        {
            // W = mask o G (row i, columns of this warp's half) over Qr
            const int i = (warp & 3) * 32 + lane;
            const float li = lcum[i], gi = gam[i];
#pragma unroll
            for (int cb = 0; cb < 2; ++cb) {
                float g[32];
                tmem_ld32(tG + t_lane + hc * 64 + cb * 32, g);
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    const int j0 = hc * 64 + cb * 32 + c8 * 8;
                    const float4 la = *reinterpret_cast<const float4*>(lcum + j0);
                    const float4 lb = *reinterpret_cast<const float4*>(lcum + j0 + 4);
                    const float4 sa = *reinterpret_cast<const float4*>(scl + j0);
                    const float4 sb = *reinterpret_cast<const float4*>(scl + j0 + 4);
                    const float lj[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                    const float sj[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
                    float wv[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int j = j0 + c;
                        // lcum is non-increasing, so li - lj <= 0 for j < i
                        const float m = j < i ? ex2_approx(li - lj[c]) * sj[c] : (j == i ? gi : 0.f);
                        wv[c] = m * g[c8 * 8 + c];
                    }
                    *reinterpret_cast<uint4*>(smem + kCQ + kmaj_off(i, j0, 128)) = pack8(wv);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t id_Y = instr_desc(128, kTcP, false, true);
            for (int kb = 0; kb < kTcQ / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kCQ + kb * 2 * 16 * 128, 16 * 128, 128);
                const uint64_t b = smem_desc(sbase + kCX + kb * 2 * 8 * 128, 8 * 128, 128);
                umma(tY, a, b, id_Y, kb > 0);
            }
            umma_commit(bar);
        }
        ok = cta_wait(bar, phase);
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        {
            const int i = (warp & 3) * 32 + lane;
            float y[32];
            tmem_ld32(tY + t_lane + hc * 32, y);
            if (ch > 0) {
                float zt[32];
                tmem_ld32(tZ + t_lane + hc * 32, zt);
                const float el = ex2_approx(lcum[i]);
#pragma unroll
                for (int q = 0; q < 32; ++q) y[q] = fmaf(el, zt[q], y[q]);
            }
            const int64_t it = it0 + i;
            if (it < L) {
                const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
                const int64_t t = p.reverse ? L - 1 - it : it;
                const int64_t voff = ((bi * L + t) * H + h) * kTcP + hc * 32;
                float* o = p.out + (bh * L + t) * kTcP + hc * 32;
                float4 vv[8], zz[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    vv[q] = __ldg(reinterpret_cast<const float4*>(p.v + voff) + q);
                    zz[q] = p.z ? __ldg(reinterpret_cast<const float4*>(p.z + voff) + q)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    float r4[4] = {fmaf(dsk, vv[q].x, y[4 * q]), fmaf(dsk, vv[q].y, y[4 * q + 1]),
                                   fmaf(dsk, vv[q].z, y[4 * q + 2]), fmaf(dsk, vv[q].w, y[4 * q + 3])};
                    if (p.z) {
                        r4[0] *= silu_f(zz[q].x);
                        r4[1] *= silu_f(zz[q].y);
                        r4[2] *= silu_f(zz[q].z);
                        r4[3] *= silu_f(zz[q].w);
                    }
                    *reinterpret_cast<float4*>(o + 4 * q) = make_float4(r4[0], r4[1], r4[2], r4[3]);
                }
            }
        }
        // the next tile overwrites shared memory and tensor memory
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (!ok) mbar_wait(bar, phase ^ 1);  // MMAs still in flight: bounded second wait
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ---------------------------------------------------------------------------
// Fused single-launch variant (default).  Persistent CTAs take tiles from an
// atomic counter in chunk-major order (tile = chunk * batch*heads + bh), so a
// tile's predecessor chunk (same bh) was always taken earlier by a running
// CTA.  Per tile:
//   0. (bf16 inputs, raw angles) the tile's q, k rows are bulk-copied into
//      the Q, K regions; the theta scan (thread per pair and quarter, into a
//      table over the X region) and the gates (four warps) run meanwhile;
//      the rotation reads both from shared memory;
//   1. G = Qr Kr^T and dS^T = Kr^T (w o X) in one MMA group;
//   2. the chain, first because the successor chunk's tile waits for it:
//      wait for the predecessor's outgoing state (flag per bh, acquire),
//      S_out = 2^{l2_last} S_in + dS in fp32, publish it (release) to the
//      bh's other slot, then build the bf16 S_in^T operand;
//   3. W = mask o G over Kr (free once group 1 completed);
//   4. Y = W X and Z = Qr S_in^T in one group;  y = (Y + 2^{l2_i} Z + D x) * silu(z).
// The outgoing states live in two fp32 slots per bh (chunk c reads slot
// (c+1)&1, writes slot c&1): 64 KB per bh, resident in L2, laid out so that a
// warp's accesses are contiguous.
// The wait for a predecessor is bounded (with nanosleep backoff); on expiry
// the tile sets the status flag, and the CTA stops after its MMAs drain.
constexpr uint32_t kFQ = 0;                        // Qr K-major (A of G, Z)
constexpr uint32_t kFK = kFQ + kChunkImg;          // Kr K-major (B of G, A of dS^T); then W
constexpr uint32_t kFX = kFK + kChunkImg;          // X MN-major (B of Y)
constexpr uint32_t kFXw = kFX + 128 * 64 * 2;      // w o X MN-major (B of dS^T)
// S_in^T MN-major (B of Z) reuses w o X: it is written in the chain step,
// after group 1 (the only reader of w o X) has completed
constexpr uint32_t kFS = kFXw;
constexpr uint32_t kFGate = kFXw + 128 * 64 * 2;   // lcum, scale, gamma, w
constexpr uint32_t kFQtot = kFGate + 4 * 128 * 4;  // angles mode: [4 quadrants][64 pairs], theta0[64]
constexpr uint32_t kFBias = kFQtot + 5 * 64 * 4;   // this head's q, k biases: [2][rank <= 4][dqk]
constexpr uint32_t kFMisc = kFBias + 2 * 4 * 128 * 4;
constexpr uint32_t kFSmem = kFMisc + 64;

struct ChainWs {
    float* slots;            // [bh][2][dqk][dv] fp32 outgoing states
    unsigned int* flags;     // [bh] chunks published (zeroed per launch)
    unsigned int* counter;   // tile counter (zeroed per launch)
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// bounded wait until *flag >= want; false on expiry (about a second)
__device__ __forceinline__ bool wait_flag(const unsigned int* flag, unsigned int want) {
    for (uint32_t it = 0; it < (1u << 25); ++it) {
        if (ld_acquire(flag) >= want) return true;
        __nanosleep(32);
    }
    return false;
}

// ---- typed input helpers (fp32 or bf16 rows of 8) ------------------------
__device__ __forceinline__ float bf16_to_f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

template <bool IN16>
__device__ __forceinline__ void ld8_in(const void* base, int64_t idx, float (&f)[8]) {
    if (IN16) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            f[2 * e] = bf16_to_f(w[e] & 0xFFFFu);
            f[2 * e + 1] = bf16_to_f(w[e] >> 16);
        }
    } else {
        ldg8(static_cast<const float*>(base) + idx, f);
    }
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = bf16_to_f(w[e] & 0xFFFFu);
        f[2 * e + 1] = bf16_to_f(w[e] >> 16);
    }
}
__device__ __forceinline__ uint4 ld8_raw16(const void* base, int64_t idx) {
    return __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx));
}

template <bool IN16>
__device__ __forceinline__ float ld1_in(const void* base, int64_t idx) {
    if (IN16) return bf16_to_f(__ldg(static_cast<const uint16_t*>(base) + idx));
    return __ldg(static_cast<const float*>(base) + idx);
}

template <bool IN16>
__device__ __forceinline__ void load_x_t(const M3Params& p, int64_t bi, int64_t h, int64_t it0,
                                         float (&xv)[kXItems][8]) {
    const int64_t L = p.len, H = p.heads;
#pragma unroll
    for (int r = 0; r < kXItems; ++r) {
        int j, pc;
        x_item(r, j, pc);
        const int64_t it = it0 + j;
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[r][e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            ld8_in<IN16>(p.v, ((bi * L + t) * H + h) * kTcP + pc * 8, xv[r]);
        }
    }
}

// ---- angle pre-pass (angles mode) ----------------------------------------
// Natural-time range [lo, hi) of traversal chunk c.
__device__ __forceinline__ void chunk_range(int64_t L, int c, int reverse, int64_t& lo, int64_t& hi) {
    if (!reverse) {
        lo = static_cast<int64_t>(c) * kTcQ;
        hi = lo + kTcQ < L ? lo + kTcQ : L;
    } else {
        hi = L - static_cast<int64_t>(c) * kTcQ;
        lo = hi - kTcQ > 0 ? hi - kTcQ : 0;
    }
}

// Per (traversal chunk, bh, pair): sum of tanh(angle) * pi * dt over the
// chunk's steps -> theta0[bh][c][pair]; also the table ta = tanh(angle) * pi
// (written once per angle row: by head 0 when angles are shared).  256
// threads: pair = tid % 64, quarter = tid / 64 takes 32 of the 128 steps.
template <bool IN16>
__global__ void __launch_bounds__(256) m3_tc_angle_sums(M3Params p, float* ta, float* theta0,
                                                       int n_chunks) {
    __shared__ float part[4][64];
    const int c = blockIdx.x;
    const int64_t bh = blockIdx.y;
    const int pr = threadIdx.x & 63, qr = threadIdx.x >> 6;
    const int64_t H = p.heads, L = p.len, NA = p.n_angles;
    const int64_t bi = bh / H, h = bh % H;
    int64_t lo, hi;
    chunk_range(L, c, p.reverse, lo, hi);
    const int64_t qlo = lo + 32 * qr < hi ? lo + 32 * qr : hi;
    const int64_t qhi = qlo + 32 < hi ? qlo + 32 : hi;
    const bool writer = !p.angles_shared || h == 0;
    const float* dt = p.dt + bh * L;
    constexpr float kPiF = 3.14159265358979323846f;
    // element (step t, pair pr) of the angle rows and of the ta table
    const int64_t step = p.angles_shared ? NA : H * NA;
    const int64_t base = (p.angles_shared ? bi * L * NA : (bi * L * H + h) * NA) + pr;
    float s = 0.f;
    if (pr < NA) {
        for (int64_t t = qlo; t < qhi; t += 8) {
            float a[8], d[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const bool in = t + u < qhi;
                a[u] = in ? ld1_in<IN16>(p.angles, base + (t + u) * step) : 0.f;
                d[u] = in ? __ldg(dt + t + u) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (t + u >= qhi) break;
                // tanh x = 1 - 2 / (1 + e^{2x}): absolute error <= ~2.5e-7
                const float tv = (1.f - __fdividef(2.f, 1.f + __expf(2.f * a[u]))) * kPiF;
                s = fmaf(tv, d[u], s);
                if (writer) ta[base + (t + u) * step] = tv;
            }
        }
    }
    part[qr][pr] = s;
    __syncthreads();
    if (qr == 0 && pr < NA)
        theta0[(bh * n_chunks + c) * 64 + pr] = ((part[0][pr] + part[1][pr]) + part[2][pr]) + part[3][pr];
}

// Shared angles (one row per (batch, step) for every head): one CTA per
// (traversal chunk, batch) computes the chunk's ta rows once (tanh, written
// to the table) and every head's chunk sums theta0[bh][c][pair] =
// sum over the chunk's steps of ta * dt_h, from shared memory: ta as
// [128 steps][64 pairs], dt as [heads][128 steps].
template <bool IN16>
__global__ void __launch_bounds__(256) m3_tc_angle_sums_shared(M3Params p, float* ta, float* theta0,
                                                              int n_chunks) {
    extern __shared__ float ang_sm[];
    float* tas = ang_sm;             // [128][64]
    float* dts = ang_sm + kTcQ * 64;  // [heads][128]
    constexpr float kPiF = 3.14159265358979323846f;
    const int c = blockIdx.x;
    const int64_t bi = blockIdx.y;
    const int64_t H = p.heads, L = p.len, NA = p.n_angles;
    int64_t lo, hi;
    chunk_range(L, c, p.reverse, lo, hi);
    const int n = static_cast<int>(hi - lo);
    for (int i = threadIdx.x; i < kTcQ * 64; i += blockDim.x) {
        const int st = i >> 6, pr = i & 63;
        float tv = 0.f;
        if (st < n && pr < NA) {
            const int64_t e = (bi * L + lo + st) * NA + pr;
            // tanh x = 1 - 2 / (1 + e^{2x}): absolute error <= ~2.5e-7
            tv = (1.f - __fdividef(2.f, 1.f + __expf(2.f * ld1_in<IN16>(p.angles, e)))) * kPiF;
            ta[e] = tv;
        }
        tas[i] = tv;
    }
    for (int i = threadIdx.x; i < H * kTcQ; i += blockDim.x) {
        const int64_t hh = i / kTcQ;
        const int st = i % kTcQ;
        dts[i] = st < n ? __ldg(p.dt + (bi * H + hh) * L + lo + st) : 0.f;
    }
    __syncthreads();
    const int pr = threadIdx.x & 63, hg = threadIdx.x >> 6;
    constexpr int kHk = 6;  // heads per thread and pass: hg + 4 k
    for (int64_t h0 = hg; h0 < H; h0 += 4 * kHk) {
        // per quarter of 32 steps, then ((q0 + q1) + q2) + q3: the order of
        // m3_tc_angle_sums, so shared and per-head angles agree bit for bit
        float acc[kHk];
#pragma unroll
        for (int k = 0; k < kHk; ++k) acc[k] = 0.f;
        for (int qr = 0; qr < 4; ++qr) {
            float part[kHk];
#pragma unroll
            for (int k = 0; k < kHk; ++k) part[k] = 0.f;
            const int se = 32 * qr + 32 < n ? 32 * qr + 32 : n;
            for (int st = 32 * qr; st < se; ++st) {
                const float tv = tas[st * 64 + pr];
#pragma unroll
                for (int k = 0; k < kHk; ++k) {
                    const int64_t hh = h0 + 4 * k;
                    if (hh < H) part[k] = fmaf(tv, dts[hh * kTcQ + st], part[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < kHk; ++k) acc[k] = qr == 0 ? part[k] : acc[k] + part[k];
        }
#pragma unroll
        for (int k = 0; k < kHk; ++k) {
            const int64_t hh = h0 + 4 * k;
            if (hh < H && pr < NA) theta0[((bi * H + hh) * n_chunks + c) * 64 + pr] = acc[k];
        }
    }
}

// ---- rank generalization: a tile holds 128 rows = (128 / R) steps x R ranks,
// row i = step (i / R), rank (i % R).  R = 1 is SISO.

// Gates of one tile's steps (warp 0), replicated into the R rows of each
// step: cumulative log2 decay, trapezoid scale, gamma, state weight.
template <int R>
__device__ __forceinline__ void tile_gates_r(const M3Params& p, int64_t bh, int64_t s0, float* lcum,
                                             float* scl, float* gam, float* wdec, float* decay) {
    constexpr float kLog2eF = 1.4426950408889634f;
    constexpr int SPL = kTcQ / R / 32;  // steps per lane
    const int lane = threadIdx.x & 31;
    const int64_t L = p.len, gate_base = bh * L;
    float lv[SPL], sc[SPL], gm[SPL];
#pragma unroll
    for (int e = 0; e < SPL; ++e) {
        const int64_t it = s0 + lane * SPL + e;
        lv[e] = sc[e] = gm[e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t g = gate_base + t;
            const float gamma = __ldg(p.dt + g) * sigmoid_f(__ldg(p.trap + g));
            float shifted = 0.f;
            if (it + 1 < L) {
                const int64_t nx = p.reverse ? g - 1 : g + 1;
                shifted = __ldg(p.dt + nx) * (1.f - sigmoid_f(__ldg(p.trap + nx)));
            }
            lv[e] = __ldg(p.adt + g) * kLog2eF;
            sc[e] = gamma + shifted;
            gm[e] = gamma;
        }
    }
#pragma unroll
    for (int e = 1; e < SPL; ++e) lv[e] += lv[e - 1];
    float run = lv[SPL - 1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += v;
    }
    const float before = run - lv[SPL - 1];
    const float last = __shfl_sync(0xffffffffu, run, 31);
#pragma unroll
    for (int e = 0; e < SPL; ++e) {
        const float l = before + lv[e];
        const float w = ex2_approx(last - l) * sc[e];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            const int row = (lane * SPL + e) * R + rr;
            lcum[row] = l;
            scl[row] = sc[e];
            gam[row] = gm[e];
            wdec[row] = w;
        }
    }
    if (decay && lane == 0) *decay = ex2_approx(last);
}

// SISO gates over four warps (angles mode): thread j = tid < 128 takes step
// j of the tile.  Part 1 (before the stage barrier): trapezoid scale,
// gamma, and the warp-local inclusive prefix of the log2 decay into lcum,
// the warp's total into wtot.  Part 2 (after it, same threads): add the
// totals of the warps before, then the state weight and the chunk's decay.
__device__ __forceinline__ void gates_split_1(const M3Params& p, int64_t bh, int64_t it0, float* lcum,
                                              float* scl, float* gam, float* wtot) {
    constexpr float kLog2eF = 1.4426950408889634f;
    const int j = threadIdx.x, lane = j & 31;
    const int64_t L = p.len, gate_base = bh * L;
    const int64_t it = it0 + j;
    float lv = 0.f, sc = 0.f, gm = 0.f;
    if (it < L) {
        const int64_t t = p.reverse ? L - 1 - it : it;
        const int64_t g = gate_base + t;
        const bool more = it + 1 < L;
        const int64_t nx = more ? (p.reverse ? g - 1 : g + 1) : g;
        const float dtg = __ldg(p.dt + g), trg = __ldg(p.trap + g);
        const float dtn = __ldg(p.dt + nx), trn = __ldg(p.trap + nx);
        const float adt = __ldg(p.adt + g);
        const float gamma = dtg * sigmoid_f(trg);
        const float shifted = more ? dtn * (1.f - sigmoid_f(trn)) : 0.f;
        lv = adt * kLog2eF;
        sc = gamma + shifted;
        gm = gamma;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, lv, o);
        if (lane >= o) lv += v;
    }
    lcum[j] = lv;
    scl[j] = sc;
    gam[j] = gm;
    if (lane == 31) wtot[j >> 5] = lv;
}
__device__ __forceinline__ void gates_split_2(float* lcum, const float* scl, float* wdec,
                                              const float* wtot, float* decay) {
    const int j = threadIdx.x, w = j >> 5;
    float before = 0.f, last = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float v = wtot[q];
        before += q < w ? v : 0.f;
        last += v;
    }
    const float l = lcum[j] + before;
    lcum[j] = l;
    wdec[j] = ex2_approx(last - l) * scl[j];
    if (j == 0) *decay = ex2_approx(last);
}

// X rows (fp32 inputs): SISO x = v; MIMO x_r = psi_r o v.
template <int R>
__device__ __forceinline__ void load_x_r(const M3Params& p, int64_t bi, int64_t h, int64_t s0,
                                         float (&xv)[kXItems][8]) {
    const int64_t L = p.len, H = p.heads;
#pragma unroll
    for (int q = 0; q < kXItems; ++q) {
        int j, pc;
        x_item(q, j, pc);
        const int64_t it = s0 + j / R;
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[q][e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            ldg8(p.v + ((bi * L + t) * H + h) * kTcP + pc * 8, xv[q]);
            if (R > 1) {
                float ps[8];
                ldg8(p.psi + (h * R + j % R) * kTcP + pc * 8, ps);
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[q][e] *= ps[e];
            }
        }
    }
}

// Per-rank MIMO (p.x_per_rank): X rows of the tile, row j = (step j / R,
// rank j % R), channels 8pc..8pc+7 of X (b, l, h, dv, R), i.e. stride R.
template <int R, bool IN16>
__device__ __forceinline__ void load_x_xr(const M3Params& p, int64_t bi, int64_t h, int64_t s0,
                                          float (&xv)[kXItems][8]) {
    const int64_t L = p.len, H = p.heads;
#pragma unroll
    for (int q = 0; q < kXItems; ++q) {
        int j, pc;
        x_item(q, j, pc);
        const int64_t it = s0 + j / R;
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[q][e] = 0.f;
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t base = (((bi * L + t) * H + h) * kTcP + pc * 8) * R + j % R;
#pragma unroll
            for (int e = 0; e < 8; ++e) xv[q][e] = ld1_in<IN16>(p.v, base + e * R);
        }
    }
}

// bf16 per-rank MIMO, 16-byte loads: a tile's X is TS = 128 / R steps of
// dv x R contiguous elements; item (step s, 16-byte chunk i) holds channels
// i*8/R .. +8/R-1 of every rank.  4 items per thread (1024 chunks).
template <int R>
__device__ __forceinline__ void load_x_xr16_raw(const M3Params& p, int64_t bi, int64_t h, int64_t s0,
                                                uint4 (&raw)[4]) {
    const int64_t L = p.len, H = p.heads;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int item = threadIdx.x + m * kTcThreads2;
        const int st = item / (8 * R), ci = item % (8 * R);
        const int64_t it = s0 + st;
        raw[m] = make_uint4(0u, 0u, 0u, 0u);
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            raw[m] = ld8_raw16(p.v, ((bi * L + t) * H + h) * kTcP * R + ci * 8);
        }
    }
}
// The X and w o X operand images (MN-major, m = channel, k = row (step, rank))
// from those chunks: each rank's 8/R adjacent channels go in one store.
template <int R>
__device__ __forceinline__ void store_x_xr16(const uint4 (&raw)[4], const float* wdec, uint8_t* img_x,
                                             uint8_t* img_xw) {
    constexpr int CPI = 8 / R;  // channels per item
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int item = threadIdx.x + m * kTcThreads2;
        const int st = item / (8 * R), ci = item % (8 * R);
        float v[8];
        unpack8(raw[m], v);
#pragma unroll
        for (int rk = 0; rk < R; ++rk) {
            const int j = st * R + rk;
            const float w = wdec[j];
            const uint32_t o = mnmaj_off(ci * CPI, j, kTcP);
            if (CPI == 2) {
                *reinterpret_cast<uint32_t*>(img_x + o) = pack_bf16x2(v[rk], v[R + rk]);
                *reinterpret_cast<uint32_t*>(img_xw + o) = pack_bf16x2(w * v[rk], w * v[R + rk]);
            } else {
                *reinterpret_cast<uint2*>(img_x + o) =
                    make_uint2(pack_bf16x2(v[rk], v[R + rk]), pack_bf16x2(v[2 * R + rk], v[3 * R + rk]));
                *reinterpret_cast<uint2*>(img_xw + o) = make_uint2(
                    pack_bf16x2(w * v[rk], w * v[R + rk]), pack_bf16x2(w * v[2 * R + rk], w * v[3 * R + rk]));
            }
        }
    }
}

// bf16 per-rank MIMO C (q) and B (k) with 16-byte loads: item (step s, low
// chunk i) covers dims i*8/R .. +8/R-1 of every rank and their split-halves
// partners 64 dims up; rotated, bias-added, stored 8/R dims per row at once.
template <int R>
__device__ __forceinline__ void stage_qk_xr16(const M3Params& p, int64_t bi, int64_t h, int64_t s0,
                                              uint8_t* img_q, uint8_t* img_k, const float* qbs,
                                              const float* kbs) {
    const int64_t L = p.len, H = p.heads;
    constexpr int half = kTcN / 2, CPI = 8 / R;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int item = threadIdx.x + m * kTcThreads2;
        const int st = item / (8 * R), ci = item % (8 * R);
        const int n0 = ci * CPI;
        const int64_t it = s0 + st;
        float ql[8], qh[8], kl[8], kh[8], c[CPI], sn[CPI];
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t base = (bi * L + t) * kTcN * R + ci * 8;
            unpack8(ld8_raw16(p.q, base), ql);
            unpack8(ld8_raw16(p.q, base + half * R), qh);
            unpack8(ld8_raw16(p.k, base), kl);
            unpack8(ld8_raw16(p.k, base + half * R), kh);
            const int64_t cs = ((bi * L + t) * H + h) * half + n0;
#pragma unroll
            for (int e = 0; e < CPI; ++e) {
                c[e] = __ldg(p.cos + cs + e);
                sn[e] = __ldg(p.sin + cs + e);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) ql[e] = qh[e] = kl[e] = kh[e] = 0.f;
#pragma unroll
            for (int e = 0; e < CPI; ++e) c[e] = 1.f, sn[e] = 0.f;
        }
#pragma unroll
        for (int rk = 0; rk < R; ++rk) {
            const int j = st * R + rk;
            float qlo[CPI], qhi[CPI], klo[CPI], khi[CPI];
#pragma unroll
            for (int e = 0; e < CPI; ++e) {
                const int bb = rk * kTcN + n0 + e;
                float a0 = ql[e * R + rk] + qbs[bb], a1 = qh[e * R + rk] + qbs[bb + half];
                qlo[e] = a0 * c[e] - a1 * sn[e];
                qhi[e] = a0 * sn[e] + a1 * c[e];
                a0 = kl[e * R + rk] + kbs[bb];
                a1 = kh[e * R + rk] + kbs[bb + half];
                klo[e] = a0 * c[e] - a1 * sn[e];
                khi[e] = a0 * sn[e] + a1 * c[e];
            }
            const uint32_t ol = kmaj_off(j, n0, 128), oh = kmaj_off(j, n0 + half, 128);
            if (CPI == 2) {
                *reinterpret_cast<uint32_t*>(img_q + ol) = pack_bf16x2(qlo[0], qlo[CPI - 1]);
                *reinterpret_cast<uint32_t*>(img_q + oh) = pack_bf16x2(qhi[0], qhi[CPI - 1]);
                *reinterpret_cast<uint32_t*>(img_k + ol) = pack_bf16x2(klo[0], klo[CPI - 1]);
                *reinterpret_cast<uint32_t*>(img_k + oh) = pack_bf16x2(khi[0], khi[CPI - 1]);
            } else {
                *reinterpret_cast<uint2*>(img_q + ol) =
                    make_uint2(pack_bf16x2(qlo[0], qlo[1 % CPI]), pack_bf16x2(qlo[2 % CPI], qlo[3 % CPI]));
                *reinterpret_cast<uint2*>(img_q + oh) =
                    make_uint2(pack_bf16x2(qhi[0], qhi[1 % CPI]), pack_bf16x2(qhi[2 % CPI], qhi[3 % CPI]));
                *reinterpret_cast<uint2*>(img_k + ol) =
                    make_uint2(pack_bf16x2(klo[0], klo[1 % CPI]), pack_bf16x2(klo[2 % CPI], klo[3 % CPI]));
                *reinterpret_cast<uint2*>(img_k + oh) =
                    make_uint2(pack_bf16x2(khi[0], khi[1 % CPI]), pack_bf16x2(khi[2 % CPI], khi[3 % CPI]));
            }
        }
    }
}

// Per-rank MIMO rotated C (q) and B (k) rows: element (rank rk, dim n) of
// step t at ((b * L + t) * dqk + n) * R + rk; biases may be absent; same
// split-halves RoPE and item split as stage_qk_mimo.
template <int R, bool IN16>
__device__ __forceinline__ void stage_qk_xr(const M3Params& p, int64_t bi, int64_t h, int64_t s0,
                                            uint8_t* img_q, uint8_t* img_k, const float* qbs,
                                            const float* kbs) {
    const int64_t L = p.len, H = p.heads;
    constexpr int half = kTcN / 2;
#pragma unroll
    for (int m = 0; m < 128 * 8 / kTcThreads2; ++m) {
        const int item = threadIdx.x + m * kTcThreads2;
        const int j = (item >> 8) * 32 + (item & 31);
        const int kc = (item >> 5) & 7;
        const int rk = j % R;
        const int64_t it = s0 + j / R;
        float qlo[8], qhi[8], klo[8], khi[8];
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t base = ((bi * L + t) * kTcN + kc * 8) * R + rk;
            const int bb = rk * kTcN + kc * 8;
            const int64_t cs = ((bi * L + t) * H + h) * half + kc * 8;
            float c[8], sn[8];
            ldg8(p.cos + cs, c);
            ldg8(p.sin + cs, sn);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float a0 = ld1_in<IN16>(p.q, base + e * R) + qbs[bb + e];
                float a1 = ld1_in<IN16>(p.q, base + (half + e) * R) + qbs[bb + half + e];
                qlo[e] = a0 * c[e] - a1 * sn[e];
                qhi[e] = a0 * sn[e] + a1 * c[e];
                a0 = ld1_in<IN16>(p.k, base + e * R) + kbs[bb + e];
                a1 = ld1_in<IN16>(p.k, base + (half + e) * R) + kbs[bb + half + e];
                klo[e] = a0 * c[e] - a1 * sn[e];
                khi[e] = a0 * sn[e] + a1 * c[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) qlo[e] = qhi[e] = klo[e] = khi[e] = 0.f;
        }
        *reinterpret_cast<uint4*>(img_q + kmaj_off(j, kc * 8, 128)) = pack8(qlo);
        *reinterpret_cast<uint4*>(img_q + kmaj_off(j, kc * 8 + half, 128)) = pack8(qhi);
        *reinterpret_cast<uint4*>(img_k + kmaj_off(j, kc * 8, 128)) = pack8(klo);
        *reinterpret_cast<uint4*>(img_k + kmaj_off(j, kc * 8 + half, 128)) = pack8(khi);
    }
}

// MIMO rotated q, k rows from cos/sin, split-halves RoPE: pair m rotates
// dims (m, m + dqk/2).  One item = row j (step, rank) x low dim chunk kc
// (dims 8kc..8kc+7) and its partner chunk kc + 8; 1024 items, 4 per thread.
template <int R>
__device__ __forceinline__ void stage_qk_mimo(const M3Params& p, int64_t bi, int64_t h,
                                              int64_t s0, uint8_t* img_q, uint8_t* img_k,
                                              const float* qbs, const float* kbs) {
    const int64_t L = p.len, H = p.heads;
    constexpr int half = kTcN / 2;
#pragma unroll
    for (int m = 0; m < 128 * 8 / kTcThreads2; ++m) {
        const int item = threadIdx.x + m * kTcThreads2;
        const int j = (item >> 8) * 32 + (item & 31);   // a warp covers 32 rows of one chunk
        const int kc = (item >> 5) & 7;
        const int rk = j % R;
        const int64_t it = s0 + j / R;
        float qlo[8], qhi[8], klo[8], khi[8];
        if (it < L) {
            const int64_t t = p.reverse ? L - 1 - it : it;
            const int64_t qk = ((bi * L + t) * R + rk) * kTcN + kc * 8;
            const int bb = rk * kTcN + kc * 8;  // this head's bias block [R][dqk]
            const int64_t cs = ((bi * L + t) * H + h) * half + kc * 8;
            float bq0[8], bq1[8], bk0[8], bk1[8], c[8], s[8];
            ldg8(p.q + qk, qlo);
            ldg8(p.q + qk + half, qhi);
            ldg8(p.k + qk, klo);
            ldg8(p.k + qk + half, khi);
            ld8(qbs + bb, bq0);
            ld8(qbs + bb + half, bq1);
            ld8(kbs + bb, bk0);
            ld8(kbs + bb + half, bk1);
            ldg8(p.cos + cs, c);
            ldg8(p.sin + cs, s);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float a0 = qlo[e] + bq0[e], a1 = qhi[e] + bq1[e];
                qlo[e] = a0 * c[e] - a1 * s[e];
                qhi[e] = a0 * s[e] + a1 * c[e];
                a0 = klo[e] + bk0[e];
                a1 = khi[e] + bk1[e];
                klo[e] = a0 * c[e] - a1 * s[e];
                khi[e] = a0 * s[e] + a1 * c[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) qlo[e] = qhi[e] = klo[e] = khi[e] = 0.f;
        }
        *reinterpret_cast<uint4*>(img_q + kmaj_off(j, kc * 8, 128)) = pack8(qlo);
        *reinterpret_cast<uint4*>(img_q + kmaj_off(j, kc * 8 + half, 128)) = pack8(qhi);
        *reinterpret_cast<uint4*>(img_k + kmaj_off(j, kc * 8, 128)) = pack8(klo);
        *reinterpret_cast<uint4*>(img_k + kmaj_off(j, kc * 8 + half, 128)) = pack8(khi);
    }
}

// Rotated q, k rows of one chunk from raw angles, in two parts around the
// gate pass's barrier.  theta(step, pair) = theta0(chunk) + prefix over the
// chunk's steps, in natural time order, of ta * dt.
//
// Part A (before the barrier): thread = (pair pr = tid % 64, quarter qd =
// tid / 64 of the tile's 128 rows); it walks its 32 rows in natural time
// order, accumulating ta * dt (lanes = consecutive pairs, so every load is
// one coalesced row segment and dt a broadcast), and writes the running sum
// into a [128 rows][64 pairs] fp32 table in shared memory (16-byte chunk c
// of row j stored at chunk c ^ (j % 16), so that both the row-wise writes
// here and the per-row 16-byte reads of part B are free of bank conflicts).
// The quarter's total goes to qtot, the chunk's theta0 row to th0s.
template <bool SWZ>
__device__ __forceinline__ uint32_t ang_tab_idx(int j, int pr) {
    return SWZ ? static_cast<uint32_t>(j * 64 + ((((pr >> 2) ^ (j & 15)) << 2) | (pr & 3)))
               : static_cast<uint32_t>(j * 64 + pr);
}
template <bool SWZ>
__device__ __forceinline__ void ang_part_a(const M3Params& p, const float* ta, const float* theta0,
                                           int64_t bi, int64_t h, int64_t bh, int ch,
                                           int n_chunks, float* tab, float* qtot, float* th0s) {
    const int tid = threadIdx.x, pr = tid & 63, qd = tid >> 6;
    const int64_t L = p.len, H = p.heads, NA = p.n_angles;
    const bool rev = p.reverse != 0;
    int64_t lo, hi;
    chunk_range(L, ch, p.reverse, lo, hi);
    const int n = static_cast<int>(hi - lo);  // valid rows of the tile
    if (tid >= 128 && tid < 192) {  // warps 4, 5: no gate work in this stage
        const int pt = tid - 128;
        // theta0 of the chunk: the chunk sums of the chunks before it in
        // natural time (traversal chunks 0..ch-1, or ch+1..n_chunks-1 in
        // reverse), summed in natural time order
        float acc = 0.f;
        if (pt < NA) {
            const float* col = theta0 + bh * n_chunks * 64 + pt;
            const int cnt = rev ? n_chunks - 1 - ch : ch;
            for (int i0 = 0; i0 < cnt; i0 += 8) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int i = i0 + u;
                    v[u] = i < cnt ? __ldg(col + (rev ? n_chunks - 1 - i : i) * 64) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) acc += v[u];
            }
        }
        th0s[pt] = acc;
    }
    // rows of this quarter in natural time order: forward j = 32 qd + u,
    // reverse j = 32 qd + 31 - u; natural time t(j) = lo + j / hi - 1 - j
    const int jbase = rev ? qd * 32 + 31 : qd * 32;
    const int jstep = rev ? -1 : 1;
    const int64_t t0 = rev ? hi - 1 - jbase : lo + jbase;  // natural time of u = 0
    const int64_t astep = p.angles_shared ? NA : H * NA;
    const bool act = pr < NA;
    const float* tp = ta + (p.angles_shared ? (bi * L + t0) * NA : ((bi * L + t0) * H + h) * NA) + pr;
    // dt of the quarter's rows: lane u holds row u's, shuffled to the pairs
    const int lane = tid & 31;
    const float dtl = (jbase + jstep * lane < n) ? __ldg(p.dt + bh * L + t0 + lane) : 0.f;
    float a[32];
#pragma unroll
    for (int u = 0; u < 32; ++u) {
        const bool in = jbase + jstep * u < n;
        a[u] = (in && act) ? __ldg(tp + u * astep) : 0.f;
    }
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < 32; ++u) {
        acc = fmaf(a[u], __shfl_sync(0xffffffffu, dtl, u), acc);
        tab[ang_tab_idx<SWZ>(jbase + jstep * u, pr)] = acc;
    }
    qtot[qd * 64 + pr] = acc;
}

// Part B (after the barrier): the tile's 128 rows x 16 dim chunks (8 dims,
// 4 rotation pairs each) as 8 items per thread: row j = 32 (warp & 3) +
// lane, chunk kc = 2 m + (warp >> 2) for item m (the warp pair (w, w + 4)
// shares every 32-byte sector of a row).  (A mapping with 8 rows x 4 chunks
// per warp load, fewer sectors per request, measured 13% slower.)  Per
// item: theta from the table plus theta0 and the totals of the quarters
// before, q, k loads (all eight items in flight at once for bf16 inputs),
// rotation, bf16 operand images, and the fp32 carry k.
template <bool IN16>
__device__ __forceinline__ void ang_part_b(const M3Params& p, int64_t bi, int64_t h, int64_t bh,
                                           int64_t it0, const float* tab, const float* qtot,
                                           const float* th0s, uint8_t* img_q, uint8_t* img_k,
                                           const float* scl, const float* qb, const float* kb) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t L = p.len, NA = p.n_angles;
    const bool rev = p.reverse != 0;
    auto item = [&](int m, int& j, int& kc) {
        j = (warp & 3) * 32 + lane;
        kc = 2 * m + (warp >> 2);
    };
    constexpr int kPer = IN16 ? 8 : 2;  // items per round trip
#pragma unroll
    for (int m0 = 0; m0 < 8; m0 += kPer) {
        uint4 qraw[kPer], kraw[kPer];
        float qa[kPer][8], ka[kPer][8];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            int j, kc;
            item(m0 + u, j, kc);
            const int64_t it = it0 + j;
            const bool live = it < L;
            const int64_t t = live ? (rev ? L - 1 - it : it) : 0;
            const int64_t qrow = (bi * L + t) * kTcN;
            if (IN16) {
                qraw[u] = live ? ld8_raw16(p.q, qrow + kc * 8) : make_uint4(0u, 0u, 0u, 0u);
                kraw[u] = live ? ld8_raw16(p.k, qrow + kc * 8) : make_uint4(0u, 0u, 0u, 0u);
            } else if (live) {
                ld8_in<false>(p.q, qrow + kc * 8, qa[u]);
                ld8_in<false>(p.k, qrow + kc * 8, ka[u]);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) qa[u][e] = ka[u][e] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            if (IN16) {
                unpack8(qraw[u], qa[u]);
                unpack8(kraw[u], ka[u]);
            }
            int j, kc;
            item(m0 + u, j, kc);
            const int64_t it = it0 + j;
            const bool live = it < L;
            const int qd = j >> 5;  // quarter of the row (uniform over the warp)
            float4 t4 = *reinterpret_cast<const float4*>(th0s + 4 * kc);
            for (int q = 0; q < 4; ++q) {
                if (rev ? q > qd : q < qd) {
                    const float4 v = *reinterpret_cast<const float4*>(qtot + q * 64 + 4 * kc);
                    t4.x += v.x; t4.y += v.y; t4.z += v.z; t4.w += v.w;
                }
            }
            {
                const float4 v = *reinterpret_cast<const float4*>(tab + ang_tab_idx<true>(j, 4 * kc));
                t4.x += v.x; t4.y += v.y; t4.z += v.z; t4.w += v.w;
            }
            const float th[4] = {t4.x, t4.y, t4.z, t4.w};
            float qbb[8], kbb[8], qr[8], kr[8];
            ld8(qb + kc * 8, qbb);
            ld8(kb + kc * 8, kbb);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float sn = 0.f, cs = 1.f;
                if (4 * kc + e < NA) __sincosf(th[e], &sn, &cs);
                float a0 = qa[u][2 * e] + qbb[2 * e], a1 = qa[u][2 * e + 1] + qbb[2 * e + 1];
                qr[2 * e] = a0 * cs - a1 * sn;
                qr[2 * e + 1] = a0 * sn + a1 * cs;
                a0 = ka[u][2 * e] + kbb[2 * e];
                a1 = ka[u][2 * e + 1] + kbb[2 * e + 1];
                kr[2 * e] = a0 * cs - a1 * sn;
                kr[2 * e + 1] = a0 * sn + a1 * cs;
            }
            if (!live) {
#pragma unroll
                for (int e = 0; e < 8; ++e) qr[e] = kr[e] = 0.f;
            }
            if (p.last_bx && live && it == L - 1) {
                // scale_T * k_T for the carry: rotated k of the final step, fp32
#pragma unroll
                for (int e = 0; e < 8; ++e) p.last_bx[bh * kTcN + kc * 8 + e] = scl[j] * kr[e];
            }
            const uint32_t ko = kmaj_off(j, kc * 8, 128);
            *reinterpret_cast<uint4*>(img_q + ko) = pack8(qr);
            *reinterpret_cast<uint4*>(img_k + ko) = pack8(kr);
        }
    }
}

// Part B for bf16 inputs, from raw q, k rows staged in shared memory.  The
// tile's q and k rows ([n rows][dqk] bf16, natural time order, 256 bytes a
// row) arrive by two bulk copies issued at the start of the tile into the
// Q and K operand regions (still free then).  Item mapping: a thread keeps
// one dim chunk kc (8 dims, 4 rotation pairs; its q, k biases stay in
// registers) and takes 8 rows j = 8 (2 m + s) + (lane & 7); with
// kc = 8 hh + ((lane + c) & 7), the 8 lanes of a shared-memory phase see 8
// different row residues and chunk residues, so the raw-row and theta-table
// reads and the K-major image stores (bank group = j mod 8) are free of
// conflicts.  Rotated rows stay packed in registers until every thread has
// read its raw rows (the caller's barrier); store_qk_img then writes the
// operand images over them.  qoff holds each quarter's theta offset (theta0
// plus the quarters before it in natural time).
__device__ __forceinline__ void qk16_item(int m, int& j, int& kc) {
    const int lane = threadIdx.x & 31, idx = (threadIdx.x >> 5) * 4 + (lane >> 3);
    const int hh = idx & 1, c = (idx >> 1) & 7, sg = idx >> 4;
    j = 8 * (2 * m + sg) + (lane & 7);
    kc = 8 * hh + ((lane + c) & 7);
}
__device__ __forceinline__ void ang_part_b16(const M3Params& p, int64_t bh, int64_t it0, int n,
                                             const float* tab, const float* qoff,
                                             const uint8_t* raw_q, const uint8_t* raw_k,
                                             const float* scl, const float* qb, const float* kb,
                                             uint4 (&qi)[8], uint4 (&ki)[8]) {
    const int64_t L = p.len, NA = p.n_angles;
    const bool rev = p.reverse != 0;
    int j0, kc;
    qk16_item(0, j0, kc);
    float qbb[8], kbb[8];
    ld8(qb + kc * 8, qbb);
    ld8(kb + kc * 8, kbb);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int j = j0 + 16 * m;
        const int64_t it = it0 + j;
        const bool live = it < L;
        const int rr = live ? (rev ? n - 1 - j : j) : 0;  // raw row (natural time) of row j
        float qa[8], ka[8];
        unpack8(*reinterpret_cast<const uint4*>(raw_q + rr * 256 + kc * 16), qa);
        unpack8(*reinterpret_cast<const uint4*>(raw_k + rr * 256 + kc * 16), ka);
        float4 t4 = *reinterpret_cast<const float4*>(qoff + (j >> 5) * 64 + 4 * kc);
        {
            const float4 v = *reinterpret_cast<const float4*>(tab + ang_tab_idx<false>(j, 4 * kc));
            t4.x += v.x; t4.y += v.y; t4.z += v.z; t4.w += v.w;
        }
        const float th[4] = {t4.x, t4.y, t4.z, t4.w};
        float qr[8], kr[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float sn = 0.f, cs = 1.f;
            if (4 * kc + e < NA) __sincosf(th[e], &sn, &cs);
            float a0 = qa[2 * e] + qbb[2 * e], a1 = qa[2 * e + 1] + qbb[2 * e + 1];
            qr[2 * e] = a0 * cs - a1 * sn;
            qr[2 * e + 1] = a0 * sn + a1 * cs;
            a0 = ka[2 * e] + kbb[2 * e];
            a1 = ka[2 * e + 1] + kbb[2 * e + 1];
            kr[2 * e] = a0 * cs - a1 * sn;
            kr[2 * e + 1] = a0 * sn + a1 * cs;
        }
        if (!live) {
#pragma unroll
            for (int e = 0; e < 8; ++e) qr[e] = kr[e] = 0.f;
        }
        if (p.last_bx && live && it == L - 1) {
            // scale_T * k_T for the carry: rotated k of the final step, fp32
#pragma unroll
            for (int e = 0; e < 8; ++e) p.last_bx[bh * kTcN + kc * 8 + e] = scl[j] * kr[e];
        }
        qi[m] = pack8(qr);
        ki[m] = pack8(kr);
    }
}
__device__ __forceinline__ void store_qk_img(const uint4 (&qi)[8], const uint4 (&ki)[8], uint8_t* img_q,
                                             uint8_t* img_k) {
    int j0, kc;
    qk16_item(0, j0, kc);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t o = kmaj_off(j0 + 16 * m, kc * 8, 128);
        *reinterpret_cast<uint4*>(img_q + o) = qi[m];
        *reinterpret_cast<uint4*>(img_k + o) = ki[m];
    }
}

// Requests every row tile `tile` will read into L2 (one 16-byte-aligned bulk
// prefetch per row), so that its loads, issued a tile later, hit L2.
template <bool ANG, bool IN16, int R, bool XR = false>
__device__ __forceinline__ void prefetch_tile(const M3Params& p, const float* ta,
                                              const float* theta0, int64_t tile, int n_chunks,
                                              int tid) {
    const int64_t BH = p.batch * p.heads, H = p.heads, L = p.len;
    const int64_t bh = tile % BH, bi = bh / H, h = bh % H;
    const int ch = static_cast<int>(tile / BH);
    constexpr int TS = kTcQ / R;
    const int64_t s0 = static_cast<int64_t>(ch) * TS;
    const uint32_t es = IN16 ? 2 : 4;  // bytes per element of q, k, v, z
    // per-row work: v rows on threads [0, TS), z rows on [TS, 2 TS) (wrapping),
    // plus per-head ta or cos/sin rows; the contiguous blocks (q, k and shared
    // ta rows of the tile's natural-time range), the gate spans and theta0 on
    // threads 0..6 as a second task
    const int ri = tid % TS;
    const int64_t it = s0 + ri;
    if (it < L) {
        const int64_t t = p.reverse ? L - 1 - it : it;
        const int64_t row = (bi * L + t) * H + h;
        if (tid < TS) {
            const uint8_t* v = static_cast<const uint8_t*>(static_cast<const void*>(p.v));
            prefetch_lines(v + row * kTcP * R * es, kTcP * R * es);
            if (ANG) {
                if (!p.angles_shared && (p.n_angles & 3) == 0 && p.n_angles > 0)
                    prefetch_lines(ta + row * p.n_angles, static_cast<uint32_t>(p.n_angles * 4));
            } else {
                prefetch_lines(p.cos + row * (kTcN / 2), kTcN * 2);
                prefetch_lines(p.sin + row * (kTcN / 2), kTcN * 2);
            }
        } else if (tid < 2 * TS && p.z) {
            prefetch_lines(static_cast<const uint8_t*>(static_cast<const void*>(p.z)) + row * kTcP * es, kTcP * es);
        }
    }
    if (tid < 7) {
        int64_t lo = p.reverse ? L - (s0 + TS) : s0;
        int64_t hi = p.reverse ? L - s0 : s0 + TS;
        lo = lo < 0 ? 0 : lo;
        hi = hi > L ? L : hi;
        if (hi <= lo) return;
        const int64_t n = hi - lo;
        if (tid < 2) {
            if (h != 0) return;  // q, k rows are shared by all heads
            const uint8_t* b = static_cast<const uint8_t*>(static_cast<const void*>(tid == 0 ? p.q : p.k));
            prefetch_l2(b + (bi * L + lo) * R * kTcN * es, static_cast<uint32_t>(n * R * kTcN * es));
        } else if (tid == 2) {
            if (ANG && p.angles_shared && h == 0 && (p.n_angles & 3) == 0 && p.n_angles > 0)
                prefetch_l2(ta + (bi * L + lo) * p.n_angles, static_cast<uint32_t>(n * p.n_angles * 4));
        } else if (tid < 6) {
            // gate rows (+1 step for the trapezoid's next step), 16-byte aligned span
            const float* g = tid == 3 ? p.dt : tid == 4 ? p.trap : p.adt;
            if (reinterpret_cast<uintptr_t>(g) & 15u) return;  // bulk prefetch needs 16-byte alignment
            const int64_t glo = lo > 0 ? lo - 1 : 0, ghi = hi < L ? hi + 1 : L;
            const int64_t a = (bh * L + glo) & ~int64_t(3), b = ((bh * L + ghi) + 3) & ~int64_t(3);
            if (b > a) prefetch_l2(g + a, static_cast<uint32_t>((b - a) * 4));
        } else if (ANG && p.n_angles > 0) {
            prefetch_l2(theta0 + (bh * n_chunks + ch) * 64, 256);
        }
    }
}

template <bool ANG, bool IN16, bool OUT16, int R, bool XR>
__global__ void __launch_bounds__(kTcThreads2, 2) m3_tc_fused(M3Params p, ChainWs cw, int n_chunks,
                                                             const float* ta, const float* theta0) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* lcum = reinterpret_cast<float*>(smem + kFGate);  // log2 units
    float* scl = lcum + kTcQ;
    float* gam = scl + kTcQ;
    float* wdec = gam + kTcQ;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kFMisc);
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + kFMisc + 8);  // raw q, k staging
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kFMisc + 16);
    int* tile_slot = reinterpret_cast<int*>(smem + kFMisc + 24);  // the next tile

    float* last_decay = reinterpret_cast<float*>(smem + kFMisc + 28);
    float* gwtot = reinterpret_cast<float*>(smem + kFMisc + 32);  // angles mode: gate warp totals
    float* qtot = reinterpret_cast<float*>(smem + kFQtot);  // angles mode: quadrant totals
    float* th0s = qtot + 4 * 64;                            // angles mode: chunk's theta0
    float* qbs = reinterpret_cast<float*>(smem + kFBias);   // [R][dqk]
    float* kbs = qbs + R * kTcN;
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    constexpr int kSt = kTcN * kTcP;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t H = p.heads, L = p.len, BH = p.batch * p.heads;
    const int64_t n_tiles = BH * n_chunks;

    if (warp == 0) tmem_alloc(tmem_slot, 256);
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(bar_ld, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // bf16 angles mode: the tile's raw q, k rows are bulk-copied into the Q
    // and K operand regions at the start of the tile
    constexpr bool kStageQK = ANG && IN16 && R == 1 && !XR;
    uint32_t ld_phase = 0;
    bool ld_pending = false;
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int hc = warp >> 2;                 // column half of this warp
    const int r = (warp & 3) * 32 + lane;     // TMEM lane: row i (G, Y, Z) / state row n (dS)
    const uint32_t tG = tmem, tY = tmem, tZ = tmem + 64, tS = tmem + 128;
    uint32_t phase = 0;
    bool ok = true;

    // Thread 0 takes the next tile when the current one starts; the CTA
    // prefetches it into L2 during the current one.  Tiles still come from
    // the counter in order: the lowest tile any CTA is working on always has
    // a finished predecessor, so the chain cannot stall.
    if (tid == 0) *tile_slot = static_cast<int>(atomicAdd(cw.counter, 1u));
    __syncthreads();
    int64_t tile = *tile_slot;
    if (tile < n_tiles) prefetch_tile<ANG, IN16, R, XR>(p, ta, theta0, tile, n_chunks, tid);
    __syncthreads();  // every thread has read the first tile
    while (ok && tile < n_tiles) {
        // every thread read the slot (the next tile) before the previous
        // tile's closing barrier, so thread 0 may refill it now
        if (tid == kTcThreads2 - 32) *tile_slot = static_cast<int>(atomicAdd(cw.counter, 1u));
        const int64_t bh = tile % BH;
        const int ch = static_cast<int>(tile / BH);
        const int64_t bi = bh / H, h = bh % H;
        const int64_t it0 = static_cast<int64_t>(ch) * (kTcQ / R);  // first step of the tile
        int n_rows = 0;  // kStageQK: rows of the tile
        if (kStageQK) {
            int64_t lo, hi;
            chunk_range(L, ch, p.reverse, lo, hi);
            n_rows = static_cast<int>(hi - lo);
            if (tid == 32) {
                const uint32_t bytes = static_cast<uint32_t>(n_rows) * kTcN * 2;
                const uint16_t* q16 = static_cast<const uint16_t*>(static_cast<const void*>(p.q));
                const uint16_t* k16 = static_cast<const uint16_t*>(static_cast<const void*>(p.k));
                mbar_expect_tx(bar_ld, 2 * bytes);
                bulk_g2s(smem + kFQ, q16 + (bi * L + lo) * kTcN, bytes, bar_ld);
                bulk_g2s(smem + kFK, k16 + (bi * L + lo) * kTcN, bytes, bar_ld);
            }
            ld_pending = true;
        }

        float xv[kXItems][8];
        uint4 xraw[kXItems];  // bf16 inputs: v stays packed until after the gate barrier
        auto load_xraw = [&]() {
#pragma unroll
            for (int q = 0; q < kXItems; ++q) {
                int j, pc;
                x_item(q, j, pc);
                const int64_t itx = it0 + j;
                xraw[q] = make_uint4(0u, 0u, 0u, 0u);
                if (itx < L) {
                    const int64_t t = p.reverse ? L - 1 - itx : itx;
                    xraw[q] = ld8_raw16(p.v, ((bi * L + t) * H + h) * kTcP + pc * 8);
                }
            }
        };
        uint4 xr16[4];  // bf16 per-rank X: raw 16-byte chunks until the gate barrier
        if (XR && IN16) {
            load_x_xr16_raw<R>(p, bi, h, it0, xr16);
        } else if (XR) {
            load_x_xr<R, IN16>(p, bi, h, it0, xv);
        } else if (R > 1) {
            load_x_r<R>(p, bi, h, it0, xv);
        } else if (IN16) {
            if (!kStageQK) load_xraw();  // staged mode: after the rotation (registers)
        } else {
            if (!ANG) load_x_t<false>(p, bi, h, it0, xv);  // angles mode: after the rotation
        }
        if (ANG)
            ang_part_a<!IN16>(p, ta, theta0, bi, h, bh, ch, n_chunks, reinterpret_cast<float*>(smem + kFX),
                       qtot, th0s);
        for (int i = tid; i < R * kTcN; i += kTcThreads2) {
            qbs[i] = (!XR || p.q_bias) ? __ldg(p.q_bias + h * R * kTcN + i) : 0.f;
            kbs[i] = (!XR || p.k_bias) ? __ldg(p.k_bias + h * R * kTcN + i) : 0.f;
        }
        if (ANG) {
            if (warp < 4) gates_split_1(p, bh, it0, lcum, scl, gam, gwtot);
        } else if (warp == 0) {
            tile_gates_r<R>(p, bh, it0, lcum, scl, gam, wdec, last_decay);
        }
        __syncthreads();
        const int64_t next_tile = *tile_slot;
        if (next_tile < n_tiles) prefetch_tile<ANG, IN16, R, XR>(p, ta, theta0, next_tile, n_chunks,
                                                             (tid + kTcThreads2 / 2) % kTcThreads2);
        // X and w o X operand images (in angles mode after the rotation,
        // whose theta table shares their shared memory)
        auto store_x = [&]() {
            if (ANG && !IN16) load_x_t<false>(p, bi, h, it0, xv);
            if (kStageQK) load_xraw();
            if (IN16 && R == 1 && !XR) {
#pragma unroll
                for (int q = 0; q < kXItems; ++q) unpack8(xraw[q], xv[q]);
            }
            if (XR && IN16) {
                store_x_xr16<R>(xr16, wdec, smem + kFX, smem + kFXw);
            } else {
#pragma unroll
                for (int q = 0; q < kXItems; ++q) {
                    int j, pc;
                    x_item(q, j, pc);
                    const float w = wdec[j];
                    float xw[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) xw[e] = w * xv[q][e];
                    const uint32_t o = mnmaj_off(pc * 8, j, kTcP);
                    *reinterpret_cast<uint4*>(smem + kFX + o) = pack8(xv[q]);
                    *reinterpret_cast<uint4*>(smem + kFXw + o) = pack8(xw);
                }
            }
        };
        if (!ANG) store_x();
        if (kStageQK) {
            if (tid < kTcQ) {
                gates_split_2(lcum, scl, wdec, gwtot, last_decay);
            } else if (tid < kTcQ + 64) {
                // theta offset of each quarter (theta0 + the quarters before it
                // in natural time), in place over the quarter totals
                const int pr = tid - kTcQ;
                float v[4], acc = th0s[pr];
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = qtot[q * 64 + pr];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int qq = p.reverse ? 3 - q : q;
                    qtot[qq * 64 + pr] = acc;
                    acc += v[qq];
                }
            }
            __syncthreads();
            const bool got = mbar_wait(bar_ld, ld_phase);
            ld_phase ^= 1;
            ld_pending = !got;
            uint4 qi[8], ki[8];
            ang_part_b16(p, bh, it0, n_rows, reinterpret_cast<const float*>(smem + kFX), qtot,
                         smem + kFQ, smem + kFK, scl, qbs, kbs, qi, ki);
            // every read of the raw rows and of the theta table precedes the
            // operand-image and X stores over them
            if (__syncthreads_or(!got)) {
                if (tid == 0) atomicExch(&g_tc_status, 1);
                ok = false;
                break;
            }
            store_qk_img(qi, ki, smem + kFQ, smem + kFK);
            store_x();
        } else if (ANG) {
            if (tid < kTcQ) gates_split_2(lcum, scl, wdec, gwtot, last_decay);
            ang_part_b<IN16>(p, bi, h, bh, it0, reinterpret_cast<const float*>(smem + kFX), qtot, th0s,
                             smem + kFQ, smem + kFK, scl, qbs, kbs);
            __syncthreads();  // every read of the theta table precedes the X stores
            store_x();
        } else if (XR && IN16)
            stage_qk_xr16<R>(p, bi, h, it0, smem + kFQ, smem + kFK, qbs, kbs);
        else if (XR)
            stage_qk_xr<R, IN16>(p, bi, h, it0, smem + kFQ, smem + kFK, qbs, kbs);
        else if (R > 1)
            stage_qk_mimo<R>(p, bi, h, it0, smem + kFQ, smem + kFK, qbs, kbs);
        else
            stage_qk<true>(p, bi, h, it0, smem + kFQ, smem + kFK, qbs, kbs);
        if (!ANG && R == 1 && p.last_bx && ch == n_chunks - 1 && tid < kTcN / 2) {
            const int jl = static_cast<int>(L - 1 - it0);
            const int64_t t = p.reverse ? 0 : L - 1;
            const int64_t qk = (bi * L + t) * kTcN;
            const float* kb = p.k_bias + h * kTcN;
            const int64_t cs = ((bi * L + t) * H + h) * (kTcN / 2) + tid;
            const float c = p.cos[cs], s = p.sin[cs];
            const float a0 = p.k[qk + 2 * tid] + kb[2 * tid];
            const float a1 = p.k[qk + 2 * tid + 1] + kb[2 * tid + 1];
            p.last_bx[bh * kTcN + 2 * tid] = scl[jl] * (a0 * c - a1 * s);
            p.last_bx[bh * kTcN + 2 * tid + 1] = scl[jl] * (a0 * s + a1 * c);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- group 1: G = Qr Kr^T; dS^T = Kr^T (w o X)
        if (tid == 0) {
            const uint32_t id_G = instr_desc(128, 128, false, false);
            const uint32_t id_S = instr_desc(128, kTcP, true, true);
#pragma unroll
            for (int kb = 0; kb < kTcN / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kFQ + kb * 2 * 16 * 128, 16 * 128, 128);
                const uint64_t b = smem_desc(sbase + kFK + kb * 2 * 16 * 128, 16 * 128, 128);
                umma(tG, a, b, id_G, kb > 0);
            }
            for (int kb = 0; kb < kTcQ / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kFK + kb * 2 * 128, 128, 16 * 128);
                const uint64_t b = smem_desc(sbase + kFXw + kb * 2 * 8 * 128, 8 * 128, 128);
                umma(tS, a, b, id_S, kb > 0);
            }
            umma_commit(bar);
        }
        ok = cta_wait(bar, phase);
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        // ---- chain first (it gates the successor chunk's tile): S_in from
        // the predecessor chunk, S_out published
        {
            bool got = true;
            if (tid == 0 && ch > 0) got = wait_flag(cw.flags + bh, static_cast<unsigned>(ch));
            if (__syncthreads_or(!got)) {
                if (tid == 0) atomicExch(&g_tc_status, 1);
                ok = false;
                break;
            }
            float sin_[32], ds[32];
            // slot layout: float4 q of thread (r, hc) at [hc * 8 + q][r], so
            // that a warp's accesses are 512 contiguous bytes
            const float4* slot_in = reinterpret_cast<const float4*>(cw.slots + (bh * 2 + ((ch + 1) & 1)) * kSt) +
                                    hc * 8 * kTcN + r;
            float4* slot_out = reinterpret_cast<float4*>(cw.slots + (bh * 2 + (ch & 1)) * kSt) + hc * 8 * kTcN + r;
            if (ch > 0) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 v4 = __ldcg(slot_in + q * kTcN);
                    sin_[4 * q] = v4.x; sin_[4 * q + 1] = v4.y; sin_[4 * q + 2] = v4.z; sin_[4 * q + 3] = v4.w;
                }
            } else {
#pragma unroll
                for (int q = 0; q < 32; ++q) sin_[q] = 0.f;
            }
            tmem_ld32(tS + t_lane + hc * 32, ds);
            const float dec = *last_decay;
            float so[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) so[q] = fmaf(dec, sin_[q], ds[q]);
            if (ch + 1 < n_chunks) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    __stcg(slot_out + q * kTcN,
                           make_float4(so[4 * q], so[4 * q + 1], so[4 * q + 2], so[4 * q + 3]));
            } else if (p.last_state) {
                // final state, (p, n) layout
#pragma unroll
                for (int q = 0; q < 32; ++q) p.last_state[(bh * kTcP + hc * 32 + q) * kTcN + r] = so[q];
            }
            // S_in^T operand image (m = p, k = n): 4 chunks of 8 p at state row r
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = sin_[c8 * 8 + e];
                *reinterpret_cast<uint4*>(smem + kFS + mnmaj_off(hc * 32 + c8 * 8, r, kTcP)) = pack8(f);
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();  // every thread's S_out stores precede the release below
            tc_fence_after();
            // the barrier orders every thread's S_out stores before this
            // release (cumulative at gpu scope)
            if (tid == 0 && ch + 1 < n_chunks) st_release(cw.flags + bh, static_cast<unsigned>(ch + 1));
        }
        {
            // W = mask o G (row i = r, this warp's column half) over Kr
            const float li = lcum[r], gi = gam[r];
#pragma unroll
            for (int cb = 0; cb < 2; ++cb) {
                float g[32];
                tmem_ld32(tG + t_lane + hc * 64 + cb * 32, g);
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    const int j0 = hc * 64 + cb * 32 + c8 * 8;
                    const float4 la = *reinterpret_cast<const float4*>(lcum + j0);
                    const float4 lb = *reinterpret_cast<const float4*>(lcum + j0 + 4);
                    const float4 sa = *reinterpret_cast<const float4*>(scl + j0);
                    const float4 sb = *reinterpret_cast<const float4*>(scl + j0 + 4);
                    const float lj[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                    const float sj[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
                    float wv[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        // steps of rows j and r: the mask couples every rank of a step
                        const int sjr = (j0 + c) / R, sir = r / R;
                        const float m = sjr < sir ? ex2_approx(li - lj[c]) * sj[c] : (sjr == sir ? gi : 0.f);
                        wv[c] = m * g[c8 * 8 + c];
                    }
                    *reinterpret_cast<uint4*>(smem + kFK + kmaj_off(r, j0, 128)) = pack8(wv);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t id_Y = instr_desc(128, kTcP, false, true);
            for (int kb = 0; kb < kTcQ / 16; ++kb) {
                const uint64_t a = smem_desc(sbase + kFK + kb * 2 * 16 * 128, 16 * 128, 128);
                const uint64_t b = smem_desc(sbase + kFX + kb * 2 * 8 * 128, 8 * 128, 128);
                umma(tY, a, b, id_Y, kb > 0);
            }
            if (ch > 0) {
                const uint32_t id_Z = instr_desc(128, kTcP, false, true);
#pragma unroll
                for (int kb = 0; kb < kTcN / 16; ++kb) {
                    const uint64_t a = smem_desc(sbase + kFQ + kb * 2 * 16 * 128, 16 * 128, 128);
                    const uint64_t b = smem_desc(sbase + kFS + kb * 2 * 8 * 128, 8 * 128, 128);
                    umma(tZ, a, b, id_Z, kb > 0);
                }
            }
            umma_commit(bar);
        }
        // bf16 SISO: this row's v and z for the epilogue, requested before
        // waiting for the last MMAs
        uint4 vraw[4], zraw[4];
        if (IN16 && R == 1) {
            const int64_t ite = it0 + r;
            const int64_t te = ite < L ? (p.reverse ? L - 1 - ite : ite) : 0;
            const int64_t voff = ((bi * L + te) * H + h) * kTcP + hc * 32;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                vraw[q] = ite < L ? ld8_raw16(p.v, voff + 8 * q) : make_uint4(0u, 0u, 0u, 0u);
                zraw[q] = (ite < L && p.z) ? ld8_raw16(p.z, voff + 8 * q) : make_uint4(0u, 0u, 0u, 0u);
            }
        }
        ok = cta_wait(bar, phase);
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        {
            float y[32];
            tmem_ld32(tY + t_lane + hc * 32, y);
            if (ch > 0) {
                float zt[32];
                tmem_ld32(tZ + t_lane + hc * 32, zt);
                const float el = ex2_approx(lcum[r]);
#pragma unroll
                for (int q = 0; q < 32; ++q) y[q] = fmaf(el, zt[q], y[q]);
            }
            if (XR && R == 4) {
                // per-rank MIMO, rank 4: out (b, l, h, dv, R) row (t, rank) =
                // y + D x.  The 4 lanes of a step (adjacent lanes, one rank
                // each) exchange 8-channel blocks in two butterfly stages so
                // that lane k ends with channels 8k..8k+7 of every rank: 32
                // contiguous output elements, written as 16-byte stores.
                const int64_t it = it0 + r / R;
                const int rk = r % R;
                const bool hi = rk & 2, lo = rk & 1;
                float A0[8], A1[8], B0[8], B1[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    // stage 1 (lanes k, k ^ 2): keep blocks 2 hi, 2 hi + 1
                    const float s0 = hi ? y[i] : y[16 + i], s1 = hi ? y[8 + i] : y[24 + i];
                    A0[i] = hi ? y[16 + i] : y[i];
                    A1[i] = hi ? y[24 + i] : y[8 + i];
                    B0[i] = __shfl_xor_sync(0xffffffffu, s0, 2);
                    B1[i] = __shfl_xor_sync(0xffffffffu, s1, 2);
                }
                float vk[8], vk2[8], vk1[8], vk3[8];  // ranks k, k^2, k^1, k^3; block k
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    // stage 2 (lanes k, k ^ 1): keep block 2 hi + lo
                    vk[i] = lo ? A1[i] : A0[i];
                    vk2[i] = lo ? B1[i] : B0[i];
                    vk1[i] = __shfl_xor_sync(0xffffffffu, lo ? A0[i] : A1[i], 1);
                    vk3[i] = __shfl_xor_sync(0xffffffffu, lo ? B0[i] : B1[i], 1);
                }
                if (it < L) {
                    const int64_t t = p.reverse ? L - 1 - it : it;
                    const int64_t o0 = (((bi * L + t) * H + h) * kTcP + hc * 32 + 8 * rk) * R;
                    float o[32];  // o[4 i + rank]: channel 8k + i
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            o[4 * i + q] = q == rk ? vk[i] : q == (rk ^ 2) ? vk2[i] : q == (rk ^ 1) ? vk1[i] : vk3[i];
                    if (p.d_skip) {
                        const float dsk = p.d_skip[h];
#pragma unroll
                        for (int c8 = 0; c8 < 4; ++c8) {
                            float xv8[8];
                            ld8_in<IN16>(p.v, o0 + 8 * c8, xv8);
#pragma unroll
                            for (int e = 0; e < 8; ++e) o[8 * c8 + e] = fmaf(dsk, xv8[e], o[8 * c8 + e]);
                        }
                    }
#pragma unroll
                    for (int c8 = 0; c8 < 4; ++c8) {
                        float f8[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f8[e] = o[8 * c8 + e];
                        if (OUT16) {
                            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + o0 + 8 * c8) = pack8(f8);
                        } else {
                            float4* o4 = reinterpret_cast<float4*>(p.out + o0 + 8 * c8);
                            o4[0] = make_float4(f8[0], f8[1], f8[2], f8[3]);
                            o4[1] = make_float4(f8[4], f8[5], f8[6], f8[7]);
                        }
                    }
                }
            } else if (XR) {
                // per-rank MIMO: out (b, l, h, dv, R) row (t, rank) = y + D x
                const int64_t it = it0 + r / R;
                const int rk = r % R;
                if (it < L) {
                    const int64_t t = p.reverse ? L - 1 - it : it;
                    const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
                    const int64_t base = (((bi * L + t) * H + h) * kTcP + hc * 32) * R + rk;
#pragma unroll
                    for (int q = 0; q < 32; ++q) {
                        float o = y[q];
                        if (p.d_skip) o = fmaf(dsk, ld1_in<IN16>(p.v, base + q * R), o);
                        if (OUT16)
                            reinterpret_cast<__nv_bfloat16*>(p.out)[base + q * R] = __float2bfloat16_rn(o);
                        else
                            p.out[base + q * R] = o;
                    }
                }
            } else if (R > 1) {
                // MIMO: out_t = sum_r phi_r o g_r o (y_(t,r) + D x_(t,r)),
                // g_r = silu(z o zeta_r) (1 without z); the R rows of a step
                // are R adjacent lanes of this warp
                const int64_t it = it0 + r / R;
                const int rk = r % R;
                const bool live = it < L;
                const int64_t t = live ? (p.reverse ? L - 1 - it : it) : 0;
                const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
                const int64_t voff = ((bi * L + t) * H + h) * kTcP + hc * 32;
                const int64_t poff = (h * R + rk) * kTcP + hc * 32;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float vv[8], ps[8], ph[8], zt[8], ze[8];
                    if (live) {
                        ldg8(p.v + voff + 8 * q, vv);
                        ldg8(p.psi + poff + 8 * q, ps);
                        ldg8(p.phi + poff + 8 * q, ph);
                        if (p.z) {
                            ldg8(p.z + voff + 8 * q, zt);
                            ldg8(p.zeta + poff + 8 * q, ze);
                        }
                    }
                    float o8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float a = live ? fmaf(dsk, ps[e] * vv[e], y[8 * q + e]) * ph[e] : 0.f;
                        if (live && p.z) a *= silu_f(zt[e] * ze[e]);
#pragma unroll
                        for (int o = 1; o < R; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                        o8[e] = a;
                    }
                    if (live && rk == 0) {
                        float* o = p.out + (p.out_blh ? ((bi * L + t) * H + h) : (bh * L + t)) * kTcP +
                                   hc * 32 + 8 * q;
                        reinterpret_cast<float4*>(o)[0] = make_float4(o8[0], o8[1], o8[2], o8[3]);
                        reinterpret_cast<float4*>(o)[1] = make_float4(o8[4], o8[5], o8[6], o8[7]);
                    }
                }
            } else {
                const int64_t it = it0 + r;
                if (it < L) {
                    const float dsk = p.d_skip ? p.d_skip[h] : 0.f;
                    const int64_t t = p.reverse ? L - 1 - it : it;
                    const int64_t voff = ((bi * L + t) * H + h) * kTcP + hc * 32;
                    const int64_t ooff = (p.out_blh ? ((bi * L + t) * H + h) : (bh * L + t)) * kTcP + hc * 32;
                    float vv[4][8], zz[4][8];
    #pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (IN16) {
                            unpack8(vraw[q], vv[q]);
                            unpack8(zraw[q], zz[q]);
                        } else {
                            ld8_in<IN16>(p.v, voff + 8 * q, vv[q]);
                            if (p.z) ld8_in<IN16>(p.z, voff + 8 * q, zz[q]);
                        }
                    }
    #pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float r8[8];
    #pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            r8[e] = fmaf(dsk, vv[q][e], y[8 * q + e]);
                            if (p.z) r8[e] *= silu_f(zz[q][e]);
                        }
                        if (OUT16) {
                            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + ooff + 8 * q) = pack8(r8);
                        } else {
                            float4* o4 = reinterpret_cast<float4*>(p.out + ooff + 8 * q);
                            o4[0] = make_float4(r8[0], r8[1], r8[2], r8[3]);
                            o4[1] = make_float4(r8[4], r8[5], r8[6], r8[7]);
                        }
                    }
                }
            }
            }
        // the next tile overwrites shared memory and tensor memory
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tile = next_tile;
    }
    if (!ok) mbar_wait(bar, phase ^ 1);  // MMAs still in flight: bounded second wait
    if (ld_pending) mbar_wait(bar_ld, ld_phase);  // a staging copy in flight: bounded wait
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace

bool m3_tc_applicable(const M3Params& p) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool siso = p.psi == nullptr && p.rank == 1;
    const bool mimo = p.psi != nullptr && (p.rank == 2 || p.rank == 4) && al(p.psi) && al(p.zeta) &&
                      al(p.phi);
    return (siso || mimo) && p.dqk == kTcN && p.dv == kTcP && al(p.q) && al(p.k) && al(p.v) &&
           al(p.z) && al(p.out) && al(p.q_bias) && al(p.k_bias) && al(p.cos) && al(p.sin) &&
           p.len > 0;
}

bool m3_tc_angles_applicable(const M3Params& p) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return p.psi == nullptr && p.rank == 1 && p.dqk == kTcN && p.dv == kTcP && p.len > 0 &&
           p.n_angles >= 0 && p.n_angles <= kTcN / 2 && al(p.q) && al(p.k) && al(p.v) &&
           al(p.z) && al(p.out) && al(p.q_bias) && al(p.k_bias);
}

size_t m3_tc_workspace_bytes(const M3Params& p) {
    const int64_t nc = (p.len + kTcQ - 1) / kTcQ;
    return static_cast<size_t>(p.batch * p.heads * nc) * (kChunkSt + kStImg + 16);
}

// Per-device memory pool for the workspace.  It keeps what it has reserved
// (release threshold = max), so repeated calls reuse the same pages instead
// of mapping fresh ones on every call, as the default pool (threshold 0)
// does after each synchronization.
namespace {
constexpr int kMaxPoolDevices = 64;
std::mutex g_pool_mu;
cudaMemPool_t g_pool[kMaxPoolDevices] = {};

}  // namespace

cudaError_t device_workspace_pool(cudaMemPool_t* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxPoolDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    if (!g_pool[dev]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        e = cudaMemPoolCreate(&pool, &props);
        if (e != cudaSuccess) return e;
        uint64_t keep = ~0ull;
        e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(pool);
            return e;
        }
        g_pool[dev] = pool;
    }
    *out = g_pool[dev];
    return cudaSuccess;
}


// Three-launch form (kernels A, B, C): selected with the kernel override
// kKnobM3TcSplit = 1 (arm_scan_set_kernel_override).
cudaError_t m3_tc_launch_split(const M3Params& p, cudaStream_t stream) {
    const int64_t bh = p.batch * p.heads;
    const int n_chunks = static_cast<int>((p.len + kTcQ - 1) / kTcQ);
    cudaError_t e = cudaFuncSetAttribute(m3_tc_out, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kCSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(m3_tc_out, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(m3_tc_dstate, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kASmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(m3_tc_dstate, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    // stream-ordered workspace: valid under stream capture, freed after use
    void* raw = nullptr;
    cudaMemPool_t pool = nullptr;
    e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    e = cudaMallocFromPoolAsync(&raw, m3_tc_workspace_bytes(p), pool, stream);
    if (e != cudaSuccess) return e;
    const size_t units = static_cast<size_t>(bh) * n_chunks;
    TcWs ws;
    ws.st = static_cast<float*>(raw);
    ws.simg = reinterpret_cast<uint8_t*>(ws.st + units * (kTcN * kTcP));
    ws.decay = reinterpret_cast<float*>(ws.simg + units * kStImg);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    m3_tc_dstate<<<static_cast<unsigned>(units), kTcThreads2, kASmem, stream>>>(p, ws, n_chunks);
    note_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess) {
        m3_tc_state<<<dim3(static_cast<unsigned>(bh), kStSlices), kTcThreads2, 0, stream>>>(p, ws, n_chunks);
        note_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        const size_t grid = units < static_cast<size_t>(2 * sms) ? units : static_cast<size_t>(2 * sms);
        m3_tc_out<<<static_cast<unsigned>(grid), kTcThreads2, kCSmem, stream>>>(p, ws, n_chunks);
        note_launch();
        e = cudaGetLastError();
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}


template <bool ANG, bool IN16, bool OUT16, int R = 1, bool XR = false>
cudaError_t launch_fused_kernel(const M3Params& p, const ChainWs& cw, int n_chunks, const float* ta,
                                const float* theta0, cudaStream_t stream) {
    auto kern = m3_tc_fused<ANG, IN16, OUT16, R, XR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kFSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t units = p.batch * p.heads * n_chunks;
    const int64_t grid = units < 2 * sms ? units : 2 * sms;
    kern<<<static_cast<unsigned>(grid), kTcThreads2, kFSmem, stream>>>(p, cw, n_chunks, ta, theta0);
    note_launch();
    return cudaGetLastError();
}

cudaError_t m3_tc_launch_fused(const M3Params& p, cudaStream_t stream) {
    const int64_t bh = p.batch * p.heads;
    const int64_t steps = kTcQ / p.rank;  // steps per tile (128 rows = steps x rank)
    const int n_chunks = static_cast<int>((p.len + steps - 1) / steps);
    const bool ang = p.angles != nullptr;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    const size_t slot_bytes = static_cast<size_t>(bh) * 2 * kChunkSt;
    const size_t flag_bytes = (static_cast<size_t>(bh + 1) * sizeof(unsigned int) + 255) / 256 * 256;
    const size_t ta_floats =
        ang ? static_cast<size_t>(p.batch * p.len * (p.angles_shared ? 1 : p.heads) * p.n_angles) : 0;
    const size_t th_floats = ang ? static_cast<size_t>(bh) * n_chunks * 64 : 0;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, slot_bytes + flag_bytes + (ta_floats + th_floats) * 4 + 16,
                                pool, stream);
    if (e != cudaSuccess) return e;
    ChainWs cw;
    cw.slots = static_cast<float*>(raw);
    cw.flags = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(raw) + slot_bytes);
    cw.counter = cw.flags + bh;
    float* theta0 = reinterpret_cast<float*>(static_cast<uint8_t*>(raw) + slot_bytes + flag_bytes);
    float* ta = theta0 + th_floats;
    e = cudaMemsetAsync(cw.flags, 0, flag_bytes, stream);
    if (e == cudaSuccess && ang && p.n_angles > 0) {
        // chunk sums of ta * dt per (bh, chunk, pair); each tile of the main
        // kernel sums the ones before it into its theta0
        const size_t sh_bytes = static_cast<size_t>(kTcQ) * (64 + p.heads) * 4;
        if (p.angles_shared && sh_bytes <= 200 * 1024) {
            auto kern = p.in_bf16 ? m3_tc_angle_sums_shared<true> : m3_tc_angle_sums_shared<false>;
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(sh_bytes));
            if (e == cudaSuccess) {
                kern<<<dim3(static_cast<unsigned>(n_chunks), static_cast<unsigned>(p.batch)), 256, sh_bytes,
                       stream>>>(p, ta, theta0, n_chunks);
                note_launch();
                e = cudaGetLastError();
            }
        } else {
            const dim3 g(static_cast<unsigned>(n_chunks), static_cast<unsigned>(bh));
            if (p.in_bf16)
                m3_tc_angle_sums<true><<<g, 256, 0, stream>>>(p, ta, theta0, n_chunks);
            else
                m3_tc_angle_sums<false><<<g, 256, 0, stream>>>(p, ta, theta0, n_chunks);
            note_launch();
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess && p.x_per_rank) {
#define XR_PICK(RK)                                                                                   \
    (p.in_bf16 ? (p.out_bf16 ? launch_fused_kernel<false, true, true, RK, true>(p, cw, n_chunks, nullptr, nullptr, stream)   \
                             : launch_fused_kernel<false, true, false, RK, true>(p, cw, n_chunks, nullptr, nullptr, stream)) \
               : (p.out_bf16 ? launch_fused_kernel<false, false, true, RK, true>(p, cw, n_chunks, nullptr, nullptr, stream)  \
                             : launch_fused_kernel<false, false, false, RK, true>(p, cw, n_chunks, nullptr, nullptr, stream)))
        e = p.rank == 4 ? XR_PICK(4) : XR_PICK(2);
#undef XR_PICK
    } else if (e == cudaSuccess) {
        if (p.rank == 4)
            e = launch_fused_kernel<false, false, false, 4>(p, cw, n_chunks, nullptr, nullptr, stream);
        else if (p.rank == 2)
            e = launch_fused_kernel<false, false, false, 2>(p, cw, n_chunks, nullptr, nullptr, stream);
        else if (!ang)
            e = launch_fused_kernel<false, false, false>(p, cw, n_chunks, nullptr, nullptr, stream);
        else if (p.in_bf16 && p.out_bf16)
            e = launch_fused_kernel<true, true, true>(p, cw, n_chunks, ta, theta0, stream);
        else if (p.in_bf16)
            e = launch_fused_kernel<true, true, false>(p, cw, n_chunks, ta, theta0, stream);
        else if (p.out_bf16)
            e = launch_fused_kernel<true, false, true>(p, cw, n_chunks, ta, theta0, stream);
        else
            e = launch_fused_kernel<true, false, false>(p, cw, n_chunks, ta, theta0, stream);
    }
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

cudaError_t m3_tc_launch(const M3Params& p, cudaStream_t stream) {
    if (p.angles || p.rank > 1) return m3_tc_launch_fused(p, stream);
    return kernel_override(kKnobM3TcSplit) == 1 ? m3_tc_launch_split(p, stream) : m3_tc_launch_fused(p, stream);
}

bool m3_tc_xr_applicable(const M3Params& p) {
    auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return (p.rank == 2 || p.rank == 4) && p.dqk == kTcN && p.dv == kTcP && p.len > 0 && !p.psi && !p.z &&
           al(p.q_bias) && al(p.k_bias) && p.batch * p.heads <= 65535;
}

// Per-rank MIMO: the RoPE pre-pass (raw angles -> cos/sin in a stream-ordered
// workspace; one angle row per step when angles_shared; no rotated pairs
// gives cos 1, sin 0), then the fused tensor-core scan.
cudaError_t m3_tc_launch_xr(const M3Params& p0, const float* angles, int64_t n_angles, int angles_shared,
                            cudaStream_t stream) {
    M3Params p = p0;
    p.x_per_rank = 1;
    const int64_t half = kTcN / 2;
    const size_t cs_floats = static_cast<size_t>(p.batch * p.len * p.heads * half);
    const size_t ws_bytes = n_angles > 0 ? angle_workspace_bytes(p.batch, p.heads, p.len, n_angles) : 0;
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return e;
    void* raw = nullptr;
    e = cudaMallocFromPoolAsync(&raw, 2 * cs_floats * 4 + ws_bytes + 256, pool, stream);
    if (e != cudaSuccess) return e;
    float* cosv = static_cast<float*>(raw);
    float* sinv = cosv + cs_floats;
    float* ws = sinv + cs_floats;
    AngleParams a{angles, p.dt, cosv, sinv, p.batch, p.heads, p.len, n_angles, half};
    a.angles_shared = angles_shared;
    e = angle_launch(a, ws, stream);
    p.cos = cosv;
    p.sin = sinv;
    if (e == cudaSuccess) e = m3_tc_launch_fused(p, stream);
    const cudaError_t ef = cudaFreeAsync(raw, stream);
    return e != cudaSuccess ? e : ef;
}

int m3_tc_status_and_clear() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
    cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
    return v;
}

}  // namespace b200scan

