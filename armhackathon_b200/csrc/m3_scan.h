// Internal launch interface of the Mamba-3 kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200scan {

// Device pointers, layouts as reference kernel/arm-scan-core/src/mamba3/
// mod.rs:44-56 (with rank: q, k (b, l, rank, dqk); biases (h, rank, dqk)).
struct M3Params {
    const float* q;
    const float* k;
    const float* v;
    const float* adt;
    const float* dt;
    const float* trap;
    const float* q_bias;
    const float* k_bias;
    const float* cos;
    const float* sin;
    const float* d_skip;  // nullable
    const float* z;       // nullable
    const float* psi;     // MIMO only (all three or none)
    const float* zeta;
    const float* phi;
    float* out;           // (b, h, l, dv) head-major
    float* last_state;    // nullable, (b, h, dv, dqk)
    float* last_bx;       // nullable, (b, h, dqk), SISO only
    int64_t batch, heads, dv, dqk, len, rank;
    int reverse;
    // tensor-core extension (arm_scan_mamba3_siso_tc_async); zero otherwise
    const void* angles;     // raw RoPE angles, (b, l, n_angles) shared or (b, l, h, n_angles)
    int64_t n_angles;       // rotated pairs; pairs >= n_angles are unrotated
    int angles_shared;      // 1: one angle row per (b, l) for all heads
    int in_bf16;            // q, k, v, z, angles are bf16 (else fp32)
    int out_bf16;           // out is bf16 (else fp32)
    int out_blh;            // out is (b, l, h, dv) (else head-major (b, h, l, dv))
    // traversal of a (len / grid_w) x grid_w token grid stored row-major:
    // col_major 1 walks it column by column (SS2D); q, k, v, z, adt, dt, trap
    // and out are read / written at the grid position of each step, cos/sin
    // at the step (the angle pre-pass writes them in traversal order)
    int64_t grid_w;
    int col_major;
    int out_acc;            // out += y (the four SS2D traversals sum in place)
    // MIMO with the input given per rank (tensor-core kernel only): v is X
    // (b, l, h, dv, rank), q / k are C / B (b, l, dqk, rank), out is
    // (b, l, h, dv, rank) per rank; no psi / zeta / phi / z, biases nullable
    int x_per_rank;
};

// grid position of traversal step t
__host__ __device__ inline int64_t m3_phys(const M3Params& p, int64_t t) {
    if (!p.col_major) return t;
    const int64_t rows = p.len / p.grid_w;
    return (t % rows) * p.grid_w + t / rows;
}

bool m3_shape_supported(int64_t dv, int64_t dqk, int64_t rank);
cudaError_t m3_scan_launch(const M3Params& p, int backend, cudaStream_t stream);
// Chunked dual-form kernel (m3_chunk.cu): the default when applicable.
bool m3_chunk_applicable(const M3Params& p);
cudaError_t m3_chunk_launch(const M3Params& p, cudaStream_t stream);
// Tensor-core kernel (m3_tc.cu): bf16 operands, fp32 accumulation; backend 3.
bool m3_tc_applicable(const M3Params& p);
cudaError_t m3_tc_launch(const M3Params& p, cudaStream_t stream);
int m3_tc_status_and_clear();
// Per-rank MIMO on the tensor cores (x_per_rank layouts; q = C, k = B):
// shape test and launcher (RoPE pre-pass from raw fp32 angles, then the scan).
bool m3_tc_xr_applicable(const M3Params& p);
// out -= count * (D + gamma_t (q_t . k_t)) v_t [* silu(z_t)] per (b, t, h):
// the diagonal correction of the non-causal aggregation (m3_noncausal.cu);
// q, k (b, len, dqk) unrotated, out / v / z (b, len, h, dv).
cudaError_t m3_diag_sub_launch(const M3Params& p, int count, cudaStream_t stream);
cudaError_t m3_tc_launch_xr(const M3Params& p, const float* angles, int64_t n_angles, int angles_shared,
                            cudaStream_t stream);  // 1 if a bounded wait expired since the last call
// true if p (with angles set) is a shape the extension entry covers
bool m3_tc_angles_applicable(const M3Params& p);

}  // namespace b200scan
