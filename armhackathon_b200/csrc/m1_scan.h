// Internal launch interface of the Mamba-1 kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200scan {

constexpr int kBackendAuto = 0;
constexpr int kBackendSequential = 1;  // the ABI's "scalar" backend value
constexpr int64_t kMaxState = 256;

// Device pointers, layouts as reference kernel/arm-scan-core/src/lib.rs:9-16.
struct M1Params {
    const float* u;
    const float* delta;
    const float* A;
    const float* B;
    const float* C;
    const float* d_skip;      // nullable
    const float* z;           // nullable
    const float* delta_bias;  // nullable
    const float* h0;          // nullable
    float* out;
    float* last_state;        // nullable
    int64_t batch, dim, len, state, groups;
    int delta_softplus;
    int reverse;
    // Segmented view (time-split scans; tile kernel only): logical batch
    // b' = b * seg_count + s is segment s (steps s*len .. s*len+len-1) of
    // batch b of tensors whose rows are len_full long.  seg_count 0 or 1
    // with len_full 0: the plain layout.  out == nullptr: state only.
    int64_t seg_count = 1;
    int64_t len_full = 0;
    // Two-pass kernel only: add y to what out already holds (the second
    // traversal of a bidirectional scan summed in place).
    int out_acc = 0;
    // Lane kernel only: segment count to use (0: chosen from the shape).
    int segments = 0;
    // Final-state forms only: sum over the sequence of dt per (batch,
    // channel) row, written when non-null (a segment summary).
    float* dt_sum = nullptr;
};

bool m1_pointers_aligned16(const M1Params& p);
// Per-device stream-ordered memory pool for kernel workspaces; keeps what it
// has reserved (defined in m3_tc.cu).
cudaError_t device_workspace_pool(cudaMemPool_t* out);
// Final state only (no outputs): the two-pass kernel's first pass and
// carries, or the tile kernel in its state-only mode.  cudaErrorNotSupported
// for d_state > 16.
cudaError_t m1_final_state_launch(const M1Params& p, cudaStream_t stream);
// Single-token state update (m1_decode.cu): p.u = x (batch, dim), p.delta =
// dt (batch, dim), p.B/p.C (batch, groups, state), p.out (batch, dim);
// state (batch, dim, state) is read and updated in place.
cudaError_t m1_decode_launch(const M1Params& p, float* state, cudaStream_t stream);
// Lanes-over-states kernel (m1_lane.cu), the default for d_state <= 16,
// length a multiple of 4 and 16-byte aligned tensors: segment count (0: not
// applicable) and launcher.
int m1_lane_segments(const M1Params& p);
cudaError_t m1_lane_launch(const M1Params& p, int segments, cudaStream_t stream);
// Both traversals of one bidirectional scan with the lane kernel: one shared
// first pass (bwd is fwd with reverse = 1 and its own out / last_state;
// bwd.out_acc sums into fwd.out; fwd.out == nullptr: final states only).
int m1_lane_bidir_segments(const M1Params& fwd);
cudaError_t m1_lane_bidir_launch(const M1Params& fwd, const M1Params& bwd, int segments,
                                 cudaStream_t stream);
// Two-phase bidirectional form over a caller's workspace (sequence
// parallelism): the plan (segment count, 0 when the lane kernel cannot take
// the shape; *ws_bytes its workspace) and a phase: summary (shared pass 1,
// carries from fwd.h0 / bwd.h0 into last_state and fwd.dt_sum) or finish
// (carries from the incoming states, both rescans; pass 1's aggregates are
// read from the workspace, which must be unchanged since the summary call).
int m1_lane_bidir_plan(const M1Params& shape, size_t* ws_bytes);
cudaError_t m1_lane_bidir_phase(const M1Params& fwd, const M1Params& bwd, void* workspace, size_t ws_bytes,
                                bool summary, cudaStream_t stream);
// SS2D column-major traversals (forward and reverse) of (batch, dim, h, w)
// grids read in place, added into p.out (which holds the row-major
// traversals' sum); the finished sum is multiplied by scale.
// cudaErrorNotSupported when d_state > 16 or the dims do not fit.
cudaError_t m1_ss2d_cols_launch(const M1Params& p, int64_t h, int64_t w, float scale, cudaStream_t stream);
// Device status of the lane kernels (1: a bounded staging wait expired),
// cleared by the read.
int m1_lane_status_and_clear();
// Final states of both traversals (no outputs); each from its own h0.
cudaError_t m1_bidir_states_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                   cudaStream_t stream);
// Both final states and the per-row sum of dt (fwd.dt_sum), from zero.
cudaError_t m1_segment_summary_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                      cudaStream_t stream);
// Bidirectional scan summed into fwd.out (bwd.out unused).
cudaError_t m1_bidir_sum_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                                cudaStream_t stream);
// Causal depthwise conv1d (kernel K, zero history) + bias + SiLU over
// (batch, dim, len) rows, weights (dim, K) (m1_conv.cu).
cudaError_t m1_conv_silu_launch(const float* x, const float* w, const float* bias, float* out,
                                int64_t batch, int64_t dim, int64_t len, int K, cudaStream_t stream);
// Segments of a time-split Mamba-1 scan (1: no split) and its launcher.
int m1_timesplit_segments(const M1Params& p);
cudaError_t m1_timesplit_launch(const M1Params& p, int segments, cudaStream_t stream);
int m1_pick_channels_per_cta(int64_t rows);
cudaError_t m1_scan_launch(const M1Params& p, int backend, cudaStream_t stream);
// Pipelined row-tile kernel (m1_tile.cu); requires state <= 16.
cudaError_t m1_tile_launch(const M1Params& p, int variant, cudaStream_t stream);
// Forward and reverse scans of the same inputs (fused bidirectional entry).
cudaError_t m1_bidir_launch(const M1Params& fwd, const M1Params& bwd, int backend,
                            cudaStream_t stream);

}  // namespace b200scan
