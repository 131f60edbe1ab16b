// Internal launch interface of the Mamba-3 angle pre-pass (m3_angles.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200scan {

struct AngleParams {
    const float* angles;  // (batch, len, heads, n_angles)
    const float* dt;      // (batch, heads, len)
    float* cos;           // (batch, len, heads, half)
    float* sin;
    int64_t batch, heads, len, n_angles, half;
    // traversal of a (len / grid_w) x grid_w grid stored row-major (SS2D):
    // col_major 1 reads angles and dt at step t's grid position; cos/sin are
    // written in traversal order
    int64_t grid_w = 0;
    int col_major = 0;
    // 1: angles are (batch, len, n_angles), one row per step shared by the
    // heads (theta still differs per head through dt)
    int angles_shared = 0;
};

size_t angle_workspace_bytes(int64_t batch, int64_t heads, int64_t len, int64_t n_angles);
cudaError_t angle_launch(const AngleParams& a, float* workspace, cudaStream_t stream);

// Allocation-free variant: chunk sums in a fixed device array of this many
// floats (4 MiB); sets *too_big (and launches nothing) when the problem needs
// more.  The first call on a device looks up the array's device address.
constexpr int64_t kAngleNoAllocMaxFloats = int64_t(1) << 20;
cudaError_t angle_noalloc_launch(const AngleParams& a, cudaStream_t stream, bool* too_big);

}  // namespace b200scan
