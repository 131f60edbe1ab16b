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
};

size_t angle_workspace_bytes(int64_t batch, int64_t heads, int64_t len, int64_t n_angles);
cudaError_t angle_launch(const AngleParams& a, float* workspace, cudaStream_t stream);

}  // namespace b200scan
