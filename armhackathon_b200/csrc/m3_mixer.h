// Mamba-3 mixer prologue (m3_mixer.cu): the in_proj split, gates, B/C
// RMSNorm and relayouts of the reference's Mamba3Mixer.forward.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200scan {

struct MixerParams {
    const float* proj;      // (batch, len, W) in_proj output, one B/C group
    const float* dt_bias;   // (heads,)
    const float* b_norm_w;  // (d_state,)
    const float* c_norm_w;  // (d_state,)
    float a_floor, eps;
    float* z;       // (batch, len, heads, headdim)
    float* x;       // (batch, len, heads, headdim)
    float* q;       // (batch, len, rank, d_state)  RMSNorm(C) * C_norm weight
    float* k;       // (batch, len, rank, d_state)  RMSNorm(B) * B_norm weight
    float* dt;      // (batch, heads, len)
    float* adt;     // (batch, heads, len)
    float* trap;    // (batch, heads, len)
    float* angles;  // (batch, len, n_angles)
    int64_t batch, len, heads, headdim, d_state, rank, n_angles;
};

cudaError_t m3_mixer_prologue_launch(const MixerParams& p, cudaStream_t stream);

}  // namespace b200scan
