/*
 * b200scan -- C ABI of the B200 selective-scan engine (libb200scan.so).
 *
 * Drop-in replacement for the reference's Rust cdylib
 * kernel/arm-scan-ffi/src/lib.rs (ABI v7).  Entry points, structs, enum values
 * and return codes 0-5 keep the reference's names, argument order and meaning
 * so an existing ctypes/cgo binding only changes the library path and the
 * expected version number (now 12; it was 7).  Added since v7:
 *   - device-pointer, stream-ordered variants (suffix _async) that take a
 *     cudaStream_t as `void* stream` and never synchronize;
 *   - a final-state output for the Mamba-3 SISO and MIMO scans;
 *   - return codes 6 (CUDA error) and 7 (timeout of a bounded wait);
 *   - arm_scan_last_error(), a per-thread message for the last failure;
 *   - arm_scan_set_device(), the device ordinal the synchronous entries use;
 *   - extension entry points for the tensor-core Mamba-3 paths, the
 *     per-rank MIMO form, the fused bidirectional forms, non-causal and 2D
 *     compositions, segment summaries for sequence parallelism, decode, the
 *     mixers' prologues and an allocation-free angle pre-pass (each
 *     declared below with its contract).
 *
 * Memory.  The synchronous v7-shaped entry points accept either HOST pointers
 * (every buffer in host memory: inputs are copied to the CUDA device chosen by
 * arm_scan_set_device, by default the calling thread's current device,
 * the scan runs, outputs are copied back, and the call returns when the
 * results are in the caller's buffers -- the reference's blocking contract) or
 * DEVICE pointers (every buffer on the current device: the scan runs on the
 * default stream and the call returns after it completes).  Mixing host and
 * device buffers in one call is rejected with code 2.  The _async variants
 * require device pointers and return as soon as the work is enqueued.
 *
 * Layouts are the reference's (row-major, contiguous, fp32):
 *   Mamba-1  u, delta, z, out (batch, dim, len); a (dim, state);
 *            b, c (batch, groups, state, len); d_skip, delta_bias (dim);
 *            h0, last_state (batch, dim, state)
 *   Mamba-3  q, k (batch, len, rank, dqk); v, z (batch, len, heads, dv);
 *            adt, dt, trap (batch, heads, len); cos, sin (batch, len, heads,
 *            dqk/2); q_bias, k_bias (heads, rank, dqk); d_skip (heads);
 *            psi, zeta, phi (heads, rank, dv);
 *            out (batch, heads, len, dv) -- HEAD-major;
 *            last_state (batch, heads, dv, dqk); last_bx (batch, heads, dqk)
 * state (Mamba-1 d_state) must be <= 256.
 */
#ifndef B200SCAN_H
#define B200SCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ARM_SCAN_ABI_VERSION 13u

/* Return codes (0-5: reference arm-scan-ffi/src/lib.rs:53-58). */
#define ARM_SCAN_OK 0
#define ARM_SCAN_ERR_NULL_POINTER 1
#define ARM_SCAN_ERR_INVALID_DIMS 2
#define ARM_SCAN_ERR_BACKEND_UNAVAILABLE 3
#define ARM_SCAN_ERR_BAD_ENUM 4
#define ARM_SCAN_ERR_PANIC 5
#define ARM_SCAN_ERR_CUDA 6
#define ARM_SCAN_ERR_TIMEOUT 7

/* backend: 0 = auto (chunked sm_100a kernels, fp32 arithmetic), 1 = scalar
 * (a sequential on-device restatement of the reference's scalar loop, for
 * cross-checks), 2 = neon (not available here: code 3), 3 = tensor
 * (extension, Mamba-3 entry points only: tcgen05 tensor-core kernels with
 * bf16 matrix operands, fp32 accumulation and fp32 state, for bf16 models;
 * SISO, or MIMO of rank 2 or 4, with dqk 128, dv 64 and 16-byte aligned
 * tensors, otherwise code 3).
 * threading: 0/1/2 are accepted (auto/sequential/rayon in the reference)
 * and have no effect on a GPU. */

/* Replaces ArmScanDims, arm-scan-ffi/src/lib.rs:44-50. */
typedef struct ArmScanDims {
    size_t batch;
    size_t dim;
    size_t len;
    size_t state;
    size_t groups;
} ArmScanDims;

/* Replaces ArmMamba3Dims, arm-scan-ffi/src/lib.rs:363-373. */
typedef struct ArmMamba3Dims {
    size_t batch;
    size_t heads;
    size_t dv;
    size_t dqk;
    size_t len;
    size_t rank;
} ArmMamba3Dims;

/* Replaces arm_scan_abi_version, arm-scan-ffi/src/lib.rs:37-40.  Returns
 * ARM_SCAN_ABI_VERSION (13). */
uint32_t arm_scan_abi_version(void);

/* Message describing the calling thread's most recent non-zero return. */
const char* arm_scan_last_error(void);

/* Replaces arm_scan_selective_scan_f32, arm-scan-ffi/src/lib.rs:97-116.
 * Nullable: d_skip, z, delta_bias, last_state, h0. */
int arm_scan_selective_scan_f32(const ArmScanDims* dims, const float* u,
                                const float* delta, const float* a,
                                const float* b, const float* c,
                                const float* d_skip, const float* z,
                                const float* delta_bias, int delta_softplus,
                                int reverse, int backend, int threading,
                                float* out, float* last_state, const float* h0);

/* Replaces arm_scan_selective_scan_bidirectional_f32,
 * arm-scan-ffi/src/lib.rs:233-252.  last_fwd/last_bwd both or neither. */
int arm_scan_selective_scan_bidirectional_f32(
    const ArmScanDims* dims, const float* u, const float* delta,
    const float* a, const float* b, const float* c, const float* d_skip,
    const float* z, const float* delta_bias, int delta_softplus, int backend,
    int threading, float* out_fwd, float* out_bwd, float* last_fwd,
    float* last_bwd);

/* Replaces arm_scan_mamba3_scan_f32, arm-scan-ffi/src/lib.rs:417-445.
 * SISO when psi/zeta/phi are all null (rank must be 1), MIMO when all three
 * are given; a partial set is code 1.  last_state/last_bx both or neither
 * (code 1).  For MIMO, last_bx must be null and last_state may be given
 * (v8 extension: the reference rejects any carry for MIMO). */
int arm_scan_mamba3_scan_f32(
    const ArmMamba3Dims* dims, const float* q, const float* k, const float* v,
    const float* adt, const float* dt, const float* trap, const float* q_bias,
    const float* k_bias, const float* cos, const float* sin,
    const float* d_skip, const float* z, const float* mimo_psi,
    const float* mimo_zeta, const float* mimo_phi, int reverse, int backend,
    int threading, float* out, float* last_state, float* last_bx);

/* v8: device pointers, enqueued on `stream` (a cudaStream_t; NULL = the
 * legacy default stream).  Same arguments and codes as the synchronous forms;
 * a CUDA error raised by the enqueue is code 6. */
int arm_scan_selective_scan_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta,
    const float* a, const float* b, const float* c, const float* d_skip,
    const float* z, const float* delta_bias, int delta_softplus, int reverse,
    int backend, int threading, float* out, float* last_state,
    const float* h0, void* stream);

int arm_scan_selective_scan_bidirectional_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta,
    const float* a, const float* b, const float* c, const float* d_skip,
    const float* z, const float* delta_bias, int delta_softplus, int backend,
    int threading, float* out_fwd, float* out_bwd, float* last_fwd,
    float* last_bwd, void* stream);

int arm_scan_mamba3_scan_f32_async(
    const ArmMamba3Dims* dims, const float* q, const float* k, const float* v,
    const float* adt, const float* dt, const float* trap, const float* q_bias,
    const float* k_bias, const float* cos, const float* sin,
    const float* d_skip, const float* z, const float* mimo_psi,
    const float* mimo_zeta, const float* mimo_phi, int reverse, int backend,
    int threading, float* out, float* last_state, float* last_bx,
    void* stream);

/* v8: the Mamba-3 RoPE angle pre-pass on the GPU (device pointers), replacing
 * the torch computation of the reference's angles_to_cos_sin
 * (python/arm_scan/mamba3.py:41-89):
 *   theta[b,t,h,p] = sum_{s<=t} tanh(angles[b,s,h,p]) * pi * dt[b,h,s]
 *   cos/sin (batch, len, heads, dqk/2) = cos/sin(theta) for p < n_angles,
 *   1/0 for n_angles <= p < dqk/2.
 * angles (batch, len, heads, n_angles), dt (batch, heads, len); uses
 * dims->batch, heads, len, dqk (rank and dv are ignored).  `workspace` must
 * hold arm_scan_mamba3_angles_workspace_bytes(...) bytes of device memory,
 * used only during the call's stream-ordered execution. */
size_t arm_scan_mamba3_angles_workspace_bytes(const ArmMamba3Dims* dims, size_t n_angles);
int arm_scan_mamba3_angles_f32_async(const ArmMamba3Dims* dims, const float* angles,
                                     size_t n_angles, const float* dt, float* cos,
                                     float* sin, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* No counterpart in the reference.  The same angle pre-pass for callers that
 * cannot allocate device memory at call time: a host framework or inference
 * server whose device memory is owned by its own allocator (an extra
 * cudaMalloc from a plugin can fail or fragment its pool), or a real-time
 * caller that forbids allocation once it is running.  It calls no cudaMalloc
 * or cudaFree; its scratch is a fixed 4 MiB device array inside the library
 * (held by every GPU that loads the library until the process exits), so a
 * problem needing more than 4 MiB of chunk sums
 * (batch*heads*ceil(len/128)*n_angles*4 bytes) is rejected with code 2.
 * Every call looks up the array's device address for the current device
 * and context (cudaGetSymbolAddress, no allocation), so the entry stays
 * valid across cudaDeviceReset and context changes.  All calls share the one array:
 * calls whose executions overlap on the GPU (different streams, or different
 * host threads) race on it and must be serialized by the caller.  Arguments
 * and results are those of arm_scan_mamba3_angles_f32_async. */
int arm_scan_mamba3_angles_f32_noalloc(const ArmMamba3Dims* dims, const float* angles,
                                       size_t n_angles, const float* dt, float* cos,
                                       float* sin, void* stream);

/* Extension (no counterpart in the reference): Mamba-3 SISO on the tensor
 * cores for bf16 models, with the RoPE angle pre-pass fused in.  Options: */
#define ARM_SCAN_DTYPE_F32 0
#define ARM_SCAN_DTYPE_BF16 1
typedef struct ArmMamba3TcOptions {
    int in_dtype;      /* q, k, v, z and angles: ARM_SCAN_DTYPE_F32 or _BF16 */
    int out_dtype;     /* out: ARM_SCAN_DTYPE_F32 or _BF16 */
    int out_layout;    /* 0: (batch, heads, len, dv) as arm_scan_mamba3_scan_f32;
                          1: (batch, len, heads, dv), the Python op's layout */
    int angles_shared; /* 1: angles (batch, len, n_angles), one row for all heads;
                          0: angles (batch, len, heads, n_angles) */
    size_t n_angles;   /* rotated pairs per step, <= dqk / 2; pairs beyond it are unrotated */
} ArmMamba3TcOptions;

/* Same recurrence and arguments as arm_scan_mamba3_scan_f32_async with
 * rank 1, except: raw angles replace cos/sin (theta = forward cumsum over
 * time of tanh(angle) * pi * dt, computed on the device, as
 * arm_scan_mamba3_angles_f32_async does), the dtypes and output layout come
 * from opts, and MIMO projections do not exist.  adt, dt, trap, q_bias,
 * k_bias, d_skip, last_state, last_bx stay fp32; the state is fp32; matrix
 * operands are rounded to bf16 (the tensor backend).  Device pointers only,
 * 16-byte aligned; dqk must be 128 and dv 64 (else code 3).  Stream-ordered;
 * an expired internal wait is reported by arm_scan_tensor_status. */
int arm_scan_mamba3_siso_tc_async(const ArmMamba3Dims* dims, const ArmMamba3TcOptions* opts,
                                  const void* q, const void* k, const void* v, const float* adt,
                                  const float* dt, const float* trap, const float* q_bias,
                                  const float* k_bias, const void* angles, const float* d_skip,
                                  const void* z, int reverse, void* out, float* last_state,
                                  float* last_bx, void* stream);

/* Extension: Mamba-3 MIMO with the input given per rank, on the tensor
 * cores.  Per (batch, head), with X_t (dv x rank), B_t and C_t (dqk x rank)
 * RoPE-rotated split-halves by theta_t = cumsum(tanh(angle) * pi * dt):
 *   h_t = alpha_t h_{t-1} + beta_t X_{t-1} B_{t-1}^T + gamma_t X_t B_t^T
 *   Y_t = h_t C_t (+ D X_t)
 * alpha = exp(adt), gamma = dt sigmoid(trap), beta = alpha dt (1 -
 * sigmoid(trap)) (the gates of arm_scan_mamba3_scan_f32; "previous" is
 * t + 1 with reverse).  It is the reference's MIMO op
 * (python/arm_scan/mamba3.py:261-334, kernel/arm-scan-core/src/mamba3/
 * mimo.rs:98-284) with x_r given directly instead of psi_r * v and the
 * per-rank outputs returned instead of the zeta-gated, phi-weighted sum.
 * Layouts: x, out (batch, len, heads, dv, rank); b, c (batch, len, dqk,
 * rank); adt, dt, trap (batch, heads, len) fp32; angles fp32, (batch, len,
 * n_angles) with opts->angles_shared = 1 or (batch, len, heads, n_angles)
 * (nullable with n_angles 0: no rotation); d_skip (heads) nullable;
 * last_state (batch, heads, dv, dqk) = h after the last step, nullable.
 * opts->in_dtype is the dtype of x, b, c; opts->out_dtype that of out;
 * opts->out_layout is ignored.  rank 2 or 4, dqk 128, dv 64 (else code 3).
 * Device pointers, stream-ordered; fp32 state, bf16 matrix operands. */
int arm_scan_mamba3_mimo_x_tc_async(const ArmMamba3Dims* dims, const ArmMamba3TcOptions* opts,
                                    const void* x, const void* b, const void* c, const float* adt,
                                    const float* dt, const float* trap, const float* angles,
                                    const float* d_skip, int reverse, void* out, float* last_state,
                                    void* stream);

/* Extension (no counterpart in the reference): the four-direction Mamba-3
 * SISO cross-scan of a token grid in one call (the reference composes it in
 * Python, python/arm_scan/ss2d_mamba3.py).  The grid is len / grid_w rows of
 * grid_w tokens, stored row-major: q, k (batch, len, 1, dqk); v, z (batch,
 * len, heads, dv); angles (batch, len, heads, n_angles); adt, dt, trap
 * (batch, heads, len).  The scan runs row-major and column-major, each
 * forward and backward, reading the grid in place (the angle pre-pass runs
 * per ordering, in its traversal order), and the four outputs are summed
 * into out (batch, len, heads, dv).  n_angles in [1, dqk/2]; d_skip and z
 * nullable.  Device pointers, stream-ordered; fp32 chunk kernels. */
int arm_scan_mamba3_ss2d_f32_async(const ArmMamba3Dims* dims, size_t grid_w, const float* q,
                                   const float* k, const float* v, const float* adt,
                                   const float* dt, const float* trap, const float* q_bias,
                                   const float* k_bias, const float* angles, size_t n_angles,
                                   const float* d_skip, const float* z, float* out, void* stream);

/* Extension: the non-causal Mamba-3 aggregation (every token sees every
 * other), forward + reverse - diagonal, in one call (the reference composes
 * it in Python, python/arm_scan/mamba3_noncausal.py:89-98 for 1D and
 * :178-218 for a grid).  grid_w == 0 or len: one sequence (1D), with raw
 * angles or with precomputed cos / sin (batch, len, heads, dqk/2); otherwise
 * a token grid of len / grid_w rows, row-major and column-major orderings
 * summed, raw angles only.  Layouts as arm_scan_mamba3_ss2d_f32_async; out
 * (batch, len, heads, dv).  The scans sum into out in place and one kernel
 * subtracts the doubly counted diagonal term.  fp32 chunk kernels. */
int arm_scan_mamba3_noncausal_f32_async(const ArmMamba3Dims* dims, size_t grid_w, const float* q,
                                        const float* k, const float* v, const float* adt,
                                        const float* dt, const float* trap, const float* q_bias,
                                        const float* k_bias, const float* angles, size_t n_angles,
                                        const float* cos, const float* sin, const float* d_skip,
                                        const float* z, float* out, void* stream);

/* Extension (no counterpart in the reference): the final state of
 * arm_scan_selective_scan_f32_async's recurrence without computing the
 * outputs (D, z and out play no part): the first step of a sequence-parallel
 * scan, whose ranks exchange end states before scanning from them.
 * last_state (batch, dim, state) is required; h0 is nullable.  d_state must
 * be <= 16 (else code 3).  Device pointers, stream-ordered. */
int arm_scan_selective_scan_final_state_f32_async(const ArmScanDims* dims, const float* u,
                                                  const float* delta, const float* a,
                                                  const float* b, const float* c,
                                                  const float* delta_bias, int delta_softplus,
                                                  int reverse, const float* h0,
                                                  float* last_state, void* stream);

/* Extension (no counterpart in the reference; mamba_ssm's
 * selective_state_update): one decode step of the Mamba-1 recurrence for
 * every (batch, channel), updating `state` (batch, dim, state) in place:
 * dt' = softplus(dt + dt_bias) if dt_softplus, h = exp(dt' A) h + dt' x B,
 * out = C.h + D x, times silu(z).  x, dt, z, out are (batch, dim); B, C are
 * (batch, groups, state); A (dim, state); D, dt_bias (dim,).  dims->len is
 * ignored.  Device pointers, stream-ordered; nullable: d_skip, z, dt_bias. */
int arm_scan_selective_state_update_f32_async(const ArmScanDims* dims, float* state,
                                              const float* x, const float* dt, const float* a,
                                              const float* b, const float* c,
                                              const float* d_skip, const float* z,
                                              const float* dt_bias, int dt_softplus, float* out,
                                              void* stream);

/* Extension (no counterpart in the reference): status of the kernels with
 * device-side waits: the tensor-core kernels (backend 3), whose waits on
 * their own MMA completions are bounded, and the Mamba-1 lane kernel, whose
 * waits on its own TMA staging are bounded; an expired wait abandons the
 * remaining work and sets a device flag.  The synchronous entry points check it themselves (code 7); after
 * an _async call, synchronize the stream and call this: returns 0, or 7
 * (message in arm_scan_last_error) if a wait expired since the last check,
 * and clears the flag. */
int arm_scan_tensor_status(void);

/* Extension (diagnostics, no counterpart in the reference): number of GPU
 * kernels this library has launched in the process so far (all devices,
 * all threads); the difference around a call is that call's launch count. */
unsigned long long arm_scan_kernel_launches(void);

/* Extension (tests and measurements, no counterpart in the reference):
 * process-wide kernel-selection overrides; value 0 everywhere is the
 * default dispatch.  Knobs: 0 Mamba-1 kernel (0 auto, 1 lane kernel,
 * 2 row-tile, 3 block-chunked, 4 row-tile with a time split); 1 segment
 * count of the lane / time-split kernels (0 auto; ignored unless it divides
 * the length into segments of a multiple of 4 steps); 2 bidirectional form
 * (0 shared first pass, 1 two independent traversals); 3 Mamba-3 tensor
 * kernel (0 fused, 1 three-launch form); 4 Mamba-3 fp32 chunk form (0 auto,
 * 1 sequential, 2 chunk-parallel); 5 programmatic dependent launch (0 on,
 * 1 off).  Returns 0, or 4 for an unknown knob or a negative value. */
int arm_scan_set_kernel_override(int knob, int value);

/* Extension: the device ordinal the synchronous entry points stage HOST
 * buffers through, for the calling thread (the reference runs on the host
 * and has no device argument; this is the boundary's device_ordinal).  -1
 * (the default) means the thread's current CUDA device.  Device-pointer
 * calls always run on the device that owns the buffers.  Returns 0, or 2
 * for an ordinal outside [-1, device count). */
int arm_scan_set_device(int ordinal);

/* Extension: the bidirectional scan merged by sum, as the reference's
 * bidirectional_scan(merge="sum") computes it from the two outputs of
 * arm_scan_selective_scan_bidirectional_f32 (python/arm_scan/bidirectional.py:
 * 98-175): out = out_fwd + out_bwd, (batch, dim, len).  Same inputs, dims and
 * codes as the bidirectional entry (backend 0 or 1); last_fwd / last_bwd are
 * both-or-neither.  Device pointers, stream-ordered.  Where the two-pass
 * kernel applies, both traversals share their first pass (every exp of it
 * computed once) and the reverse traversal adds into `out` in place.
 * h0_fwd / h0_bwd (nullable, (batch, dim, state)): incoming state of each
 * traversal (the reverse one's at t = len - 1). */
int arm_scan_selective_scan_bidirectional_sum_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* d_skip, const float* z, const float* delta_bias,
    int delta_softplus, int backend, int threading, float* out, float* last_fwd,
    float* last_bwd, const float* h0_fwd, const float* h0_bwd, void* stream);

/* Extension: final states of both traversals of a bidirectional scan, without
 * outputs: last_fwd = the state after the forward traversal, last_bwd = after
 * the reverse one (at t = 0), each (batch, dim, state) from a zero start.
 * Inputs and codes as the bidirectional entry (no D or z: they do not reach
 * the states).  Where the two-pass kernel applies both come from one shared
 * first pass.  With the sum entry's h0_fwd / h0_bwd this gives a sequence
 * split over devices its segment summaries and then its outputs. */
int arm_scan_selective_scan_bidirectional_final_states_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, int backend, float* last_fwd,
    float* last_bwd, void* stream);

/* Extension (no counterpart in the reference): the summary a segment of a
 * sequence split over devices contributes -- both traversals' final states
 * from zero (as arm_scan_selective_scan_bidirectional_final_states_f32_async)
 * and dt_sum (batch, dim), the sum over the segment of dt = softplus(delta +
 * delta_bias) (or delta + delta_bias), from the same pass over the inputs
 * where the lane kernel applies.  Device pointers, stream-ordered. */
int arm_scan_selective_scan_segment_summary_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, int backend, float* last_fwd,
    float* last_bwd, float* dt_sum, void* stream);

/* Extension (no counterpart in the reference, whose HF patch leaves it to
 * torch, python/arm_scan/patch.py:57-116): the Mamba-1 mixer's input
 * prologue, causal depthwise conv1d + bias + SiLU, in one pass:
 *   out[b, d, t] = silu(bias[d] + sum_{j < kernel} weight[d, j] x[b, d, t - kernel + 1 + j])
 * with zeros before t = 0.  x, out (batch, dim, len); weight (dim, kernel);
 * bias (dim) nullable; kernel in [1, 8].  Device pointers, stream-ordered. */
int arm_scan_causal_conv1d_silu_f32_async(size_t batch, size_t dim, size_t len, size_t kernel,
                                          const float* x, const float* weight, const float* bias,
                                          float* out, void* stream);

/* Extension (no counterpart in the reference): the bidirectional sum in two
 * phases around an exchange, for a sequence split over devices.  The
 * summary phase makes one shared pass over this segment and returns its
 * summary (both traversals' end states from zero, the per-row sum of dt) --
 * as arm_scan_selective_scan_segment_summary_f32_async does -- and keeps
 * the pass's per-segment aggregates in the caller's workspace; the finish
 * phase, given the incoming states folded from the other segments'
 * summaries, writes out = forward + reverse outputs (as the sum entry with
 * h0_fwd / h0_bwd) without a second pass over the inputs to rebuild those
 * aggregates.  The workspace (16-byte aligned, the size reported by
 * ..._bidirectional_workspace_bytes for the same dims, 0 when the shape is
 * not covered: d_state > 16 or len not a multiple of 4) must not change
 * between the two calls.  Device pointers, stream-ordered; code 3 if the
 * tensors are not 16-byte aligned. */
size_t arm_scan_selective_scan_bidirectional_workspace_bytes(const ArmScanDims* dims);
int arm_scan_selective_scan_bidirectional_summary_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, void* workspace, size_t ws_bytes,
    float* last_fwd, float* last_bwd, float* dt_sum, void* stream);
int arm_scan_selective_scan_bidirectional_finish_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* d_skip, const float* z, const float* delta_bias, int delta_softplus,
    void* workspace, size_t ws_bytes, const float* h0_fwd, const float* h0_bwd, float* out,
    void* stream);

/* Extension: the Mamba-1 SS2D cross-scan (reference python/arm_scan/ss2d.py
 * :102-167, merges "sum" and "mean") as one call over grids read in place:
 * u, delta (batch, dim, h, w), B, C (batch, groups, state, h, w), A (dim,
 * state), d_skip, delta_bias (dim) nullable; no z.  out (batch, dim, h, w)
 * = row-major forward + backward + column-major forward + backward, each
 * with its own D u (times 0.25 when merge_mean).  dims->len must be h * w;
 * d_state <= 16 and, with groups > 1, dim / groups a multiple of 8 (code 3
 * otherwise).  Device pointers, stream-ordered. */
int arm_scan_selective_scan_ss2d_f32_async(
    const ArmScanDims* dims, size_t h, size_t w, const float* u, const float* delta,
    const float* a, const float* b, const float* c, const float* d_skip, const float* delta_bias,
    int delta_softplus, int merge_mean, float* out, void* stream);

/* Extension: shape of the Mamba-3 mixer whose prologue
 * arm_scan_mamba3_mixer_prologue_f32_async runs (one B/C group; rank 1 for
 * SISO).  The in_proj row is W = 2*heads*headdim + 2*rank*d_state + 3*heads
 * + n_angles floats wide (apps/mamba3_lm/block.py:116-121). */
typedef struct ArmMamba3MixerDims {
    size_t batch;
    size_t len;
    size_t heads;
    size_t headdim;
    size_t d_state;
    size_t rank;
    size_t n_angles;
} ArmMamba3MixerDims;

/* Extension (reference apps/mamba3_lm/block.py:146-177, Mamba3Mixer.forward
 * between in_proj and the scan, in torch there): one pass over the in_proj
 * output proj (batch, len, W), fp32, writing the scan's inputs:
 *   z, x       (batch, len, heads, headdim)  the first two slices, contiguous
 *   q, k       (batch, len, rank, d_state)   RMSNorm(C) * c_norm_weight and
 *              RMSNorm(B) * b_norm_weight, rstd = 1/sqrt(mean(v^2) + eps)
 *   dt, adt    (batch, heads, len)           dt = softplus(dd_dt + dt_bias)
 *              (threshold 20), adt = min(-heavy_tail(dd_A), -a_floor) * dt,
 *              heavy_tail(v) = max(v, 0) + 1 / (1 - min(v, 0))
 *   trap       (batch, heads, len)           the pre-sigmoid slice, transposed
 *   angles     (batch, len, n_angles)        the last slice, contiguous
 * Device pointers, stream-ordered; none nullable.  n_angles <= d_state / 2. */
int arm_scan_mamba3_mixer_prologue_f32_async(const ArmMamba3MixerDims* dims, const float* proj,
                                             const float* dt_bias, const float* b_norm_weight,
                                             const float* c_norm_weight, float a_floor, float eps,
                                             float* z, float* x, float* q, float* k, float* dt,
                                             float* adt, float* trap, float* angles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200SCAN_H */
