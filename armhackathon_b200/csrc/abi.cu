// The C ABI (include/b200scan.h): validation, host/device buffer handling and
// dispatch to the sm_100a kernels.
//
// Validation follows the reference's C boundary, kernel/arm-scan-ffi/src/
// lib.rs: null checks first (code 1), then enum decoding (code 4), then
// overflow-checked element counts and shape rules (code 2), mirroring
// arm-scan-core's validate() (lib.rs:181-249) and mamba3/mod.rs:213-335.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b200scan.h"
#include "common.cuh"
#include "m1_scan.h"
#include "m3_mixer.h"
#include "m3_angles.h"
#include "m3_scan.h"

using namespace b200scan;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(ARM_SCAN_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

bool mul_ok(size_t a, size_t b, size_t* out) {
    if (a != 0 && b > SIZE_MAX / a) return false;
    *out = a * b;
    return true;
}

bool mul3(size_t a, size_t b, size_t c, size_t* out) {
    size_t t;
    return mul_ok(a, b, &t) && mul_ok(t, c, out);
}

bool mul4(size_t a, size_t b, size_t c, size_t d, size_t* out) {
    size_t t;
    return mul3(a, b, c, &t) && mul_ok(t, d, out);
}

int check_enums(int backend, int threading, bool allow_tensor = false) {
    if (allow_tensor && backend == 3 && threading >= 0 && threading <= 2) return ARM_SCAN_OK;
    if (backend < 0 || backend > 2 || threading < 0 || threading > 2)
        return fail(ARM_SCAN_ERR_BAD_ENUM, "backend %d / threading %d out of range", backend,
                    threading);
    if (backend == 2)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the NEON backend does not exist on a GPU");
    return ARM_SCAN_OK;
}

// ---------------------------------------------------------------------------
// Buffers of one call: where they live and how many bytes each spans.
struct Buf {
    const void* ptr;
    size_t bytes;
    bool output;
};

enum class Where { Host, Device, Mixed };

Where classify(const std::vector<Buf>& bufs, int* device) {
    int n_host = 0, n_dev = 0;
    *device = -1;
    for (const Buf& b : bufs) {
        if (!b.ptr) continue;
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, b.ptr) != cudaSuccess) {
            cudaGetLastError();
            ++n_host;
            continue;
        }
        if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
            ++n_dev;
            if (*device < 0) *device = at.device;
        } else {
            ++n_host;
        }
    }
    if (n_dev && n_host) return Where::Mixed;
    return n_dev ? Where::Device : Where::Host;
}

// Device staging area for host-pointer calls: one per device, grown on
// demand and kept for the life of the process.
struct Staging {
    std::mutex mu;
    void* base = nullptr;
    size_t cap = 0;
    cudaStream_t stream = nullptr;
};
Staging g_staging[64];

class DeviceGuard {
  public:
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&old_);
        if (dev >= 0 && dev != old_) {
            cudaSetDevice(dev);
            switched_ = true;
        }
    }
    ~DeviceGuard() {
        if (switched_) cudaSetDevice(old_);
    }

  private:
    int old_ = 0;
    bool switched_ = false;
};

size_t round_up(size_t x) { return (x + 255) & ~size_t(255); }

// Runs `run(device_ptrs, stream)` either directly on device buffers (then
// synchronizes) or after staging host buffers through device memory.
int m1_status_code() {
    return m1_lane_status_and_clear() ? fail(ARM_SCAN_ERR_TIMEOUT, "a Mamba-1 staging wait expired")
                                      : ARM_SCAN_OK;
}

int tensor_status_code() {
    const int m1 = m1_lane_status_and_clear();
    if (m1) return fail(ARM_SCAN_ERR_TIMEOUT, "a Mamba-1 staging wait expired");
    return m3_tc_status_and_clear()
               ? fail(ARM_SCAN_ERR_TIMEOUT, "a tensor-core MMA completion wait expired")
               : ARM_SCAN_OK;
}

// post (optional) runs after a successful synchronization and may turn the
// result into an error (device-side status flags).
// Device the synchronous entries stage host buffers through, per calling
// thread (arm_scan_set_device); -1: the thread's current CUDA device.
thread_local int g_host_device = -1;

template <class Run>
int run_sync(std::vector<Buf>& bufs, Run&& run, int (*post)() = nullptr) {
    int dev = -1;
    const Where w = classify(bufs, &dev);
    if (w == Where::Mixed)
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "buffers mix host and device memory; pass all host or all device pointers");
    std::vector<void*> dptr(bufs.size(), nullptr);
    if (w == Where::Device) {
        DeviceGuard g(dev);
        for (size_t i = 0; i < bufs.size(); ++i) dptr[i] = const_cast<void*>(bufs[i].ptr);
        int rc = run(dptr, static_cast<cudaStream_t>(nullptr));
        if (rc != ARM_SCAN_OK) return rc;
        cudaError_t e = cudaStreamSynchronize(nullptr);
        if (e != cudaSuccess) return cuda_fail(e, "kernel");
        return post ? post() : ARM_SCAN_OK;
    }
    DeviceGuard pick(g_host_device);
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur < 0 || cur >= 64) return fail(ARM_SCAN_ERR_CUDA, "device ordinal %d unsupported", cur);
    Staging& st = g_staging[cur];
    std::lock_guard<std::mutex> lock(st.mu);
    size_t total = 0;
    for (const Buf& b : bufs)
        if (b.ptr) total += round_up(b.bytes);
    if (total > st.cap) {
        if (st.base) cudaFree(st.base);
        st.base = nullptr;
        st.cap = 0;
        e = cudaMalloc(&st.base, total);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
        st.cap = total;
    }
    if (!st.stream) {
        e = cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
    }
    char* p = static_cast<char*>(st.base);
    for (size_t i = 0; i < bufs.size(); ++i) {
        if (!bufs[i].ptr) continue;
        dptr[i] = p;
        p += round_up(bufs[i].bytes);
        if (!bufs[i].output) {
            e = cudaMemcpyAsync(dptr[i], bufs[i].ptr, bufs[i].bytes, cudaMemcpyHostToDevice,
                                st.stream);
            if (e != cudaSuccess) return cuda_fail(e, "copy to device");
        }
    }
    int rc = run(dptr, st.stream);
    if (rc != ARM_SCAN_OK) {
        cudaStreamSynchronize(st.stream);
        return rc;
    }
    for (size_t i = 0; i < bufs.size(); ++i) {
        if (!bufs[i].ptr || !bufs[i].output) continue;
        e = cudaMemcpyAsync(const_cast<void*>(bufs[i].ptr), dptr[i], bufs[i].bytes,
                            cudaMemcpyDeviceToHost, st.stream);
        if (e != cudaSuccess) return cuda_fail(e, "copy to host");
    }
    e = cudaStreamSynchronize(st.stream);
    if (e != cudaSuccess) return cuda_fail(e, "kernel");
    return post ? post() : ARM_SCAN_OK;
}

// ---------------------------------------------------------------------------
// Mamba-1
struct M1Counts {
    size_t bdl, bgnl, dn, bdn;
};

int m1_validate(const ArmScanDims* d, M1Counts* c) {
    const size_t v[5] = {d->batch, d->dim, d->len, d->state, d->groups};
    const char* names[5] = {"batch", "dim", "len", "state", "groups"};
    for (int i = 0; i < 5; ++i)
        if (v[i] == 0) return fail(ARM_SCAN_ERR_INVALID_DIMS, "dimension `%s` is zero", names[i]);
    if (d->dim % d->groups)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "groups (%zu) does not divide dim (%zu)", d->groups,
                    d->dim);
    if (d->state > static_cast<size_t>(kMaxState))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "state %zu exceeds the supported maximum %lld",
                    d->state, static_cast<long long>(kMaxState));
    if (!mul3(d->batch, d->dim, d->len, &c->bdl) ||
        !mul4(d->batch, d->groups, d->state, d->len, &c->bgnl) ||
        !mul_ok(d->dim, d->state, &c->dn) || !mul3(d->batch, d->dim, d->state, &c->bdn))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    // every byte offset must fit in int64 for the kernels
    if (c->bdl > (SIZE_MAX >> 3) / 4 || c->bgnl > (SIZE_MAX >> 3) / 4)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "tensors too large");
    return ARM_SCAN_OK;
}

M1Params m1_params(const ArmScanDims* d, const std::vector<void*>& p, int softplus, int reverse) {
    M1Params m{};
    m.u = static_cast<const float*>(p[0]);
    m.delta = static_cast<const float*>(p[1]);
    m.A = static_cast<const float*>(p[2]);
    m.B = static_cast<const float*>(p[3]);
    m.C = static_cast<const float*>(p[4]);
    m.d_skip = static_cast<const float*>(p[5]);
    m.z = static_cast<const float*>(p[6]);
    m.delta_bias = static_cast<const float*>(p[7]);
    m.batch = static_cast<int64_t>(d->batch);
    m.dim = static_cast<int64_t>(d->dim);
    m.len = static_cast<int64_t>(d->len);
    m.state = static_cast<int64_t>(d->state);
    m.groups = static_cast<int64_t>(d->groups);
    m.delta_softplus = softplus != 0;
    m.reverse = reverse != 0;
    return m;
}

int m1_run(const M1Params& m, int backend, cudaStream_t s) {
    cudaError_t e = m1_scan_launch(m, backend, s);
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "selective_scan launch");
}

std::vector<Buf> m1_bufs(const M1Counts& c, const float* u, const float* delta, const float* a,
                         const float* b, const float* cc, const float* d_skip, const float* z,
                         const float* delta_bias, size_t dim) {
    return {{u, c.bdl * 4, false},        {delta, c.bdl * 4, false}, {a, c.dn * 4, false},
            {b, c.bgnl * 4, false},       {cc, c.bgnl * 4, false},   {d_skip, dim * 4, false},
            {z, c.bdl * 4, false},        {delta_bias, dim * 4, false}};
}

// ---------------------------------------------------------------------------
// Mamba-3
struct M3Counts {
    size_t blqk, bhl, hqk, hrv, blhv, blhr, bhvq, bhq;
};

int m3_validate(const ArmMamba3Dims* d, bool mimo, const void* last_state, const void* last_bx,
                M3Counts* c) {
    const size_t v[6] = {d->batch, d->heads, d->dv, d->dqk, d->len, d->rank};
    const char* names[6] = {"batch", "heads", "dv", "dqk", "len", "rank"};
    for (int i = 0; i < 6; ++i)
        if (v[i] == 0) return fail(ARM_SCAN_ERR_INVALID_DIMS, "dimension `%s` is zero", names[i]);
    if (d->dqk % 2)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "dqk (%zu) must be even for RoPE lane pairs", d->dqk);
    if (d->rank > 1 && !mimo)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "rank > 1 requires the MIMO projections");
    if (mimo && last_bx)
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "MIMO defines no last_bx carry (one k per step is SISO-only)");
    if (!m3_shape_supported(static_cast<int64_t>(d->dv), static_cast<int64_t>(d->dqk),
                            static_cast<int64_t>(d->rank)))
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "head dims dv=%zu dqk=%zu rank=%zu are outside the supported set "
                    "(dv, dqk <= 256, rank <= 8)",
                    d->dv, d->dqk, d->rank);
    bool ok = mul4(d->batch, d->len, d->rank, d->dqk, &c->blqk) &&
              mul3(d->batch, d->heads, d->len, &c->bhl) &&
              mul3(d->heads, d->rank, d->dqk, &c->hqk) && mul3(d->heads, d->rank, d->dv, &c->hrv) &&
              mul4(d->batch, d->len, d->heads, d->dv, &c->blhv) &&
              mul4(d->batch, d->len, d->heads, d->dqk / 2, &c->blhr) &&
              mul4(d->batch, d->heads, d->dv, d->dqk, &c->bhvq) &&
              mul3(d->batch, d->heads, d->dqk, &c->bhq);
    if (!ok) return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    (void)last_state;
    return ARM_SCAN_OK;
}

int m3_check_ptrs(const void* const* req, int n_req, const void* last_state, const void* last_bx,
                  const void* psi, const void* zeta, const void* phi, bool* mimo) {
    for (int i = 0; i < n_req; ++i)
        if (!req[i]) return fail(ARM_SCAN_ERR_NULL_POINTER, "required pointer #%d is null", i);
    const int n_mimo = (psi != nullptr) + (zeta != nullptr) + (phi != nullptr);
    if (n_mimo != 0 && n_mimo != 3)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "psi/zeta/phi must be all null or all given");
    *mimo = n_mimo == 3;
    if (!*mimo && ((last_state == nullptr) != (last_bx == nullptr)))
        return fail(ARM_SCAN_ERR_NULL_POINTER, "last_state and last_bx must be given together");
    return ARM_SCAN_OK;
}

M3Params m3_params(const ArmMamba3Dims* d, const std::vector<void*>& p, int reverse) {
    M3Params m{};
    m.q = static_cast<const float*>(p[0]);
    m.k = static_cast<const float*>(p[1]);
    m.v = static_cast<const float*>(p[2]);
    m.adt = static_cast<const float*>(p[3]);
    m.dt = static_cast<const float*>(p[4]);
    m.trap = static_cast<const float*>(p[5]);
    m.q_bias = static_cast<const float*>(p[6]);
    m.k_bias = static_cast<const float*>(p[7]);
    m.cos = static_cast<const float*>(p[8]);
    m.sin = static_cast<const float*>(p[9]);
    m.d_skip = static_cast<const float*>(p[10]);
    m.z = static_cast<const float*>(p[11]);
    m.psi = static_cast<const float*>(p[12]);
    m.zeta = static_cast<const float*>(p[13]);
    m.phi = static_cast<const float*>(p[14]);
    m.out = static_cast<float*>(p[15]);
    m.last_state = static_cast<float*>(p[16]);
    m.last_bx = static_cast<float*>(p[17]);
    m.batch = static_cast<int64_t>(d->batch);
    m.heads = static_cast<int64_t>(d->heads);
    m.dv = static_cast<int64_t>(d->dv);
    m.dqk = static_cast<int64_t>(d->dqk);
    m.len = static_cast<int64_t>(d->len);
    m.rank = static_cast<int64_t>(d->rank);
    m.reverse = reverse != 0;
    return m;
}

std::vector<Buf> m3_bufs(const M3Counts& c, const ArmMamba3Dims* d, const float* q, const float* k,
                         const float* v, const float* adt, const float* dt, const float* trap,
                         const float* q_bias, const float* k_bias, const float* cos,
                         const float* sin, const float* d_skip, const float* z, const float* psi,
                         const float* zeta, const float* phi, float* out, float* last_state,
                         float* last_bx) {
    return {{q, c.blqk * 4, false},      {k, c.blqk * 4, false},       {v, c.blhv * 4, false},
            {adt, c.bhl * 4, false},     {dt, c.bhl * 4, false},       {trap, c.bhl * 4, false},
            {q_bias, c.hqk * 4, false},  {k_bias, c.hqk * 4, false},   {cos, c.blhr * 4, false},
            {sin, c.blhr * 4, false},    {d_skip, d->heads * 4, false}, {z, c.blhv * 4, false},
            {psi, c.hrv * 4, false},     {zeta, c.hrv * 4, false},     {phi, c.hrv * 4, false},
            {out, c.blhv * 4, true},     {last_state, c.bhvq * 4, true}, {last_bx, c.bhq * 4, true}};
}

int m3_run(const M3Params& m, int backend, cudaStream_t s) {
    if (backend == 3 && !m3_tc_applicable(m))
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE,
                    "the tensor backend covers SISO and MIMO rank 2/4 with dqk 128, dv 64 and "
                    "16-byte aligned tensors");
    cudaError_t e = m3_scan_launch(m, backend, s);
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "mamba3_scan launch");
}

}  // namespace

namespace b200scan {
std::atomic<unsigned long long> g_kernel_launches{0};
void note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
std::atomic<int> g_override[kKnobCount];
int kernel_override(int knob) {
    return knob >= 0 && knob < kKnobCount ? g_override[knob].load(std::memory_order_relaxed) : 0;
}
bool pdl_enabled() { return kernel_override(kKnobPdl) == 0; }
}  // namespace b200scan

extern "C" {

uint32_t arm_scan_abi_version(void) { return ARM_SCAN_ABI_VERSION; }

const char* arm_scan_last_error(void) { return g_last_error.c_str(); }

// Host buffers with batch >= 2: a per-batch pipeline over two streams, so
// that batch b+1's upload overlaps batch b's scan and download (separate
// copy engines; rows of different batches never interact).  Buffers in the
// order of the synchronous entry: u, delta, A, B, C, D, z, delta_bias, h0,
// out, last_state; A, D, delta_bias are shared by the batches.
struct Pipe {
    std::mutex mu;
    void* base = nullptr;
    size_t cap = 0;
    cudaStream_t s[2] = {nullptr, nullptr};
    cudaEvent_t shared_ready = nullptr;
};
Pipe g_pipe[64];

bool m1_pipeline_worthwhile(const ArmScanDims* d, const std::vector<Buf>& bufs) {
    size_t total = 0;
    for (const Buf& b : bufs) total += b.ptr ? b.bytes : 0;
    return d->batch >= 2 && total >= (size_t(16) << 20);
}

int m1_host_pipelined(const ArmScanDims* d, const std::vector<Buf>& bufs, int softplus, int reverse,
                      int backend) {
    constexpr int kSliced[] = {0, 1, 3, 4, 6, 8, 9, 10};
    constexpr int kShared[] = {2, 5, 7};
    const size_t nb = d->batch;
    DeviceGuard pick(g_host_device);
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur < 0 || cur >= 64) return fail(ARM_SCAN_ERR_CUDA, "device ordinal %d unsupported", cur);
    Pipe& pp = g_pipe[cur];
    std::lock_guard<std::mutex> lock(pp.mu);
    size_t off[11] = {}, slot_bytes = 0, shared_bytes = 0;
    for (int i : kShared) {
        off[i] = shared_bytes;
        shared_bytes += bufs[i].ptr ? round_up(bufs[i].bytes) : 0;
    }
    for (int i : kSliced) {
        off[i] = slot_bytes;
        slot_bytes += bufs[i].ptr ? round_up(bufs[i].bytes / nb) : 0;
    }
    const size_t need = shared_bytes + 2 * slot_bytes;
    if (need > pp.cap) {
        if (pp.base) {
            cudaDeviceSynchronize();
            cudaFree(pp.base);
        }
        pp.base = nullptr;
        pp.cap = 0;
        e = cudaMalloc(&pp.base, need);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(pipeline staging)");
        pp.cap = need;
    }
    for (auto& st : pp.s)
        if (!st && (e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_fail(e, "cudaStreamCreate");
    if (!pp.shared_ready &&
        (e = cudaEventCreateWithFlags(&pp.shared_ready, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "cudaEventCreate");
    char* base = static_cast<char*>(pp.base);
    std::vector<void*> dptr(11, nullptr);
    for (int i : kShared) {
        if (!bufs[i].ptr) continue;
        dptr[i] = base + off[i];
        e = cudaMemcpyAsync(dptr[i], bufs[i].ptr, bufs[i].bytes, cudaMemcpyHostToDevice, pp.s[0]);
        if (e != cudaSuccess) return cuda_fail(e, "copy to device");
    }
    if ((e = cudaEventRecord(pp.shared_ready, pp.s[0])) != cudaSuccess ||
        (e = cudaStreamWaitEvent(pp.s[1], pp.shared_ready, 0)) != cudaSuccess)
        return cuda_fail(e, "pipeline event");
    ArmScanDims one = *d;
    one.batch = 1;
    for (size_t b = 0; b < nb; ++b) {
        cudaStream_t st = pp.s[b & 1];
        char* slot = base + shared_bytes + (b & 1) * slot_bytes;
        for (int i : kSliced) {
            if (!bufs[i].ptr) continue;
            const size_t sl = bufs[i].bytes / nb;
            dptr[i] = slot + off[i];
            if (!bufs[i].output) {
                e = cudaMemcpyAsync(dptr[i], static_cast<const char*>(bufs[i].ptr) + b * sl, sl,
                                    cudaMemcpyHostToDevice, st);
                if (e != cudaSuccess) return cuda_fail(e, "copy to device");
            }
        }
        M1Params m = m1_params(&one, dptr, softplus, reverse);
        m.h0 = static_cast<const float*>(dptr[8]);
        m.out = static_cast<float*>(dptr[9]);
        m.last_state = static_cast<float*>(dptr[10]);
        // the whole batch's segment count, so that every row's result is
        // the one the unpipelined call gives
        M1Params whole = m;
        whole.batch = static_cast<int64_t>(nb);
        m.segments = m1_lane_segments(whole);
        const int rc = m1_run(m, backend, st);
        if (rc != ARM_SCAN_OK) {
            cudaStreamSynchronize(pp.s[0]);
            cudaStreamSynchronize(pp.s[1]);
            return rc;
        }
        for (int i : {9, 10}) {
            if (!bufs[i].ptr) continue;
            const size_t sl = bufs[i].bytes / nb;
            e = cudaMemcpyAsync(const_cast<char*>(static_cast<const char*>(bufs[i].ptr)) + b * sl,
                                dptr[i], sl, cudaMemcpyDeviceToHost, st);
            if (e != cudaSuccess) return cuda_fail(e, "copy to host");
        }
    }
    const cudaError_t e0 = cudaStreamSynchronize(pp.s[0]);
    const cudaError_t e1 = cudaStreamSynchronize(pp.s[1]);
    if (e0 != cudaSuccess) return cuda_fail(e0, "kernel");
    if (e1 != cudaSuccess) return cuda_fail(e1, "kernel");
    return m1_status_code();
}

int arm_scan_selective_scan_f32(const ArmScanDims* dims, const float* u, const float* delta,
                                const float* a, const float* b, const float* c,
                                const float* d_skip, const float* z, const float* delta_bias,
                                int delta_softplus, int reverse, int backend, int threading,
                                float* out, float* last_state, const float* h0) {
    if (!dims || !u || !delta || !a || !b || !c || !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    int rc = check_enums(backend, threading);
    if (rc) return rc;
    M1Counts cnt;
    if ((rc = m1_validate(dims, &cnt))) return rc;
    std::vector<Buf> bufs = m1_bufs(cnt, u, delta, a, b, c, d_skip, z, delta_bias, dims->dim);
    bufs.push_back({h0, cnt.bdn * 4, false});
    bufs.push_back({out, cnt.bdl * 4, true});
    bufs.push_back({last_state, cnt.bdn * 4, true});
    int dev = -1;
    if (classify(bufs, &dev) == Where::Host && m1_pipeline_worthwhile(dims, bufs))
        return m1_host_pipelined(dims, bufs, delta_softplus, reverse, backend);
    return run_sync(bufs, [&](const std::vector<void*>& p, cudaStream_t s) {
        M1Params m = m1_params(dims, p, delta_softplus, reverse);
        m.h0 = static_cast<const float*>(p[8]);
        m.out = static_cast<float*>(p[9]);
        m.last_state = static_cast<float*>(p[10]);
        return m1_run(m, backend, s);
    }, m1_status_code);
}

int arm_scan_selective_scan_f32_async(const ArmScanDims* dims, const float* u, const float* delta,
                                      const float* a, const float* b, const float* c,
                                      const float* d_skip, const float* z,
                                      const float* delta_bias, int delta_softplus, int reverse,
                                      int backend, int threading, float* out, float* last_state,
                                      const float* h0, void* stream) {
    if (!dims || !u || !delta || !a || !b || !c || !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    int rc = check_enums(backend, threading);
    if (rc) return rc;
    M1Counts cnt;
    if ((rc = m1_validate(dims, &cnt))) return rc;
    std::vector<void*> p = {const_cast<float*>(u),     const_cast<float*>(delta),
                            const_cast<float*>(a),     const_cast<float*>(b),
                            const_cast<float*>(c),     const_cast<float*>(d_skip),
                            const_cast<float*>(z),     const_cast<float*>(delta_bias)};
    M1Params m = m1_params(dims, p, delta_softplus, reverse);
    m.h0 = h0;
    m.out = out;
    m.last_state = last_state;
    return m1_run(m, backend, static_cast<cudaStream_t>(stream));
}

static int bidir_common(const ArmScanDims* dims, const float* u, const float* delta,
                        const float* a, const float* b, const float* c, const float* d_skip,
                        const float* z, const float* delta_bias, int backend, int threading,
                        float* out_fwd, float* out_bwd, float* last_fwd, float* last_bwd,
                        M1Counts* cnt) {
    if (!dims || !u || !delta || !a || !b || !c || !out_fwd || !out_bwd)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    int rc = check_enums(backend, threading);
    if (rc) return rc;
    if ((rc = m1_validate(dims, cnt))) return rc;
    if ((last_fwd == nullptr) != (last_bwd == nullptr))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "last_fwd and last_bwd must be given together");
    return ARM_SCAN_OK;
}

static int bidir_run(const M1Params& base, float* out_fwd, float* out_bwd, float* last_fwd,
                     float* last_bwd, int backend, cudaStream_t s) {
    M1Params f = base, r = base;
    f.reverse = 0;
    f.out = out_fwd;
    f.last_state = last_fwd;
    r.reverse = 1;
    r.out = out_bwd;
    r.last_state = last_bwd;
    cudaError_t e = m1_bidir_launch(f, r, backend, s);
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "bidirectional launch");
}

int arm_scan_selective_scan_bidirectional_f32(const ArmScanDims* dims, const float* u,
                                              const float* delta, const float* a, const float* b,
                                              const float* c, const float* d_skip, const float* z,
                                              const float* delta_bias, int delta_softplus,
                                              int backend, int threading, float* out_fwd,
                                              float* out_bwd, float* last_fwd, float* last_bwd) {
    M1Counts cnt;
    int rc = bidir_common(dims, u, delta, a, b, c, d_skip, z, delta_bias, backend, threading,
                          out_fwd, out_bwd, last_fwd, last_bwd, &cnt);
    if (rc) return rc;
    std::vector<Buf> bufs = m1_bufs(cnt, u, delta, a, b, c, d_skip, z, delta_bias, dims->dim);
    bufs.push_back({out_fwd, cnt.bdl * 4, true});
    bufs.push_back({out_bwd, cnt.bdl * 4, true});
    bufs.push_back({last_fwd, cnt.bdn * 4, true});
    bufs.push_back({last_bwd, cnt.bdn * 4, true});
    return run_sync(bufs, [&](const std::vector<void*>& p, cudaStream_t s) {
        M1Params m = m1_params(dims, p, delta_softplus, 0);
        return bidir_run(m, static_cast<float*>(p[8]), static_cast<float*>(p[9]),
                         static_cast<float*>(p[10]), static_cast<float*>(p[11]), backend, s);
    }, m1_status_code);
}

int arm_scan_selective_scan_bidirectional_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* d_skip, const float* z, const float* delta_bias,
    int delta_softplus, int backend, int threading, float* out_fwd, float* out_bwd,
    float* last_fwd, float* last_bwd, void* stream) {
    M1Counts cnt;
    int rc = bidir_common(dims, u, delta, a, b, c, d_skip, z, delta_bias, backend, threading,
                          out_fwd, out_bwd, last_fwd, last_bwd, &cnt);
    if (rc) return rc;
    std::vector<void*> p = {const_cast<float*>(u),     const_cast<float*>(delta),
                            const_cast<float*>(a),     const_cast<float*>(b),
                            const_cast<float*>(c),     const_cast<float*>(d_skip),
                            const_cast<float*>(z),     const_cast<float*>(delta_bias)};
    M1Params m = m1_params(dims, p, delta_softplus, 0);
    return bidir_run(m, out_fwd, out_bwd, last_fwd, last_bwd, backend,
                     static_cast<cudaStream_t>(stream));
}

int arm_scan_selective_scan_bidirectional_sum_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* d_skip, const float* z, const float* delta_bias,
    int delta_softplus, int backend, int threading, float* out, float* last_fwd,
    float* last_bwd, const float* h0_fwd, const float* h0_bwd, void* stream) {
    M1Counts cnt;
    int rc = bidir_common(dims, u, delta, a, b, c, d_skip, z, delta_bias, backend, threading,
                          out, out, last_fwd, last_bwd, &cnt);
    if (rc) return rc;
    std::vector<void*> p = {const_cast<float*>(u),     const_cast<float*>(delta),
                            const_cast<float*>(a),     const_cast<float*>(b),
                            const_cast<float*>(c),     const_cast<float*>(d_skip),
                            const_cast<float*>(z),     const_cast<float*>(delta_bias)};
    M1Params base = m1_params(dims, p, delta_softplus, 0);
    M1Params f = base, r = base;
    f.out = out;
    f.last_state = last_fwd;
    f.h0 = h0_fwd;
    r.reverse = 1;
    r.out = nullptr;
    r.last_state = last_bwd;
    r.h0 = h0_bwd;
    cudaError_t e = m1_bidir_sum_launch(f, r, backend, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "bidirectional sum launch");
}

int arm_scan_selective_scan_bidirectional_final_states_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, int backend, float* last_fwd,
    float* last_bwd, void* stream) {
    if (!last_fwd || !last_bwd)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "last_fwd and last_bwd are required");
    M1Counts cnt;
    int rc = bidir_common(dims, u, delta, a, b, c, nullptr, nullptr, delta_bias, backend, 0,
                          last_fwd, last_bwd, last_fwd, last_bwd, &cnt);
    if (rc) return rc;
    std::vector<void*> p = {const_cast<float*>(u), const_cast<float*>(delta),
                            const_cast<float*>(a), const_cast<float*>(b),
                            const_cast<float*>(c), nullptr,
                            nullptr,               const_cast<float*>(delta_bias)};
    M1Params base = m1_params(dims, p, delta_softplus, 0);
    M1Params f = base, r = base;
    f.last_state = last_fwd;
    r.reverse = 1;
    r.last_state = last_bwd;
    cudaError_t e = m1_bidir_states_launch(f, r, backend, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "bidirectional final states launch");
}

int arm_scan_selective_scan_segment_summary_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, int backend, float* last_fwd,
    float* last_bwd, float* dt_sum, void* stream) {
    if (!last_fwd || !last_bwd || !dt_sum)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "last_fwd, last_bwd and dt_sum are required");
    M1Counts cnt;
    int rc = bidir_common(dims, u, delta, a, b, c, nullptr, nullptr, delta_bias, backend, 0,
                          last_fwd, last_bwd, last_fwd, last_bwd, &cnt);
    if (rc) return rc;
    std::vector<void*> p = {const_cast<float*>(u), const_cast<float*>(delta),
                            const_cast<float*>(a), const_cast<float*>(b),
                            const_cast<float*>(c), nullptr,
                            nullptr,               const_cast<float*>(delta_bias)};
    M1Params base = m1_params(dims, p, delta_softplus, 0);
    M1Params f = base, r = base;
    f.last_state = last_fwd;
    f.dt_sum = dt_sum;
    r.reverse = 1;
    r.last_state = last_bwd;
    cudaError_t e = m1_segment_summary_launch(f, r, backend, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "segment summary launch");
}

int arm_scan_causal_conv1d_silu_f32_async(size_t batch, size_t dim, size_t len, size_t kernel,
                                          const float* x, const float* weight, const float* bias,
                                          float* out, void* stream) {
    if (!x || !weight || !out) return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (!batch || !dim || !len || kernel < 1 || kernel > 8)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "zero dimension or kernel (%zu) outside [1, 8]", kernel);
    size_t n = 0;
    if (!mul3(batch, dim, len, &n) || n > (SIZE_MAX >> 3) / 4)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    cudaError_t e = m1_conv_silu_launch(x, weight, bias, out, static_cast<int64_t>(batch),
                                        static_cast<int64_t>(dim), static_cast<int64_t>(len),
                                        static_cast<int>(kernel), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "causal conv1d launch");
}

size_t arm_scan_selective_scan_bidirectional_workspace_bytes(const ArmScanDims* dims) {
    M1Counts cnt;
    if (!dims || m1_validate(dims, &cnt) != ARM_SCAN_OK) return 0;
    std::vector<void*> p(8, nullptr);
    M1Params m = m1_params(dims, p, 1, 0);
    size_t bytes = 0;
    m1_lane_bidir_plan(m, &bytes);
    return bytes;
}

static int bidir_phase_common(const ArmScanDims* dims, const float* u, const float* delta,
                              const float* a, const float* b, const float* c, const float* d_skip,
                              const float* z, const float* delta_bias, int delta_softplus,
                              void* workspace, size_t ws_bytes, float* out, float* last_fwd,
                              float* last_bwd, float* dt_sum, const float* h0_fwd,
                              const float* h0_bwd, bool summary, void* stream) {
    if (!dims || !u || !delta || !a || !b || !c || !workspace)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (summary ? (!last_fwd || !last_bwd || !dt_sum) : !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required output pointer is null");
    M1Counts cnt;
    int rc = m1_validate(dims, &cnt);
    if (rc) return rc;
    std::vector<void*> p = {const_cast<float*>(u), const_cast<float*>(delta),
                            const_cast<float*>(a), const_cast<float*>(b),
                            const_cast<float*>(c), const_cast<float*>(d_skip),
                            const_cast<float*>(z), const_cast<float*>(delta_bias)};
    M1Params base = m1_params(dims, p, delta_softplus, 0);
    M1Params f = base, r = base;
    r.reverse = 1;
    if (summary) {
        f.z = r.z = nullptr;
        f.d_skip = r.d_skip = nullptr;
        f.last_state = last_fwd;
        f.dt_sum = dt_sum;
        r.last_state = last_bwd;
    } else {
        f.out = out;
        r.out = out;
        r.out_acc = 1;
        f.h0 = h0_fwd;
        r.h0 = h0_bwd;
    }
    size_t need = 0;
    if (!m1_lane_bidir_plan(f, &need))
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the two-phase form needs d_state <= 16 and len a multiple of 4");
    if (ws_bytes < need) return fail(ARM_SCAN_ERR_INVALID_DIMS, "workspace of %zu bytes, %zu needed", ws_bytes, need);
    cudaError_t e = m1_lane_bidir_phase(f, r, workspace, ws_bytes, summary, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorNotSupported)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the two-phase form needs 16-byte aligned tensors");
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "bidirectional phase launch");
}

int arm_scan_selective_scan_bidirectional_summary_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* delta_bias, int delta_softplus, void* workspace, size_t ws_bytes,
    float* last_fwd, float* last_bwd, float* dt_sum, void* stream) {
    return bidir_phase_common(dims, u, delta, a, b, c, nullptr, nullptr, delta_bias, delta_softplus,
                              workspace, ws_bytes, nullptr, last_fwd, last_bwd, dt_sum, nullptr, nullptr,
                              true, stream);
}

int arm_scan_selective_scan_bidirectional_finish_f32_async(
    const ArmScanDims* dims, const float* u, const float* delta, const float* a, const float* b,
    const float* c, const float* d_skip, const float* z, const float* delta_bias, int delta_softplus,
    void* workspace, size_t ws_bytes, const float* h0_fwd, const float* h0_bwd, float* out,
    void* stream) {
    return bidir_phase_common(dims, u, delta, a, b, c, d_skip, z, delta_bias, delta_softplus, workspace,
                              ws_bytes, out, nullptr, nullptr, nullptr, h0_fwd, h0_bwd, false, stream);
}

int arm_scan_selective_scan_ss2d_f32_async(
    const ArmScanDims* dims, size_t h, size_t w, const float* u, const float* delta,
    const float* a, const float* b, const float* c, const float* d_skip, const float* delta_bias,
    int delta_softplus, int merge_mean, float* out, void* stream) {
    if (!dims || !u || !delta || !a || !b || !c || !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    M1Counts cnt;
    int rc = m1_validate(dims, &cnt);
    if (rc) return rc;
    if (h == 0 || w == 0 || h * w != dims->len || dims->len / h != w)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "len %zu is not h %zu x w %zu", dims->len, h, w);
    if (dims->state > 16)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the SS2D entry covers d_state <= 16");
    if (dims->groups > 1 && (dims->dim / dims->groups) % 8 != 0)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE,
                    "the SS2D entry needs channels per B/C group to be a multiple of 8");
    if (w > 0x7fffffffu || dims->batch > 65535 || dims->dim > 65535u * 8)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "grid too large for the SS2D entry");
    std::vector<void*> p = {const_cast<float*>(u), const_cast<float*>(delta),
                            const_cast<float*>(a), const_cast<float*>(b),
                            const_cast<float*>(c), const_cast<float*>(d_skip),
                            nullptr, const_cast<float*>(delta_bias)};
    M1Params base = m1_params(dims, p, delta_softplus, 0);
    M1Params f = base, r = base;
    f.out = out;
    r.reverse = 1;
    r.out = nullptr;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = m1_bidir_sum_launch(f, r, 0, s);
    if (e != cudaSuccess) return cuda_fail(e, "SS2D row-major traversals");
    e = m1_ss2d_cols_launch(f, static_cast<int64_t>(h), static_cast<int64_t>(w), merge_mean ? 0.25f : 1.f, s);
    if (e == cudaErrorNotSupported)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the SS2D column kernels do not cover this shape");
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "SS2D column-major traversals");
}

int arm_scan_mamba3_scan_f32(const ArmMamba3Dims* dims, const float* q, const float* k,
                             const float* v, const float* adt, const float* dt, const float* trap,
                             const float* q_bias, const float* k_bias, const float* cos,
                             const float* sin, const float* d_skip, const float* z,
                             const float* mimo_psi, const float* mimo_zeta, const float* mimo_phi,
                             int reverse, int backend, int threading, float* out,
                             float* last_state, float* last_bx) {
    const void* req[] = {dims, q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, out};
    bool mimo = false;
    int rc = m3_check_ptrs(req, 12, last_state, last_bx, mimo_psi, mimo_zeta, mimo_phi, &mimo);
    if (rc) return rc;
    if ((rc = check_enums(backend, threading, true))) return rc;
    M3Counts cnt;
    if ((rc = m3_validate(dims, mimo, last_state, last_bx, &cnt))) return rc;
    std::vector<Buf> bufs = m3_bufs(cnt, dims, q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin,
                                    d_skip, z, mimo_psi, mimo_zeta, mimo_phi, out, last_state,
                                    last_bx);
    return run_sync(
        bufs,
        [&](const std::vector<void*>& p, cudaStream_t s) {
            return m3_run(m3_params(dims, p, reverse), backend, s);
        },
        backend == 3 ? tensor_status_code : nullptr);
}

int arm_scan_tensor_status(void) { return tensor_status_code(); }

int arm_scan_selective_scan_final_state_f32_async(const ArmScanDims* dims, const float* u,
                                                  const float* delta, const float* a,
                                                  const float* b, const float* c,
                                                  const float* delta_bias, int delta_softplus,
                                                  int reverse, const float* h0,
                                                  float* last_state, void* stream) {
    if (!dims || !u || !delta || !a || !b || !c || !last_state)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    M1Counts cnt;
    int rc = m1_validate(dims, &cnt);
    if (rc) return rc;
    if (dims->state > 16)
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE, "the final-state entry covers d_state <= 16");
    std::vector<void*> p = {const_cast<float*>(u), const_cast<float*>(delta), const_cast<float*>(a),
                            const_cast<float*>(b), const_cast<float*>(c),     nullptr,
                            nullptr,               const_cast<float*>(delta_bias)};
    M1Params m = m1_params(dims, p, delta_softplus, reverse);
    m.h0 = h0;
    m.last_state = last_state;
    cudaError_t e = m1_final_state_launch(m, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "final-state launch");
}

int arm_scan_selective_state_update_f32_async(const ArmScanDims* dims, float* state,
                                              const float* x, const float* dt, const float* a,
                                              const float* b, const float* c,
                                              const float* d_skip, const float* z,
                                              const float* dt_bias, int dt_softplus, float* out,
                                              void* stream) {
    if (!dims || !state || !x || !dt || !a || !b || !c || !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (!dims->batch || !dims->dim || !dims->state || !dims->groups)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "batch, dim, state and groups must be non-zero");
    if (dims->dim % dims->groups)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "dim (%zu) must be a multiple of groups (%zu)",
                    dims->dim, dims->groups);
    size_t bd = 0, bdn = 0;
    if (!mul3(dims->batch, dims->dim, 1, &bd) || !mul3(dims->batch, dims->dim, dims->state, &bdn))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    M1Params m{};
    m.u = x;
    m.delta = dt;
    m.A = a;
    m.B = b;
    m.C = c;
    m.d_skip = d_skip;
    m.z = z;
    m.delta_bias = dt_bias;
    m.out = out;
    m.batch = static_cast<int64_t>(dims->batch);
    m.dim = static_cast<int64_t>(dims->dim);
    m.len = 1;
    m.state = static_cast<int64_t>(dims->state);
    m.groups = static_cast<int64_t>(dims->groups);
    m.delta_softplus = dt_softplus != 0;
    cudaError_t e = m1_decode_launch(m, state, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "selective_state_update launch");
}

unsigned long long arm_scan_kernel_launches(void) { return b200scan::g_kernel_launches.load(); }

int arm_scan_set_device(int ordinal) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
    if (ordinal < -1 || (ordinal >= 0 && ordinal >= n))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "device ordinal %d outside [-1, %d)", ordinal, n);
    g_host_device = ordinal;
    return ARM_SCAN_OK;
}

int arm_scan_set_kernel_override(int knob, int value) {
    if (knob < 0 || knob >= b200scan::kKnobCount)
        return fail(ARM_SCAN_ERR_BAD_ENUM, "kernel override knob %d out of range", knob);
    if (value < 0) return fail(ARM_SCAN_ERR_BAD_ENUM, "kernel override value %d is negative", value);
    b200scan::g_override[knob].store(value, std::memory_order_relaxed);
    return ARM_SCAN_OK;
}

int arm_scan_mamba3_mixer_prologue_f32_async(const ArmMamba3MixerDims* dims, const float* proj,
                                             const float* dt_bias, const float* b_norm_weight,
                                             const float* c_norm_weight, float a_floor, float eps,
                                             float* z, float* x, float* q, float* k, float* dt,
                                             float* adt, float* trap, float* angles, void* stream) {
    const void* req[] = {dims, proj, dt_bias, b_norm_weight, c_norm_weight, z, x, q, k, dt, adt,
                         trap, angles};
    for (const void* r : req)
        if (!r) return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (!dims->heads || !dims->headdim || !dims->d_state || !dims->rank)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "heads, headdim, d_state and rank must be non-zero");
    if (dims->n_angles > dims->d_state / 2)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "n_angles (%zu) exceeds d_state / 2 (%zu)",
                    dims->n_angles, dims->d_state / 2);
    size_t hp = 0, rn = 0, rows = 0;
    if (!mul3(dims->heads, dims->headdim, 1, &hp) || !mul3(dims->rank, dims->d_state, 1, &rn) ||
        !mul3(dims->batch, dims->len, 1, &rows))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    const size_t w = 2 * hp + 2 * rn + 3 * dims->heads + dims->n_angles;
    size_t total = 0;
    if (!mul3(rows, w, 1, &total) || total > (size_t(1) << 62))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    b200scan::MixerParams m{};
    m.proj = proj;
    m.dt_bias = dt_bias;
    m.b_norm_w = b_norm_weight;
    m.c_norm_w = c_norm_weight;
    m.a_floor = a_floor;
    m.eps = eps;
    m.z = z;
    m.x = x;
    m.q = q;
    m.k = k;
    m.dt = dt;
    m.adt = adt;
    m.trap = trap;
    m.angles = angles;
    m.batch = static_cast<int64_t>(dims->batch);
    m.len = static_cast<int64_t>(dims->len);
    m.heads = static_cast<int64_t>(dims->heads);
    m.headdim = static_cast<int64_t>(dims->headdim);
    m.d_state = static_cast<int64_t>(dims->d_state);
    m.rank = static_cast<int64_t>(dims->rank);
    m.n_angles = static_cast<int64_t>(dims->n_angles);
    const cudaError_t e = b200scan::m3_mixer_prologue_launch(m, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "mamba3 mixer prologue launch");
}

int arm_scan_mamba3_siso_tc_async(const ArmMamba3Dims* dims, const ArmMamba3TcOptions* opts,
                                  const void* q, const void* k, const void* v, const float* adt,
                                  const float* dt, const float* trap, const float* q_bias,
                                  const float* k_bias, const void* angles, const float* d_skip,
                                  const void* z, int reverse, void* out, float* last_state,
                                  float* last_bx, void* stream) {
    if (!opts) return fail(ARM_SCAN_ERR_NULL_POINTER, "opts is null");
    const void* req[] = {dims, q, k, v, adt, dt, trap, q_bias, k_bias, out};
    bool mimo = false;
    int rc = m3_check_ptrs(req, 10, last_state, last_bx, nullptr, nullptr, nullptr, &mimo);
    if (rc) return rc;
    if (opts->n_angles > 0 && !angles)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "angles is null with n_angles > 0");
    auto is_dtype = [](int d) { return d == ARM_SCAN_DTYPE_F32 || d == ARM_SCAN_DTYPE_BF16; };
    if (!is_dtype(opts->in_dtype) || !is_dtype(opts->out_dtype))
        return fail(ARM_SCAN_ERR_BAD_ENUM, "dtype must be ARM_SCAN_DTYPE_F32 (0) or _BF16 (1)");
    if (opts->out_layout != 0 && opts->out_layout != 1)
        return fail(ARM_SCAN_ERR_BAD_ENUM, "out_layout must be 0 or 1, got %d", opts->out_layout);
    if (opts->angles_shared != 0 && opts->angles_shared != 1)
        return fail(ARM_SCAN_ERR_BAD_ENUM, "angles_shared must be 0 or 1, got %d", opts->angles_shared);
    M3Counts cnt;
    if ((rc = m3_validate(dims, false, last_state, last_bx, &cnt))) return rc;
    if (dims->rank != 1)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "the tensor-core entry is SISO (rank 1)");
    if (opts->n_angles > dims->dqk / 2)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "n_angles (%zu) exceeds dqk/2 (%zu)", opts->n_angles,
                    dims->dqk / 2);
    std::vector<void*> p = {
        const_cast<void*>(q),        const_cast<void*>(k),        const_cast<void*>(v),
        const_cast<float*>(adt),     const_cast<float*>(dt),      const_cast<float*>(trap),
        const_cast<float*>(q_bias),  const_cast<float*>(k_bias),  nullptr,
        nullptr,                     const_cast<float*>(d_skip),  const_cast<void*>(z),
        nullptr,                     nullptr,                     nullptr,
        out,                         last_state,                  last_bx};
    M3Params m = m3_params(dims, p, reverse);
    m.angles = angles;
    m.n_angles = static_cast<int64_t>(opts->n_angles);
    m.angles_shared = opts->angles_shared;
    m.in_bf16 = opts->in_dtype == ARM_SCAN_DTYPE_BF16;
    m.out_bf16 = opts->out_dtype == ARM_SCAN_DTYPE_BF16;
    m.out_blh = opts->out_layout;
    if (!m3_tc_angles_applicable(m))
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE,
                    "the tensor-core entry covers dqk 128, dv 64 with 16-byte aligned q/k/v/z/out "
                    "and biases");
    cudaError_t e = m3_tc_launch(m, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "mamba3_siso_tc launch");
}

int arm_scan_mamba3_mimo_x_tc_async(const ArmMamba3Dims* dims, const ArmMamba3TcOptions* opts,
                                    const void* x, const void* b, const void* c, const float* adt,
                                    const float* dt, const float* trap, const float* angles,
                                    const float* d_skip, int reverse, void* out, float* last_state,
                                    void* stream) {
    if (!dims || !opts || !x || !b || !c || !adt || !dt || !trap || !out)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (opts->n_angles > 0 && !angles)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "angles is null with n_angles > 0");
    auto is_dtype = [](int d) { return d == ARM_SCAN_DTYPE_F32 || d == ARM_SCAN_DTYPE_BF16; };
    if (!is_dtype(opts->in_dtype) || !is_dtype(opts->out_dtype))
        return fail(ARM_SCAN_ERR_BAD_ENUM, "dtype must be ARM_SCAN_DTYPE_F32 (0) or _BF16 (1)");
    if (opts->angles_shared != 0 && opts->angles_shared != 1)
        return fail(ARM_SCAN_ERR_BAD_ENUM, "angles_shared must be 0 or 1, got %d", opts->angles_shared);
    if (!dims->batch || !dims->heads || !dims->dv || !dims->dqk || !dims->len || !dims->rank)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "a dimension is zero");
    if (dims->dqk % 2) return fail(ARM_SCAN_ERR_INVALID_DIMS, "dqk must be even");
    if (opts->n_angles > dims->dqk / 2)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "n_angles (%zu) exceeds dqk/2 (%zu)", opts->n_angles,
                    dims->dqk / 2);
    size_t n1 = 0, n2 = 0;
    if (!mul4(dims->batch, dims->len, dims->heads, dims->dv, &n1) || !mul_ok(n1, dims->rank, &n2) ||
        n2 > (SIZE_MAX >> 3) / 4)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "element counts overflow");
    M3Params m{};
    m.q = static_cast<const float*>(c);
    m.k = static_cast<const float*>(b);
    m.v = static_cast<const float*>(x);
    m.adt = adt;
    m.dt = dt;
    m.trap = trap;
    m.d_skip = d_skip;
    m.out = static_cast<float*>(out);
    m.last_state = last_state;
    m.batch = static_cast<int64_t>(dims->batch);
    m.heads = static_cast<int64_t>(dims->heads);
    m.dv = static_cast<int64_t>(dims->dv);
    m.dqk = static_cast<int64_t>(dims->dqk);
    m.len = static_cast<int64_t>(dims->len);
    m.rank = static_cast<int64_t>(dims->rank);
    m.reverse = reverse ? 1 : 0;
    m.in_bf16 = opts->in_dtype == ARM_SCAN_DTYPE_BF16;
    m.out_bf16 = opts->out_dtype == ARM_SCAN_DTYPE_BF16;
    m.x_per_rank = 1;
    if (!m3_tc_xr_applicable(m))
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE,
                    "the per-rank MIMO entry covers rank 2 or 4, dqk 128, dv 64 and batch*heads <= 65535");
    cudaError_t e = m3_tc_launch_xr(m, angles, static_cast<int64_t>(opts->n_angles), opts->angles_shared,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "mamba3_mimo_x_tc launch");
}

int arm_scan_mamba3_scan_f32_async(const ArmMamba3Dims* dims, const float* q, const float* k,
                                   const float* v, const float* adt, const float* dt,
                                   const float* trap, const float* q_bias, const float* k_bias,
                                   const float* cos, const float* sin, const float* d_skip,
                                   const float* z, const float* mimo_psi, const float* mimo_zeta,
                                   const float* mimo_phi, int reverse, int backend, int threading,
                                   float* out, float* last_state, float* last_bx, void* stream) {
    const void* req[] = {dims, q, k, v, adt, dt, trap, q_bias, k_bias, cos, sin, out};
    bool mimo = false;
    int rc = m3_check_ptrs(req, 12, last_state, last_bx, mimo_psi, mimo_zeta, mimo_phi, &mimo);
    if (rc) return rc;
    if ((rc = check_enums(backend, threading, true))) return rc;
    M3Counts cnt;
    if ((rc = m3_validate(dims, mimo, last_state, last_bx, &cnt))) return rc;
    std::vector<void*> p = {
        const_cast<float*>(q),      const_cast<float*>(k),         const_cast<float*>(v),
        const_cast<float*>(adt),    const_cast<float*>(dt),        const_cast<float*>(trap),
        const_cast<float*>(q_bias), const_cast<float*>(k_bias),    const_cast<float*>(cos),
        const_cast<float*>(sin),    const_cast<float*>(d_skip),    const_cast<float*>(z),
        const_cast<float*>(mimo_psi), const_cast<float*>(mimo_zeta), const_cast<float*>(mimo_phi),
        out,                        last_state,                    last_bx};
    return m3_run(m3_params(dims, p, reverse), backend, static_cast<cudaStream_t>(stream));
}

size_t arm_scan_mamba3_angles_workspace_bytes(const ArmMamba3Dims* dims, size_t n_angles) {
    if (!dims) return 0;
    return angle_workspace_bytes(static_cast<int64_t>(dims->batch),
                                 static_cast<int64_t>(dims->heads),
                                 static_cast<int64_t>(dims->len), static_cast<int64_t>(n_angles));
}

int arm_scan_mamba3_angles_f32_async(const ArmMamba3Dims* dims, const float* angles,
                                     size_t n_angles, const float* dt, float* cos, float* sin,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    if (!dims || !angles || !dt || !cos || !sin || !workspace)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (!dims->batch || !dims->heads || !dims->len || !dims->dqk || !n_angles)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "a dimension is zero");
    if (dims->dqk % 2 || n_angles > dims->dqk / 2 || dims->dqk > 256)
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "n_angles (%zu) must be <= dqk/2 with dqk (%zu) even and <= 256", n_angles,
                    dims->dqk);
    if (dims->batch * dims->heads > 65535)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "batch*heads above 65535");
    if ((dims->len + 127) / 128 > static_cast<size_t>(INT32_MAX))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "len %zu: more 128-step chunks than a grid holds", dims->len);
    const size_t need = arm_scan_mamba3_angles_workspace_bytes(dims, n_angles);
    if (workspace_bytes < need)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "workspace of %zu bytes, %zu needed",
                    workspace_bytes, need);
    AngleParams a{angles, dt, cos, sin, static_cast<int64_t>(dims->batch),
                  static_cast<int64_t>(dims->heads), static_cast<int64_t>(dims->len),
                  static_cast<int64_t>(n_angles), static_cast<int64_t>(dims->dqk / 2)};
    cudaError_t e = angle_launch(a, static_cast<float*>(workspace),
                                 static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "angle pre-pass launch");
}

// Traversals of a token grid (len / grid_w rows of grid_w tokens, row-major)
// summed into out (batch, len, heads, dv): the row-major ordering and, with
// both_orders, the column-major one, each forward and reverse, the angle
// pre-pass per ordering (reading the grid in place); with noncausal the
// diagonal term is subtracted once per ordering.  angles (n_angles > 0) or,
// for a single row-major ordering, cos / sin.
static int m3_grid_sum(const ArmMamba3Dims* dims, size_t grid_w, bool both_orders, bool noncausal,
                       const float* q, const float* k, const float* v, const float* adt,
                       const float* dt, const float* trap, const float* q_bias,
                       const float* k_bias, const float* angles, size_t n_angles,
                       const float* cos_in, const float* sin_in, const float* d_skip,
                       const float* z, float* out, void* stream) {
    const void* req[] = {dims, q, k, v, adt, dt, trap, q_bias, k_bias, out};
    bool mimo = false;
    int rc = m3_check_ptrs(req, 10, nullptr, nullptr, nullptr, nullptr, nullptr, &mimo);
    if (rc) return rc;
    M3Counts cnt;
    if ((rc = m3_validate(dims, false, nullptr, nullptr, &cnt))) return rc;
    if (dims->rank != 1) return fail(ARM_SCAN_ERR_INVALID_DIMS, "the grid entries are SISO (rank 1)");
    if (!grid_w || dims->len % grid_w)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "len (%zu) must be a multiple of grid_w (%zu)",
                    dims->len, grid_w);
    const bool trig_given = cos_in && sin_in;
    if (!trig_given) {
        if (!angles) return fail(ARM_SCAN_ERR_NULL_POINTER, "angles (or cos and sin) are required");
        if (!n_angles || n_angles > dims->dqk / 2)
            return fail(ARM_SCAN_ERR_INVALID_DIMS, "n_angles (%zu) must be in [1, dqk/2]", n_angles);
    } else if (both_orders) {
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "cos/sin serve one ordering; pass raw angles for 2D");
    }
    if (dims->batch * dims->heads > 65535)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "batch*heads above 65535");
    if ((dims->len + 127) / 128 > static_cast<size_t>(INT32_MAX))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "len %zu: more 128-step chunks than a grid holds", dims->len);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::vector<void*> p = {const_cast<float*>(q),      const_cast<float*>(k),
                            const_cast<float*>(v),      const_cast<float*>(adt),
                            const_cast<float*>(dt),     const_cast<float*>(trap),
                            const_cast<float*>(q_bias), const_cast<float*>(k_bias),
                            nullptr,                    nullptr,
                            const_cast<float*>(d_skip), const_cast<float*>(z),
                            nullptr,                    nullptr,
                            nullptr,                    out,
                            nullptr,                    nullptr};
    M3Params base = m3_params(dims, p, 0);
    base.grid_w = static_cast<int64_t>(grid_w);
    base.out_blh = 1;
    base.out_acc = 1;
    if (!m3_chunk_applicable(base))
        return fail(ARM_SCAN_ERR_BACKEND_UNAVAILABLE,
                    "the grid entries cover dv <= 128, dqk <= 128 with 16-byte aligned v, z, out");
    const int orders = both_orders ? 2 : 1;
    const size_t cs = cnt.blhr;  // floats of one cos (or sin) array
    const size_t ws_angle = trig_given ? 0 : arm_scan_mamba3_angles_workspace_bytes(dims, n_angles);
    cudaMemPool_t pool = nullptr;
    cudaError_t e = device_workspace_pool(&pool);
    if (e != cudaSuccess) return cuda_fail(e, "workspace pool");
    void* raw = nullptr;
    const size_t trig_floats = trig_given ? 0 : 2 * orders * cs;
    e = cudaMallocFromPoolAsync(&raw, trig_floats * sizeof(float) + ws_angle + 256, pool, s);
    if (e != cudaSuccess) return cuda_fail(e, "workspace");
    float* trig = static_cast<float*>(raw);  // [ordering][cos, sin]
    float* angle_ws = trig + trig_floats;
    e = cudaMemsetAsync(out, 0, cnt.blhv * sizeof(float), s);
    for (int col = 0; col < orders && e == cudaSuccess; ++col) {
        const float* cosv = cos_in;
        const float* sinv = sin_in;
        if (!trig_given) {
            float* c = trig + (2 * col) * cs;
            float* sn = c + cs;
            AngleParams a{angles, dt, c, sn, static_cast<int64_t>(dims->batch),
                          static_cast<int64_t>(dims->heads), static_cast<int64_t>(dims->len),
                          static_cast<int64_t>(n_angles), static_cast<int64_t>(dims->dqk / 2),
                          static_cast<int64_t>(grid_w), col};
            e = angle_launch(a, angle_ws, s);
            cosv = c;
            sinv = sn;
        }
        for (int rev = 0; rev < 2 && e == cudaSuccess; ++rev) {
            M3Params m = base;
            m.cos = cosv;
            m.sin = sinv;
            m.col_major = col;
            m.reverse = rev;
            e = m3_chunk_launch(m, s);
        }
    }
    if (e == cudaSuccess && noncausal) e = m3_diag_sub_launch(base, orders, s);
    const cudaError_t ef = cudaFreeAsync(raw, s);
    if (e == cudaSuccess) e = ef;
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "mamba3 grid traversals launch");
}

int arm_scan_mamba3_ss2d_f32_async(const ArmMamba3Dims* dims, size_t grid_w, const float* q,
                                   const float* k, const float* v, const float* adt,
                                   const float* dt, const float* trap, const float* q_bias,
                                   const float* k_bias, const float* angles, size_t n_angles,
                                   const float* d_skip, const float* z, float* out, void* stream) {
    if (!angles) return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    return m3_grid_sum(dims, grid_w, true, false, q, k, v, adt, dt, trap, q_bias, k_bias, angles,
                       n_angles, nullptr, nullptr, d_skip, z, out, stream);
}

int arm_scan_mamba3_noncausal_f32_async(const ArmMamba3Dims* dims, size_t grid_w, const float* q,
                                        const float* k, const float* v, const float* adt,
                                        const float* dt, const float* trap, const float* q_bias,
                                        const float* k_bias, const float* angles, size_t n_angles,
                                        const float* cos, const float* sin, const float* d_skip,
                                        const float* z, float* out, void* stream) {
    if ((cos == nullptr) != (sin == nullptr))
        return fail(ARM_SCAN_ERR_NULL_POINTER, "cos and sin must be given together");
    const bool two_d = dims && grid_w != 0 && grid_w != dims->len;
    return m3_grid_sum(dims, grid_w ? grid_w : (dims ? dims->len : 0), two_d, true, q, k, v, adt, dt,
                       trap, q_bias, k_bias, cos ? nullptr : angles, n_angles, cos, sin, d_skip, z,
                       out, stream);
}

int arm_scan_mamba3_angles_f32_noalloc(const ArmMamba3Dims* dims, const float* angles,
                                       size_t n_angles, const float* dt, float* cos, float* sin,
                                       void* stream) {
    if (!dims || !angles || !dt || !cos || !sin)
        return fail(ARM_SCAN_ERR_NULL_POINTER, "a required pointer is null");
    if (!dims->batch || !dims->heads || !dims->len || !dims->dqk || !n_angles)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "a dimension is zero");
    if (dims->dqk % 2 || n_angles > dims->dqk / 2 || dims->dqk > 256)
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "n_angles (%zu) must be <= dqk/2 with dqk (%zu) even and <= 256", n_angles,
                    dims->dqk);
    if (dims->batch * dims->heads > 65535)
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "batch*heads above 65535");
    if ((dims->len + 127) / 128 > static_cast<size_t>(INT32_MAX))
        return fail(ARM_SCAN_ERR_INVALID_DIMS, "len %zu: more 128-step chunks than a grid holds", dims->len);
    AngleParams a{angles, dt, cos, sin, static_cast<int64_t>(dims->batch),
                  static_cast<int64_t>(dims->heads), static_cast<int64_t>(dims->len),
                  static_cast<int64_t>(n_angles), static_cast<int64_t>(dims->dqk / 2)};
    bool too_big = false;
    cudaError_t e = angle_noalloc_launch(a, static_cast<cudaStream_t>(stream), &too_big);
    if (too_big)
        return fail(ARM_SCAN_ERR_INVALID_DIMS,
                    "problem needs %zu bytes of scratch; the built-in scratch holds %lld bytes "
                    "(use arm_scan_mamba3_angles_f32_async with a workspace)",
                    arm_scan_mamba3_angles_workspace_bytes(dims, n_angles),
                    static_cast<long long>(kAngleNoAllocMaxFloats * 4));
    return e == cudaSuccess ? ARM_SCAN_OK : cuda_fail(e, "allocation-free angle pre-pass");
}

}  // extern "C"
