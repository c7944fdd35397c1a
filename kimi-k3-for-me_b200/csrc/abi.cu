// abi.cu -- status reporting, the expert-bank layout helper and the host n-gram drafter.
#include <string.h>

#include "common.cuh"

namespace k3 {
thread_local int g_last_cuda_error = 0;
__device__ unsigned int g_device_status = 0;
std::atomic<long long> g_launches{0};
}  // namespace k3

extern "C" long long k3gpu_launch_count(void) { return k3::g_launches.load(std::memory_order_relaxed); }

extern "C" const char *k3gpu_strerror(int status)
{
    switch (status) {
    case K3GPU_OK: return "ok";
    case K3GPU_EINVAL: return "invalid argument (null pointer, size out of range or misaligned)";
    case K3GPU_ECAPACITY: return "capacity exceeded (workspace, log or cache too small)";
    case K3GPU_ECUDA: return "CUDA runtime error (see k3gpu_last_cuda_error)";
    case K3GPU_EDEVICE: return "device-side check failed (see k3gpu_device_status)";
    case K3GPU_ECALLBACK: return "a caller-supplied callback failed";
    default: return "unknown status";
    }
}

extern "C" int k3gpu_last_cuda_error(void) { return k3::g_last_cuda_error; }

extern "C" int k3gpu_version(void) { return 100; }  // 0.1.0

extern "C" int k3gpu_device_status(int device, int *status_out)
{
    if (!status_out) return K3GPU_EINVAL;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return k3::cuda_status(e);
    if ((e = cudaSetDevice(device)) != cudaSuccess) return k3::cuda_status(e);
    unsigned int v = 0, zero = 0;
    e = cudaMemcpyFromSymbol(&v, k3::g_device_status, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(k3::g_device_status, &zero, sizeof(zero));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return k3::cuda_status(e);
    *status_out = (int)v;
    return K3GPU_OK;
}

extern "C" void k3gpu_bank_layout(K3GpuExpertBank *b, int L, int I)
{
    if (!b) return;
    const int64_t pw = (int64_t)I * (L / 2), sw = (int64_t)I * (L / 32);
    const int64_t pd = (int64_t)L * (I / 2), sd = (int64_t)L * (I / 32);
    // w1.packed w1.scale w2.packed w2.scale w3.packed w3.scale, one contiguous run
    b->p1 = 0;
    b->s1 = pw;
    b->p2 = pw + sw;
    b->s2 = pw + sw + pd;
    b->p3 = pw + sw + pd + sd;
    b->s3 = pw + sw + pd + sd + pw;
    const int64_t run = pw + sw + pd + sd + pw + sw;
    // runs start on a whole row of both tensor-map pitches (L/2 and I/2 bytes) and on a
    // 256-byte boundary: stride = run rounded up to lcm(L/2, I/2, 256)
    auto gcd = [](int64_t a, int64_t c) { while (c) { const int64_t r = a % c; a = c; c = r; } return a; };
    int64_t q = 256;
    for (int64_t v : {(int64_t)L / 2, (int64_t)I / 2})
        if (v > 0) q = q / gcd(q, v) * v;
    b->stride = (run + q - 1) / q * q;
    b->L = L;
    b->I = I;
}

// The reference's spec_draft (src/cli/k3_run.c:450-491): match the last n ids (n from
// nmax down to nmin) against earlier positions, newest first; take the two most recent
// matches; propose what followed the newest while the older one agrees and has not run
// into the newest; return at the first n that drafts anything.
extern "C" int k3_spec_draft_ngram(const int *seq, int T, int cap, int nmax, int nmin, int *out)
{
    if (!seq || !out || cap <= 0 || nmin < 1 || nmax < nmin) return 0;
    for (int n = nmax; n >= nmin; n--) {
        if (T < n + 1) continue;
        const int *suf = seq + T - n;
        int newest = -1, older = -1;
        for (int j = T - n - 1; j >= 0; j--) {
            if (memcmp(seq + j, suf, (size_t)n * sizeof(int)) != 0) continue;
            if (newest < 0) {
                newest = j;
            } else {
                older = j;
                break;
            }
        }
        if (newest < 0) continue;
        int nd = 0;
        for (int i = 0; nd < cap && newest + n + i < T; i++) {
            const int cand = seq[newest + n + i];
            if (older >= 0 && (older + n + i >= newest || seq[older + n + i] != cand)) break;
            out[nd++] = cand;
        }
        if (nd > 0) return nd;
    }
    return 0;
}
