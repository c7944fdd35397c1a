// common.cuh -- shared helpers of libk3gpu.so: status plumbing, launch checks, the
// device status word, and exact-arithmetic helpers the kernels share.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "k3gpu.h"

namespace k3 {

// The cudaError_t behind the last K3GPU_ECUDA of this thread.
extern thread_local int g_last_cuda_error;

// Device status word: kernels OR a code in when they skip an out-of-range access, so the
// host can tell a silent skip from a clean run (k3gpu_device_status).
extern __device__ unsigned int g_device_status;

enum : unsigned int {
    DEV_BAD_INDEX = 1u,     // an expert index or row index outside its range was skipped
    DEV_BAD_COUNT = 2u,     // a commit length outside 0..T was clamped
    DEV_BAD_POSITION = 4u,  // a cache position outside 0..cap-1 was skipped
    DEV_TIMEOUT = 8u,       // a bounded wait on a pipeline barrier gave up
};

inline __device__ void flag(unsigned int code) { atomicOr(&g_device_status, code); }

inline int cuda_status(cudaError_t e)
{
    if (e == cudaSuccess) return K3GPU_OK;
    g_last_cuda_error = (int)e;
    return K3GPU_ECUDA;
}

// Kernels this process has enqueued through the library (k3gpu_launch_count).
extern std::atomic<long long> g_launches;

// Check the launch just enqueued (configuration errors surface here, not at sync); every
// kernel launch of the library is followed by this call, which also counts it.
inline int launch_status()
{
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cuda_status(cudaGetLastError());
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// 1 / (1 + exp(-v)) in float with a correctly rounded exp: the double exp of CUDA's
// libdevice is within 1 ulp of double, so rounding it to float gives the correctly
// rounded float result except within 2^-29 of a rounding midpoint.
inline __device__ float sigmoid_cr(float v)
{
    const float e = __double2float_rn(exp(-(double)v));
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

inline __device__ float expf_cr(float v) { return __double2float_rn(exp((double)v)); }

// Round-to-nearest float ops that the compiler may not contract into an FMA: the
// reference is compiled with -ffp-contract=off, and the bit-exact kernels mirror it.
inline __device__ float fmul(float a, float b) { return __fmul_rn(a, b); }
inline __device__ float fadd(float a, float b) { return __fadd_rn(a, b); }
inline __device__ float fsub(float a, float b) { return __fsub_rn(a, b); }

}  // namespace k3
