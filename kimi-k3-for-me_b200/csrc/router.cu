// router.cu -- the MoE router (k3_router, src/core/k3_ops.c:1624-1719 of the reference)
// for a whole verify batch.
//
// Scores: every (token, expert) score is ONE double chain over i = 0..hidden-1, in order,
// inside one thread -- the reference's chain (its 8-expert blocking changes issue order
// only). A float times a float is exact in double, so fma(w, x, acc) == acc + w*x rounded
// once, exactly the reference's `acc += (double)w * (double)x`. The chain length sets the
// floor (hidden dependent FMAs), so the kernel's job is to keep every chain issuing: a CTA
// owns 24 experts x 8 tokens (one chain per thread), K tiles of 128 columns arrive by
// cp.async two tiles ahead, and each tile is widened to double once in shared memory.
// Measured on B200 the loop runs at about 20 clocks a step against the 8-clock FMA
// latency: each warp-step moves four shared-memory wavefronts (operands re-read by the
// lanes that share an expert or token), and the float-to-double widening is slow. Register
// blocking over tokens and a widened copy made once per call are the way down.
//
// Selection: one warp per token, repeated max with the first-index tie rule, taken
// entries set to -inf, weights from the unbiased scores, renormalised by one double sum
// in slot order -- the reference's loop, made warp-parallel only in the comparisons,
// which are exact.
#include <math.h>

#include <mutex>

#include <cuda.h>

#include "common.cuh"

namespace k3 {

constexpr int RT_E = 24;     // experts per CTA (384 experts x 72 tokens -> 144 CTAs)
constexpr int RT_T = 8;      // tokens per CTA
constexpr int RT_R = RT_E + RT_T;
constexpr int RT_THREADS = RT_E * RT_T;   // one chain per thread
constexpr int RT_K = 128;    // hidden columns per tile
constexpr int RT_NS = 3;     // cp.async stages (float tiles in flight)
constexpr int RT_LD = RT_K + 2;   // double tile row stride: rows land on distinct banks
constexpr int RT_F_TILE = RT_R * RT_K;                      // floats per stage
constexpr int RT_SMEM = RT_NS * RT_F_TILE * 4 + 2 * RT_R * RT_LD * 8;

// one cp.async of V floats (V = 4: 16 bytes; V = 1: 4 bytes), zero-filled when !valid
template <int V>
__device__ __forceinline__ void cp_async_f(float *dst, const float *src, bool valid)
{
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    const int n = valid ? 4 * V : 0;
    if (V == 4)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

// eight chain steps from registers: acc += w[i] * x[i], i = 0..7 in order
__device__ __forceinline__ double chain8(double acc, const double2 (&w)[4], const double2 (&x)[4])
{
#pragma unroll
    for (int i = 0; i < 4; i++) {
        asm volatile("fma.rn.f64 %0, %1, %2, %0;" : "+d"(acc) : "d"(w[i].x), "d"(x[i].x));
        asm volatile("fma.rn.f64 %0, %1, %2, %0;" : "+d"(acc) : "d"(w[i].y), "d"(x[i].y));
    }
    return acc;
}

__device__ __forceinline__ void load8(double2 (&w)[4], double2 (&x)[4], const double *wr, const double *xr)
{
    const uint32_t ws = (uint32_t)__cvta_generic_to_shared(wr), xs = (uint32_t)__cvta_generic_to_shared(xr);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(w[i].x), "=d"(w[i].y) : "r"(ws + 16 * i));
        asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(x[i].x), "=d"(x[i].y) : "r"(xs + 16 * i));
    }
}

template <int V>   // V = 4 when hidden % 4 == 0 and x, W are 16-byte aligned, else 1
__global__ void __launch_bounds__(RT_THREADS) router_scores_kernel(float *__restrict__ score,
                                                                   const float *__restrict__ x,
                                                                   const float *__restrict__ W,
                                                                   int T, int hidden, int n)
{
    extern __shared__ __align__(16) unsigned char rsm[];
    float *fst = reinterpret_cast<float *>(rsm);                            // [NS][R][K]
    double *dt = reinterpret_cast<double *>(rsm + RT_NS * RT_F_TILE * 4);   // [2][R][LD]
    const int e0 = blockIdx.x * RT_E, t0 = blockIdx.y * RT_T;
    const int tid = threadIdx.x;
    const int tl = tid & 7;          // token of this thread's chain
    const int el = tid >> 3;         // expert of this thread's chain
    const int nt = (hidden + RT_K - 1) / RT_K;
    constexpr int CPR = RT_K / V;    // copies per tile row

    auto issue = [&](int kt) {
        if (kt < nt) {
            float *f = fst + (kt % RT_NS) * RT_F_TILE;
            const int k0 = kt * RT_K;
            for (int i = tid; i < RT_R * CPR; i += RT_THREADS) {
                const int r = i / CPR, c = (i % CPR) * V;
                const bool is_w = r < RT_E;
                const int row = is_w ? e0 + r : t0 + (r - RT_E);
                const bool ok = (is_w ? row < n : row < T) && k0 + c < hidden;
                const float *src = is_w ? W : x;
                if (ok) src += (size_t)row * hidden + k0 + c;
                cp_async_f<V>(f + r * RT_K + c, src, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int kt = 0; kt < RT_NS - 1; kt++) issue(kt);

    double acc = 0.0;
    for (int kt = 0; kt < nt; kt++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(RT_NS - 2) : "memory");
        __syncthreads();                       // tile kt landed for every thread's copies
        issue(kt + RT_NS - 1);                 // into the stage tile kt-1 used
        const float *f = fst + (kt % RT_NS) * RT_F_TILE;
        double *d = dt + (kt & 1) * RT_R * RT_LD;
        for (int i = tid; i < RT_F_TILE / 4; i += RT_THREADS) {   // widen once, 4 at a time
            const float4 v = reinterpret_cast<const float4 *>(f)[i];
            double *o = d + (i / (RT_K / 4)) * RT_LD + (i % (RT_K / 4)) * 4;
            reinterpret_cast<double2 *>(o)[0] = make_double2(v.x, v.y);
            reinterpret_cast<double2 *>(o)[1] = make_double2(v.z, v.w);
        }
        __syncthreads();
        const double *wr = d + el * RT_LD;
        const double *xr = d + (RT_E + tl) * RT_LD;
        const int kn = min(RT_K, hidden - kt * RT_K);
        if (kn == RT_K) {
            double2 wa[4], xa[4], wb[4], xb[4];
            load8(wa, xa, wr, xr);
#pragma unroll
            for (int c = 0; c < RT_K; c += 16) {
                load8(wb, xb, wr + c + 8, xr + c + 8);
                acc = chain8(acc, wa, xa);
                if (c + 16 < RT_K) load8(wa, xa, wr + c + 16, xr + c + 16);
                acc = chain8(acc, wb, xb);
            }
        } else {
            for (int c = 0; c < kn; c++) acc = fma(wr[c], xr[c], acc);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    const int t = t0 + tl, e = e0 + el;
    if (t < T && e < n) score[(size_t)t * n + e] = sigmoid_cr(__double2float_rn(acc));
}

// One warp per token; scores [T][n] -> idx/w [T][topk]. Each lane keeps the selection
// scores of experts lane, lane+32, ... in registers (n <= 1024).
__global__ void __launch_bounds__(128) router_topk_kernel(int *__restrict__ idx,
                                                          float *__restrict__ wout,
                                                          const float *__restrict__ score,
                                                          const float *__restrict__ bias,
                                                          int T, int n, int topk, int renorm,
                                                          float routed_scale)
{
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (t >= T) return;
    const float *st = score + (size_t)t * n;
    float ch[32];
#pragma unroll
    for (int r = 0; r < 32; r++) {
        const int e = lane + 32 * r;
        ch[r] = e < n ? __fadd_rn(st[e], bias ? bias[e] : 0.0f) : -INFINITY;
    }
    float wsel[64];
    int isel[64];
    for (int j = 0; j < topk; j++) {
        // lane-local best: strict > in ascending expert order keeps the first index
        float bv = -INFINITY;
        int be = -1;
#pragma unroll
        for (int r = 0; r < 32; r++) {
            if (ch[r] > bv) { bv = ch[r]; be = lane + 32 * r; }
        }
        // warp argmax, ties to the smaller index, "no candidate" (-1) loses to anything
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oe = __shfl_xor_sync(0xffffffffu, be, off);
            const bool take = oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be));
            if (take) { bv = ov; be = oe; }
        }
        if (be < 0) {
            isel[j] = 0;
            wsel[j] = 0.0f;
            continue;
        }
        isel[j] = be;
        wsel[j] = st[be];                       // UNBIASED score
        if ((be & 31) == lane) {
#pragma unroll
            for (int r = 0; r < 32; r++)
                if (lane + 32 * r == be) ch[r] = -INFINITY;
        }
    }
    if (lane == 0) {
        if (renorm && topk > 1) {
            double s = 0.0;
            for (int j = 0; j < topk; j++) s += (double)wsel[j];
            const float inv = __double2float_rn(1.0 / (s + 1e-20));
            for (int j = 0; j < topk; j++) wsel[j] = __fmul_rn(wsel[j], inv);
        }
        for (int j = 0; j < topk; j++) {
            idx[(size_t)t * topk + j] = isel[j];
            wout[(size_t)t * topk + j] = __fmul_rn(wsel[j], routed_scale);
        }
    }
}

// The opt-in to more than 48 KB of dynamic shared memory, once per device and variant.
static int router_smem_optin(bool v4)
{
    static std::mutex mu;
    static bool done[64][2] = {};
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev][v4]) {
        st = cuda_status(v4 ? cudaFuncSetAttribute(router_scores_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM)
                            : cudaFuncSetAttribute(router_scores_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM));
        if (st) return st;
        done[dev][v4] = true;
    }
    return K3GPU_OK;
}

int router_launch(int *idx, float *w, const float *x, const float *W, const float *bias, int T,
                  int hidden, int n, int topk, int renorm, float routed_scale, float *score,
                  cudaStream_t s)
{
    dim3 g1(ceil_div(n, RT_E), ceil_div(T, RT_T));
    const bool v4 = hidden % 4 == 0 && ((uintptr_t)x & 15u) == 0 && ((uintptr_t)W & 15u) == 0;
    int st0 = router_smem_optin(v4);
    if (st0) return st0;
    if (v4) router_scores_kernel<4><<<g1, RT_THREADS, RT_SMEM, s>>>(score, x, W, T, hidden, n);
    else router_scores_kernel<1><<<g1, RT_THREADS, RT_SMEM, s>>>(score, x, W, T, hidden, n);
    int st = launch_status();
    if (st) return st;
    router_topk_kernel<<<ceil_div(T, 4), 128, 0, s>>>(idx, w, score, bias, T, n, topk, renorm,
                                                      routed_scale);
    return launch_status();
}

}  // namespace k3

// ---- the allocation-free router (k3gpu_router_noalloc) ------------------------------
// Callers that cannot allocate device memory (their allocator owns the HBM, or they run
// where cudaMalloc's possible device synchronisation is forbidden) get the score scratch
// from this fixed array instead of a workspace. Every GPU that loads the library holds
// one copy (2 MiB) until the process exits.
namespace k3 {
static __device__ __align__(256) float g_router_noalloc_scores[K3GPU_ROUTER_NOALLOC_MAX_SCORES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static float *g_noalloc_addr[NOALLOC_MAX_DEVICES] = {};
static unsigned long long g_noalloc_ctx[NOALLOC_MAX_DEVICES] = {};   // context id of each lookup

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

// The id of the current context (cuCtxGetId, through the runtime's driver entry points), or
// 0 when it cannot be read. A device reset replaces the primary context, and with it the
// array's address, so the id tells a stale lookup from a valid one.
static unsigned long long current_ctx_id()
{
    static CtxGetCurrentFn get_cur = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (!get_cur || !get_id || get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// In host code the array's name is only a host-side stand-in, not a device address, so
// the kernels get the address cudaGetSymbolAddress returns for the current device. The
// lookup is the per-device set-up, done by the first call on each device -- and again by
// the first call after that device's context was replaced (a cudaDeviceReset), whose
// module, and so the array, has a new address.
static int noalloc_scores(float **out)
{
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return K3GPU_EINVAL;
    // (0 when no context is current on this thread yet: the lookup below makes it current
    // and records its id, so at most one extra lookup follows)
    const unsigned long long ctx = current_ctx_id();
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev] || g_noalloc_ctx[dev] != ctx) {
        void *p = nullptr;
        st = cuda_status(cudaGetSymbolAddress(&p, g_router_noalloc_scores));
        if (st) return st;
        g_noalloc_addr[dev] = static_cast<float *>(p);
        g_noalloc_ctx[dev] = current_ctx_id();
    }
    *out = g_noalloc_addr[dev];
    return K3GPU_OK;
}
}  // namespace k3

extern "C" int k3gpu_router_noalloc(int *idx, float *w, const float *x, const float *W,
                                    const float *bias, int T, int hidden, int n_experts,
                                    int topk, int renorm, float routed_scale, void *stream)
{
    if (!idx || !w || !x || !W) return K3GPU_EINVAL;
    if (T <= 0 || hidden <= 0 || n_experts <= 0 || n_experts > 1024 || topk < 1 || topk > 64 ||
        topk > n_experts)
        return K3GPU_EINVAL;
    if ((long long)T * n_experts > K3GPU_ROUTER_NOALLOC_MAX_SCORES) return K3GPU_ECAPACITY;
    float *scores = nullptr;
    const int st = k3::noalloc_scores(&scores);
    if (st) return st;
    return k3::router_launch(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm,
                             routed_scale, scores, k3::as_stream(stream));
}

extern "C" size_t k3gpu_router_workspace(int T, int n_experts)
{
    if (T <= 0 || n_experts <= 0) return 0;
    return (((size_t)T * n_experts * sizeof(float)) + 255) & ~(size_t)255;
}

extern "C" int k3gpu_router(int *idx, float *w, const float *x, const float *W,
                            const float *bias, int T, int hidden, int n_experts, int topk,
                            int renorm, float routed_scale, void *workspace, size_t ws_bytes,
                            void *stream)
{
    if (!idx || !w || !x || !W || !workspace) return K3GPU_EINVAL;
    if (T <= 0 || hidden <= 0 || n_experts <= 0 || n_experts > 1024 || topk < 1 || topk > 64 ||
        topk > n_experts)
        return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_router_workspace(T, n_experts)) return K3GPU_ECAPACITY;
    return k3::router_launch(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm,
                             routed_scale, static_cast<float *>(workspace),
                             k3::as_stream(stream));
}
