// router.cu -- the MoE router (k3_router, src/core/k3_ops.c:1624-1719 of the reference)
// for a whole verify batch.
//
// Scores: a register-tiled double-precision GEMM whose K loop runs in order inside each
// thread, so every (token, expert) score is ONE double chain over i = 0..hidden-1 -- the
// reference's chain (its 8-expert blocking changes issue order only). A float times a
// float is exact in double, so fma(w, x, acc) == acc + w*x rounded once, exactly the
// reference's `acc += (double)w * (double)x`. Tiles: 64 experts x 8 tokens per CTA,
// 256 threads, each owning 2 experts x 1 token (two independent chains for the double
// pipeline), operands staged through shared memory 64 columns at a time.
//
// Selection: one warp per token, repeated max with the first-index tie rule, taken
// entries set to -inf, weights from the unbiased scores, renormalised by one double sum
// in slot order -- the reference's loop, made warp-parallel only in the comparisons,
// which are exact.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace k3 {

constexpr int RT_E = 64;     // experts per CTA
constexpr int RT_T = 8;      // tokens per CTA
constexpr int RT_K = 64;     // hidden columns staged per step

__global__ void __launch_bounds__(256) router_scores_kernel(float *__restrict__ score,
                                                            const float *__restrict__ x,
                                                            const float *__restrict__ W,
                                                            int T, int hidden, int n)
{
    __shared__ float ws[RT_E][RT_K + 1];
    __shared__ float xs[RT_T][RT_K + 1];
    const int e0 = blockIdx.x * RT_E, t0 = blockIdx.y * RT_T;
    const int tid = threadIdx.x;
    const int tl = tid & 7;          // token within the tile
    const int el = tid >> 3;         // experts el and el + 32
    double acc0 = 0.0, acc1 = 0.0;
    for (int k0 = 0; k0 < hidden; k0 += RT_K) {
        const int kn = min(RT_K, hidden - k0);
        for (int i = tid; i < RT_E * RT_K; i += 256) {
            const int r = i / RT_K, c = i % RT_K;
            const int e = e0 + r;
            ws[r][c] = (e < n && c < kn) ? W[(size_t)e * hidden + k0 + c] : 0.0f;
        }
        for (int i = tid; i < RT_T * RT_K; i += 256) {
            const int r = i / RT_K, c = i % RT_K;
            const int t = t0 + r;
            xs[r][c] = (t < T && c < kn) ? x[(size_t)t * hidden + k0 + c] : 0.0f;
        }
        __syncthreads();
        for (int c = 0; c < kn; c++) {
            const double xv = (double)xs[tl][c];
            acc0 = fma((double)ws[el][c], xv, acc0);
            acc1 = fma((double)ws[el + 32][c], xv, acc1);
        }
        __syncthreads();
    }
    const int t = t0 + tl;
    if (t < T) {
        const int ea = e0 + el, eb = e0 + el + 32;
        if (ea < n) score[(size_t)t * n + ea] = sigmoid_cr(__double2float_rn(acc0));
        if (eb < n) score[(size_t)t * n + eb] = sigmoid_cr(__double2float_rn(acc1));
    }
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

int router_launch(int *idx, float *w, const float *x, const float *W, const float *bias, int T,
                  int hidden, int n, int topk, int renorm, float routed_scale, float *score,
                  cudaStream_t s)
{
    dim3 g1(ceil_div(n, RT_E), ceil_div(T, RT_T));
    router_scores_kernel<<<g1, 256, 0, s>>>(score, x, W, T, hidden, n);
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

// In host code the array's name is only a host-side stand-in, not a device address, so
// the kernels get the address cudaGetSymbolAddress returns for the current device. The
// lookup is the per-device set-up, done by the first call on each device.
static int noalloc_scores(float **out)
{
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return K3GPU_EINVAL;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        st = cuda_status(cudaGetSymbolAddress(&p, g_router_noalloc_scores));
        if (st) return st;
        g_noalloc_addr[dev] = static_cast<float *>(p);
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
