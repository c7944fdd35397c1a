// norm.cu -- RMSNorm and AttnRes over the T positions of a verify sweep.
//
// k3_rmsnorm (src/core/k3_ops.c:132-140): a double sum of squares, the reciprocal
// 1/sqrt(ss/n + eps) rounded to float once, y = (w * x) * inv in float.
// k3_attn_res (src/core/k3_ops.c:1722-1753): per source a double sum of squares and a
// double dot of the normalised source with the folded vector, a float softmax over the
// sources (exp in float), then out = sum_s p_s * v_s accumulated in float in source order.
// The decoder layer (src/core/k3_ops.c:2514-2557) builds each position's source stack as
// its block-residual snapshots followed by its running residual; the kernel reads that
// stack in place. The double sums are block reductions here (a fixed tree, not the
// reference's sequential order), so the float results agree to an ulp, not bit for bit.
#include "common.cuh"

namespace k3 {

constexpr int NORM_THREADS = 256;

// block-wide double sum; every thread gets the total
__device__ __forceinline__ double block_sum(double v, double *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();   // red may still be read from the previous call
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < NORM_THREADS / 32; w++) t += red[w];
    return t;
}

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(float *__restrict__ y,
                                                               const float *__restrict__ x,
                                                               const float *__restrict__ w, int n,
                                                               float eps)
{
    __shared__ double red[NORM_THREADS / 32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += NORM_THREADS) ss += (double)xr[i] * (double)xr[i];
    ss = block_sum(ss, red);
    const float inv = __double2float_rn(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = threadIdx.x; i < n; i += NORM_THREADS) yr[i] = __fmul_rn(__fmul_rn(w[i], xr[i]), inv);
}

constexpr int AR_MAXSRC = 256;   // the reference's per-call score buffer is unbounded; 256 here

// One CTA per position t: sources block_residual[t][0..nb) then cur[t].
__global__ void __launch_bounds__(NORM_THREADS) attn_res_kernel(float *__restrict__ out,
                                                                const float *__restrict__ block_residual,
                                                                const float *__restrict__ cur,
                                                                const float *__restrict__ fold,
                                                                const int *__restrict__ n_blocks,
                                                                int maxb, int n, float eps)
{
    __shared__ double red[NORM_THREADS / 32];
    __shared__ float p[AR_MAXSRC];
    const int t = blockIdx.x;
    int nb = n_blocks[t];
    if (nb < 0 || nb > maxb || nb + 1 > AR_MAXSRC) {
        if (threadIdx.x == 0) flag(DEV_BAD_COUNT);
        nb = nb < 0 ? 0 : (nb > maxb ? maxb : nb);
        if (nb + 1 > AR_MAXSRC) nb = AR_MAXSRC - 1;
    }
    const int nsrc = nb + 1;
    auto source = [&](int s) -> const float * {
        return s < nb ? block_residual + ((size_t)t * maxb + s) * n : cur + (size_t)t * n;
    };
    for (int s = 0; s < nsrc; s++) {
        const float *v = source(s);
        double ss = 0.0;
        for (int i = threadIdx.x; i < n; i += NORM_THREADS) ss += (double)v[i] * (double)v[i];
        ss = block_sum(ss, red);
        const float inv = __double2float_rn(1.0 / sqrt(ss / (double)n + (double)eps));
        double acc = 0.0;
        for (int i = threadIdx.x; i < n; i += NORM_THREADS)
            acc += (double)__fmul_rn(v[i], inv) * (double)fold[i];
        acc = block_sum(acc, red);
        if (threadIdx.x == 0) p[s] = __double2float_rn(acc);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = p[0];
        for (int s = 1; s < nsrc; s++) m = p[s] > m ? p[s] : m;
        double z = 0.0;
        for (int s = 0; s < nsrc; s++) {
            p[s] = expf_cr(__fsub_rn(p[s], m));
            z += (double)p[s];
        }
        for (int s = 0; s < nsrc; s++) p[s] = __double2float_rn((double)p[s] / z);
    }
    __syncthreads();
    float *o = out + (size_t)t * n;
    for (int i = threadIdx.x; i < n; i += NORM_THREADS) {
        float a = 0.0f;
        for (int s = 0; s < nsrc; s++) a = __fadd_rn(a, __fmul_rn(p[s], source(s)[i]));
        o[i] = a;
    }
}

}  // namespace k3

extern "C" int k3gpu_rmsnorm(float *y, const float *x, const float *w, int T, int n, float eps,
                             void *stream)
{
    if (!y || !x || !w || T <= 0 || n <= 0) return K3GPU_EINVAL;
    k3::rmsnorm_kernel<<<T, k3::NORM_THREADS, 0, k3::as_stream(stream)>>>(y, x, w, n, eps);
    return k3::launch_status();
}

extern "C" int k3gpu_attn_res(float *out, const float *block_residual, const float *cur,
                              const float *fold, const int *n_blocks, int T, int maxb, int n,
                              float eps, void *stream)
{
    if (!out || !cur || !fold || !n_blocks || T <= 0 || n <= 0 || maxb < 0) return K3GPU_EINVAL;
    if (maxb > 0 && !block_residual) return K3GPU_EINVAL;
    if (maxb + 1 > k3::AR_MAXSRC) return K3GPU_ECAPACITY;
    k3::attn_res_kernel<<<T, k3::NORM_THREADS, 0, k3::as_stream(stream)>>>(out, block_residual, cur, fold,
                                                                          n_blocks, maxb, n, eps);
    return k3::launch_status();
}
