// norm.cu -- RMSNorm and AttnRes over the T positions of a verify sweep.
//
// k3_rmsnorm (src/core/k3_ops.c:132-140): a double sum of squares, the reciprocal
// 1/sqrt(ss/n + eps) rounded to float once, y = (w * x) * inv in float.
// k3_attn_res (src/core/k3_ops.c:1722-1753): per source a double sum of squares and a
// double dot of the normalised source with the folded vector, a float softmax over the
// sources (exp in float), then out = sum_s p_s * v_s accumulated in float in source order.
// The decoder layer (src/core/k3_ops.c:2514-2557) builds each position's source stack as
// its block-residual snapshots followed by its running residual; the kernel reads that
// stack in place. The double sums are warp reductions here (a fixed tree, not the
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

// warp-wide double sum; every lane gets the total
__device__ __forceinline__ double warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One CTA per position t: sources block_residual[t][0..nb) then cur[t]. A deep stack gives a
// position dozens of sources (one snapshot per two layers), so the scores are spread over
// the warps -- warp w takes sources w, w + 8, ...: its sum of squares, the reciprocal, the
// dot of the normalised source with the fold, each a warp reduction (no block barrier per
// source), the second pass over the source mostly from L1 -- and the weighted sum reads
// every source once more. vec: rows 16-byte aligned and n % 4 == 0 (float4 loads).
__global__ void __launch_bounds__(NORM_THREADS) attn_res_kernel(float *__restrict__ out,
                                                                const float *__restrict__ block_residual,
                                                                const float *__restrict__ cur,
                                                                const float *__restrict__ fold,
                                                                const int *__restrict__ n_blocks,
                                                                int maxb, int n, float eps, int vec)
{
    __shared__ float p[AR_MAXSRC];
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    for (int s = warp; s < nsrc; s += NORM_THREADS / 32) {
        const float *v = source(s);
        double ss = 0.0;
        if (vec) {
            for (int i = 4 * lane; i < n; i += 128) {
                const float4 x = *reinterpret_cast<const float4 *>(v + i);
                ss += (double)x.x * (double)x.x;
                ss += (double)x.y * (double)x.y;
                ss += (double)x.z * (double)x.z;
                ss += (double)x.w * (double)x.w;
            }
        } else {
            for (int i = lane; i < n; i += 32) ss += (double)v[i] * (double)v[i];
        }
        ss = warp_sum_d(ss);
        const float inv = __double2float_rn(1.0 / sqrt(ss / (double)n + (double)eps));
        double acc = 0.0;
        if (vec) {
            for (int i = 4 * lane; i < n; i += 128) {
                const float4 x = *reinterpret_cast<const float4 *>(v + i);
                const float4 f = *reinterpret_cast<const float4 *>(fold + i);
                acc += (double)__fmul_rn(x.x, inv) * (double)f.x;
                acc += (double)__fmul_rn(x.y, inv) * (double)f.y;
                acc += (double)__fmul_rn(x.z, inv) * (double)f.z;
                acc += (double)__fmul_rn(x.w, inv) * (double)f.w;
            }
        } else {
            for (int i = lane; i < n; i += 32) acc += (double)__fmul_rn(v[i], inv) * (double)fold[i];
        }
        acc = warp_sum_d(acc);
        if (lane == 0) p[s] = __double2float_rn(acc);
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
    if (vec) {
        for (int i = 4 * threadIdx.x; i < n; i += 4 * NORM_THREADS) {
            float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int s = 0; s < nsrc; s++) {
                const float4 x = *reinterpret_cast<const float4 *>(source(s) + i);
                const float ps = p[s];
                a.x = __fadd_rn(a.x, __fmul_rn(ps, x.x));
                a.y = __fadd_rn(a.y, __fmul_rn(ps, x.y));
                a.z = __fadd_rn(a.z, __fmul_rn(ps, x.z));
                a.w = __fadd_rn(a.w, __fmul_rn(ps, x.w));
            }
            *reinterpret_cast<float4 *>(o + i) = a;
        }
    } else {
        for (int i = threadIdx.x; i < n; i += NORM_THREADS) {
            float a = 0.0f;
            for (int s = 0; s < nsrc; s++) a = __fadd_rn(a, __fmul_rn(p[s], source(s)[i]));
            o[i] = a;
        }
    }
}

// One CTA per position t, every source read from HBM once: thread j holds columns 4j +
// 1024v (v < NV) of the source in registers, so a row of up to 1024 NV floats is scored
// and summed from the same loads. Per source: the sum of squares (a block reduction), the
// reciprocal, the dot of the normalised source with the fold (per term rounded as the
// reference does, a second block reduction), then an online softmax -- the running
// maximum m, the weights exp(score - m) and the accumulated rows rescaled by exp(m_old -
// m_new) when the maximum rises, and out = acc / z at the end. The reference's
// normalised weights are exp(score - m_final) / z, so this agrees with it to rounding, and
// a single source gives its row unchanged. The next source's loads are issued before the
// current one's reductions. Every thread computes the same totals (the warp butterfly gives
// all lanes one value, the eight warp partials are summed in warp order), so the softmax
// state is uniform. Two reduction buffers, ss in one and the dot in the other: a buffer is
// written again only two barriers after it was read.
template <int NV>
__global__ void __launch_bounds__(NORM_THREADS, 2) attn_res_rows_kernel(float *__restrict__ out,
                                                                        const float *__restrict__ block_residual,
                                                                        const float *__restrict__ cur,
                                                                        const float *__restrict__ fold,
                                                                        const int *__restrict__ n_blocks,
                                                                        int maxb, int n, float eps)
{
    __shared__ double red[2][NORM_THREADS / 32];
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    auto load = [&](float4 (&x)[NV], const float *v) {
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int i = 4 * threadIdx.x + 4 * NORM_THREADS * k;
            x[k] = i < n ? __ldg(reinterpret_cast<const float4 *>(v + i)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    };
    auto block_total = [&](double v, double *r) {
        v = warp_sum_d(v);
        if (lane == 0) r[warp] = v;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < NORM_THREADS / 32; w++) tot += r[w];
        return tot;
    };
    float4 x[NV], a[NV];
#pragma unroll
    for (int k = 0; k < NV; k++) a[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    load(x, source(0));
    float m = 0.0f;
    double z = 0.0;
    for (int s = 0; s < nsrc; s++) {
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < NV; k++) {      // columns past n hold zeros and add nothing
            ss += (double)x[k].x * (double)x[k].x;
            ss += (double)x[k].y * (double)x[k].y;
            ss += (double)x[k].z * (double)x[k].z;
            ss += (double)x[k].w * (double)x[k].w;
        }
        float4 xn[NV];
        if (s + 1 < nsrc) load(xn, source(s + 1));
        ss = block_total(ss, red[0]);
        const float inv = __double2float_rn(1.0 / sqrt(ss / (double)n + (double)eps));
        double dot = 0.0;
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int i = 4 * threadIdx.x + 4 * NORM_THREADS * k;
            if (i < n) {
                const float4 f = __ldg(reinterpret_cast<const float4 *>(fold + i));
                dot += (double)__fmul_rn(x[k].x, inv) * (double)f.x;
                dot += (double)__fmul_rn(x[k].y, inv) * (double)f.y;
                dot += (double)__fmul_rn(x[k].z, inv) * (double)f.z;
                dot += (double)__fmul_rn(x[k].w, inv) * (double)f.w;
            }
        }
        const float sc = __double2float_rn(block_total(dot, red[1]));
        // the reference's maximum: the first score, then any later one that is greater
        float c = 1.0f;
        if (s == 0 || sc > m) {
            c = s == 0 ? 0.0f : expf_cr(__fsub_rn(m, sc));
            m = sc;
        }
        // a score of -inf weighs exp(-inf - m_final): 0, or NaN through z = 0 at the end when
        // every score is -inf, as in the reference
        const float e = sc == __int_as_float(0xff800000) ? 0.0f : expf_cr(__fsub_rn(sc, m));
        z = (double)c * z + (double)e;
#pragma unroll
        for (int k = 0; k < NV; k++) {
            if (c != 1.0f) {
                a[k].x = __fmul_rn(a[k].x, c);
                a[k].y = __fmul_rn(a[k].y, c);
                a[k].z = __fmul_rn(a[k].z, c);
                a[k].w = __fmul_rn(a[k].w, c);
            }
            a[k].x = __fadd_rn(a[k].x, __fmul_rn(e, x[k].x));
            a[k].y = __fadd_rn(a[k].y, __fmul_rn(e, x[k].y));
            a[k].z = __fadd_rn(a[k].z, __fmul_rn(e, x[k].z));
            a[k].w = __fadd_rn(a[k].w, __fmul_rn(e, x[k].w));
        }
        if (s + 1 < nsrc) {
#pragma unroll
            for (int k = 0; k < NV; k++) x[k] = xn[k];
        }
    }
    const double rz = 1.0 / z;
    float *o = out + (size_t)t * n;
#pragma unroll
    for (int k = 0; k < NV; k++) {
        const int i = 4 * threadIdx.x + 4 * NORM_THREADS * k;
        if (i < n) {
            float4 r;
            r.x = __double2float_rn((double)a[k].x * rz);
            r.y = __double2float_rn((double)a[k].y * rz);
            r.z = __double2float_rn((double)a[k].z * rz);
            r.w = __double2float_rn((double)a[k].w * rz);
            *reinterpret_cast<float4 *>(o + i) = r;
        }
    }
}

constexpr int AR_ROWS_MAXV = 7;   // register rows up to 7 x 1024 floats (K3's 7168); 8 spills

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
    const auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const int vec = (n & 3) == 0 && al16(cur) && al16(fold) && al16(out) && (!block_residual || al16(block_residual));
    cudaStream_t s = k3::as_stream(stream);
    const int nv = (n + 4 * k3::NORM_THREADS - 1) / (4 * k3::NORM_THREADS);
    if (vec && nv <= k3::AR_ROWS_MAXV) {
#define K3_AR_ROWS(V)                                                                                      \
    case V:                                                                                                \
        k3::attn_res_rows_kernel<V><<<T, k3::NORM_THREADS, 0, s>>>(out, block_residual, cur, fold, n_blocks, \
                                                                    maxb, n, eps);                         \
        break;
        switch (nv) {
            K3_AR_ROWS(1)
            K3_AR_ROWS(2)
            K3_AR_ROWS(3)
            K3_AR_ROWS(4)
            K3_AR_ROWS(5)
            K3_AR_ROWS(6)
            K3_AR_ROWS(7)
        }
#undef K3_AR_ROWS
    } else {
        k3::attn_res_kernel<<<T, k3::NORM_THREADS, 0, s>>>(out, block_residual, cur, fold, n_blocks, maxb, n, eps,
                                                           vec);
    }
    return k3::launch_status();
}
