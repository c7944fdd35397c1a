// kda_chunk.cu -- KDA prefill in the chunked (UT-transform) form: a prompt's positions
// consumed into the carried state in chunks of KC positions instead of one at a time.
//
// The reference reads a prompt with the sequential recurrence only (k3_kda_step,
// src/core/k3_ops.c:303-360); this is the parallel form of the same recurrence (the
// delta-rule chunking of Yang et al., NeurIPS 2024, with the per-channel decay). Per
// chunk of n positions from state S0 (rows = key channels i, columns = value channels j),
// with g_t[i] the cumulative log2 decay through position t and r_ts[i] = 2^(g_t - g_s):
//   A_ts  = beta_t sum_i k_s k_t r_ts           (s < t)   the UT transform's matrix
//   Aq_ts = sum_i k_s q_t r_ts                  (s <= t)  the output's (diagonal kept)
//   (I + A) W = diag(beta) (V - (2^g . K) S0)             forward substitution
//   o_t   = S0^T (2^g_t . q_t) + sum_{s<=t} Aq_ts w_s
//   S     = 2^g_n . S0 + sum_s (2^(g_n - g_s) . k_s) w_s^T
// Column j of S evolves from k, q, alpha, beta and v[j] alone, so one CTA owns one
// 32-column slice of one (sequence, head) state, resident in shared memory across the
// chunks; the chunk's pair sums are recomputed by each slice. fp32 throughout: agrees
// with the sequential recurrence to rounding (not bit for bit -- the sums are reordered).
#include <float.h>
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace k3 {

constexpr int KC = 32;        // positions per chunk
constexpr int KSL = 32;       // value columns per CTA
constexpr int KTHREADS = 256;

template <int D>
struct KdaChunkSmem {
    // rows padded by 4 floats: 16-byte aligned, and 128-bit loads of rows s = lane fall on
    // distinct banks within each quarter warp (row stride = 4 banks)
    static constexpr int P = D + 4, PA = KC + 4;
    static constexpr int K = 0, Q = K + KC * P, G = Q + KC * P, KG = G + KC * P, V = KG + KC * P,
                         W = V + KC * KSL, A = W + KC * KSL, AQ = A + KC * PA, S = AQ + KC * PA,
                         BETA = S + D * KSL, FLOATS = BETA + KC;
    static constexpr size_t BYTES = sizeof(float) * FLOATS;
    static_assert(P % 4 == 0 && PA % 4 == 0 && Q % 4 == 0 && V % 4 == 0 && A % 4 == 0 && S % 4 == 0,
                  "128-bit aligned rows");
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// grid (H, B, D / KSL), block KTHREADS. state [B][H][D][D] updated in place; q, k, v,
// alpha [B][T][H][D], beta [B][T][H]; o [B][T][H][D] (may be NULL).
template <int D>
__global__ void __launch_bounds__(KTHREADS) kda_chunk_kernel(float *__restrict__ state, float *__restrict__ o,
                                                            const float *__restrict__ q,
                                                            const float *__restrict__ k,
                                                            const float *__restrict__ v,
                                                            const float *__restrict__ al,
                                                            const float *__restrict__ beta, int T, int H,
                                                            float qscale)
{
    using L = KdaChunkSmem<D>;
    constexpr int P = L::P, PA = L::PA;
    constexpr int RT = KC / (KTHREADS / 32);   // rows t per warp in the row-blocked phases
    constexpr int RI = D / (KTHREADS / 32);    // state rows per warp in the update
    extern __shared__ __align__(16) float sm[];
    float *sK = sm + L::K, *sQ = sm + L::Q, *sG = sm + L::G, *sKG = sm + L::KG, *sV = sm + L::V,
          *sW = sm + L::W, *sA = sm + L::A, *sAQ = sm + L::AQ, *sS = sm + L::S, *sB = sm + L::BETA;
    const int h = blockIdx.x, b = blockIdx.y, j0 = blockIdx.z * KSL;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = KTHREADS / 32;

    float *Sg = state + (((size_t)b * H + h) * D) * D;
    for (int e = tid; e < D * KSL; e += KTHREADS) {
        const int i = e / KSL, j = e % KSL;
        sS[i * KSL + j] = Sg[(size_t)i * D + j0 + j];
    }

    // the chunk's raw rows are fetched into registers one chunk ahead, so their loads are
    // in flight while the chunk before computes; positions past the end read as zero keys,
    // queries and values, decay 1 and beta 0
    constexpr int NE = KC * D / KTHREADS, NV = KC * KSL / KTHREADS;
    float rk[NE], rq[NE], ra[NE], rv[NV], rb = 0.0f;
    auto fetch = [&](int c) {
        const int m = T - c < KC ? T - c : KC;
#pragma unroll
        for (int r = 0; r < NE; r++) {
            const int e = tid + r * KTHREADS, t = e / D, i = e % D;
            rk[r] = 0.0f;
            rq[r] = 0.0f;
            ra[r] = 1.0f;
            if (t < m) {
                const size_t off = (((size_t)b * T + c + t) * H + h) * D + i;
                rk[r] = k[off];
                rq[r] = q[off];
                ra[r] = al[off];
            }
        }
#pragma unroll
        for (int r = 0; r < NV; r++) {
            const int e = tid + r * KTHREADS, t = e / KSL, j = e % KSL;
            rv[r] = t < m ? v[(((size_t)b * T + c + t) * H + h) * D + j0 + j] : 0.0f;
        }
        rb = tid < m ? beta[((size_t)b * T + c + tid) * H + h] : 0.0f;
    };
    fetch(0);

    for (int c0 = 0; c0 < T; c0 += KC) {
        const int n = T - c0 < KC ? T - c0 : KC;
        __syncthreads();   // the previous chunk's readers are done
        // 1. the chunk's rows into shared memory, then the next chunk's loads
#pragma unroll
        for (int r = 0; r < NE; r++) {
            const int e = tid + r * KTHREADS, t = e / D, i = e % D;
            sK[t * P + i] = rk[r];
            sQ[t * P + i] = rq[r] * qscale;
            sG[t * P + i] = log2f(fmaxf(ra[r], FLT_MIN));
        }
#pragma unroll
        for (int r = 0; r < NV; r++) {
            const int e = tid + r * KTHREADS;
            sV[(e / KSL) * KSL + e % KSL] = rv[r];
        }
        if (tid < KC) sB[tid] = rb;
        if (c0 + KC < T) fetch(c0 + KC);
        __syncthreads();
        // 2. cumulative log2 decay per channel
        for (int i = tid; i < D; i += KTHREADS) {
            float acc = 0.0f;
            for (int t = 0; t < KC; t++) {
                acc += sG[t * P + i];
                sG[t * P + i] = acc;
            }
        }
        __syncthreads();
        // 3. the pair sums: lane = s, the warp's rows t = warp + NW r together, so row s's
        //    keys and decays are loaded once per 4 channels for RT rows
        {
            const int s = lane;
            float akk[RT], aqk[RT];
#pragma unroll
            for (int r = 0; r < RT; r++) akk[r] = aqk[r] = 0.0f;
            for (int i = 0; i < D; i += 4) {
                const float4 k4 = ld4(sK + s * P + i), g4 = ld4(sG + s * P + i);
#pragma unroll
                for (int r = 0; r < RT; r++) {
                    const int t = warp + NW * r;
                    const float4 kt = ld4(sK + t * P + i), qt = ld4(sQ + t * P + i), gt = ld4(sG + t * P + i);
                    float kr = k4.x * exp2f(gt.x - g4.x);
                    akk[r] = fmaf(kr, kt.x, akk[r]);
                    aqk[r] = fmaf(kr, qt.x, aqk[r]);
                    kr = k4.y * exp2f(gt.y - g4.y);
                    akk[r] = fmaf(kr, kt.y, akk[r]);
                    aqk[r] = fmaf(kr, qt.y, aqk[r]);
                    kr = k4.z * exp2f(gt.z - g4.z);
                    akk[r] = fmaf(kr, kt.z, akk[r]);
                    aqk[r] = fmaf(kr, qt.z, aqk[r]);
                    kr = k4.w * exp2f(gt.w - g4.w);
                    akk[r] = fmaf(kr, kt.w, akk[r]);
                    aqk[r] = fmaf(kr, qt.w, aqk[r]);
                }
            }
            // s > t lanes computed ratios above 1 (possibly infinite); they are dropped here
#pragma unroll
            for (int r = 0; r < RT; r++) {
                const int t = warp + NW * r;
                sA[t * PA + s] = s < t ? akk[r] * sB[t] : 0.0f;
                sAQ[t * PA + s] = s <= t ? aqk[r] : 0.0f;
            }
        }
        __syncthreads();
        // 4a. the decayed keys and queries (2^g . k, 2^g . q), four channels at a time
        for (int e = tid; e < KC * D / 4; e += KTHREADS) {
            const int t = (e * 4) / D, i = (e * 4) % D;
            const float4 g = ld4(sG + t * P + i), kk = ld4(sK + t * P + i), qq = ld4(sQ + t * P + i);
            const float4 d = make_float4(exp2f(g.x), exp2f(g.y), exp2f(g.z), exp2f(g.w));
            *reinterpret_cast<float4 *>(sKG + t * P + i) = make_float4(kk.x * d.x, kk.y * d.y, kk.z * d.z, kk.w * d.w);
            *reinterpret_cast<float4 *>(sQ + t * P + i) = make_float4(qq.x * d.x, qq.y * d.y, qq.z * d.z, qq.w * d.w);
        }
        __syncthreads();
        // 4b. right-hand side: beta_t (v_t - S0^T (2^g_t . k_t)), column j = lane, RT rows
        {
            float acc[RT];
#pragma unroll
            for (int r = 0; r < RT; r++) acc[r] = 0.0f;
            for (int i = 0; i < D; i += 4) {
                const float s0 = sS[(i + 0) * KSL + lane], s1 = sS[(i + 1) * KSL + lane],
                            s2 = sS[(i + 2) * KSL + lane], s3 = sS[(i + 3) * KSL + lane];
#pragma unroll
                for (int r = 0; r < RT; r++) {
                    const float4 kg = ld4(sKG + (warp + NW * r) * P + i);
                    acc[r] = fmaf(kg.x, s0, acc[r]);
                    acc[r] = fmaf(kg.y, s1, acc[r]);
                    acc[r] = fmaf(kg.z, s2, acc[r]);
                    acc[r] = fmaf(kg.w, s3, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < RT; r++) {
                const int t = warp + NW * r;
                sW[t * KSL + lane] = sB[t] * (sV[t * KSL + lane] - acc[r]);
            }
        }
        __syncthreads();
        // 5. forward substitution (I + A) W = rhs, one column per lane of warp 0
        if (warp == 0) {
            float w[KC];
#pragma unroll
            for (int t = 0; t < KC; t++) {
                float x = sW[t * KSL + lane];
#pragma unroll
                for (int s = 0; s < t; s++) x = fmaf(-sA[t * PA + s], w[s], x);
                w[t] = x;
                sW[t * KSL + lane] = x;
            }
        }
        __syncthreads();
        // 6. outputs (RT rows per warp; Aq is zero above its diagonal and W past n), and
        //    the keys decayed to the chunk's end, 2^(g_n - g_s) . k_s
        if (o) {
            float acc[RT];
#pragma unroll
            for (int r = 0; r < RT; r++) acc[r] = 0.0f;
            for (int i = 0; i < D; i += 4) {
                const float s0 = sS[(i + 0) * KSL + lane], s1 = sS[(i + 1) * KSL + lane],
                            s2 = sS[(i + 2) * KSL + lane], s3 = sS[(i + 3) * KSL + lane];
#pragma unroll
                for (int r = 0; r < RT; r++) {
                    const float4 qg = ld4(sQ + (warp + NW * r) * P + i);
                    acc[r] = fmaf(qg.x, s0, acc[r]);
                    acc[r] = fmaf(qg.y, s1, acc[r]);
                    acc[r] = fmaf(qg.z, s2, acc[r]);
                    acc[r] = fmaf(qg.w, s3, acc[r]);
                }
            }
            for (int s = 0; s < KC; s += 4) {
                const float w0 = sW[(s + 0) * KSL + lane], w1 = sW[(s + 1) * KSL + lane],
                            w2 = sW[(s + 2) * KSL + lane], w3 = sW[(s + 3) * KSL + lane];
#pragma unroll
                for (int r = 0; r < RT; r++) {
                    const float4 aq = ld4(sAQ + (warp + NW * r) * PA + s);
                    acc[r] = fmaf(aq.x, w0, acc[r]);
                    acc[r] = fmaf(aq.y, w1, acc[r]);
                    acc[r] = fmaf(aq.z, w2, acc[r]);
                    acc[r] = fmaf(aq.w, w3, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < RT; r++) {
                const int t = warp + NW * r;
                if (t < n) o[(((size_t)b * T + c0 + t) * H + h) * D + j0 + lane] = acc[r];
            }
        }
        for (int e = tid; e < KC * D / 4; e += KTHREADS) {
            const int t = (e * 4) / D, i = (e * 4) % D;
            const float4 g = ld4(sG + t * P + i), gn = ld4(sG + (KC - 1) * P + i), kk = ld4(sK + t * P + i);
            *reinterpret_cast<float4 *>(sKG + t * P + i) =
                make_float4(kk.x * exp2f(gn.x - g.x), kk.y * exp2f(gn.y - g.y), kk.z * exp2f(gn.z - g.z),
                            kk.w * exp2f(gn.w - g.w));
        }
        __syncthreads();
        // 7. the state at the chunk's end: warp rows i0 .. i0 + RI - 1, column = lane
        {
            const int i0 = warp * RI;
            float acc[RI];
#pragma unroll
            for (int q = 0; q < RI; q++) acc[q] = sS[(i0 + q) * KSL + lane] * exp2f(sG[(KC - 1) * P + i0 + q]);
            for (int s = 0; s < n; s++) {
                const float w = sW[s * KSL + lane];
#pragma unroll
                for (int q = 0; q < RI; q += 4) {
                    const float4 ke = ld4(sKG + s * P + i0 + q);
                    acc[q + 0] = fmaf(ke.x, w, acc[q + 0]);
                    acc[q + 1] = fmaf(ke.y, w, acc[q + 1]);
                    acc[q + 2] = fmaf(ke.z, w, acc[q + 2]);
                    acc[q + 3] = fmaf(ke.w, w, acc[q + 3]);
                }
            }
#pragma unroll
            for (int q = 0; q < RI; q++) sS[(i0 + q) * KSL + lane] = acc[q];
        }
    }
    __syncthreads();
    for (int e = tid; e < D * KSL; e += KTHREADS) {
        const int i = e / KSL, j = e % KSL;
        Sg[(size_t)i * D + j0 + j] = sS[i * KSL + j];
    }
}

template <int D>
static int kda_chunk_launch(float *state, float *o, const float *q, const float *k, const float *v,
                            const float *alpha, const float *beta, int B, int T, int H, float qscale,
                            cudaStream_t s)
{
    const size_t bytes = KdaChunkSmem<D>::BYTES;
    // the opt-in to >48 KB of dynamic shared memory, once per device and width (a
    // function's attributes belong to each device's context)
    static std::mutex mu;
    static bool ready[64] = {};
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!ready[dev]) {
            st = cuda_status(cudaFuncSetAttribute(kda_chunk_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)bytes));
            if (st) return st;
            ready[dev] = true;
        }
    }
    dim3 grid(H, B, D / KSL);
    kda_chunk_kernel<D><<<grid, KTHREADS, bytes, s>>>(state, o, q, k, v, alpha, beta, T, H, qscale);
    return launch_status();
}

}  // namespace k3

extern "C" int k3gpu_kda_prefill(float *state, float *o, const float *q, const float *k, const float *v,
                                 const float *alpha, const float *beta, int B, int T, int H, int D, float qscale,
                                 void *stream)
{
    if (!state || !q || !k || !v || !alpha || !beta) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || H <= 0 || H > 65535 || B > 65535) return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    switch (D) {
        case 32: return k3::kda_chunk_launch<32>(state, o, q, k, v, alpha, beta, B, T, H, qscale, s);
        case 64: return k3::kda_chunk_launch<64>(state, o, q, k, v, alpha, beta, B, T, H, qscale, s);
        case 128: return k3::kda_chunk_launch<128>(state, o, q, k, v, alpha, beta, B, T, H, qscale, s);
        default: return K3GPU_EINVAL;
    }
}
