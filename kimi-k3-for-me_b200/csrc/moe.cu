// moe.cu -- grouped MXFP4 expert FFN for a verify batch (the routed half of
// k3_moe_prefill, src/core/k3_ops.c:2058-2132 of the reference, plus shared experts).
//
// Pipeline, all on one stream, no host round trip:
//   plan     one CTA: per-expert token counts, offsets, the (token, slot) pairs grouped by
//            expert, and the compact list of experts that have any token.
//   gate/up  persistent warps over units (active expert, 8 intermediate rows): each unit
//            streams 8 rows of w1 AND the same 8 rows of w3 once, for every token routed
//            to the expert, and writes act(gate, up) -- the activation is fused.
//   down     persistent warps over units (active expert, 16 rows of w2), writing each
//            pair's contribution row.
//   combine  one CTA per token: the weighted sum in the ORIGINAL top-k order from 0.0f
//            (separately rounded multiply and add, as the reference's loop), optional
//            RMSNorm of the aggregate, then the shared experts added unweighted.
//
// Weight streaming (the HBM-bound part): a lane owns one 32-element scale group of a row
// per step -- exactly one 16-byte vector load of packed nibbles plus one scale byte -- so
// a warp reads 512 contiguous bytes of a row per load instruction. Nibble pairs become
// exact f16 pairs through the hardware e2m1x2 conversion, the group's partial dot
// product runs in fp32 against fp32 activations, and the power-of-two E8M0 scale is
// applied once per group (exact: scaling by 2^k commutes with rounding). Rows are then
// reduced across the warp with a transposing butterfly (31 shuffles for 32 sums).
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <math.h>

#include <mutex>

#include "moe.cuh"

namespace k3 {

// Expert of slot s of token t, or -1 when the slot is dropped (idx < 0) or out of range.
__device__ __forceinline__ int slot_expert(const int *idx, int t, int s, int topk, int n_routed)
{
    if (s >= topk) return n_routed + (s - topk);
    const int e = idx[(size_t)t * topk + s];
    if (e < 0) return -1;
    if (e >= n_routed) { flag(DEV_BAD_INDEX); return -1; }
    return e;
}

__global__ void __launch_bounds__(1024) moe_plan_kernel(MoePlan p, const int *__restrict__ idx,
                                                        int T, int topk, int n_routed,
                                                        int n_shared)
{
    extern __shared__ int sh[];      // [E] counts, then [E] flags scan scratch
    const int E = n_routed + n_shared, S = topk + n_shared;
    const int P = T * S;
    int *scnt = sh;
    for (int e = threadIdx.x; e < E; e += blockDim.x) scnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = slot_expert(idx, i / S, i % S, topk, n_routed);
        if (e >= 0) atomicAdd(&scnt[e], 1);
    }
    __syncthreads();
    // exclusive scan of counts and of active flags: one thread walks E (<= 4096) -- the
    // plan is a few microseconds next to the weight stream, and order is deterministic
    if (threadIdx.x == 0) {
        int run = 0, na = 0;
        for (int e = 0; e < E; e++) {
            const int c = scnt[e];
            p.off[e] = run;
            p.cnt[e] = c;
            p.fill[e] = 0;
            p.elo[e] = 0;
            p.elo[E + e] = 0;
            run += c;
            if (c > 0) p.act[na++] = e;
        }
        p.off[E] = run;
        *p.n_active = na;
    }
    __syncthreads();
    __threadfence_block();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int t = i / S, s = i % S;
        const int e = slot_expert(idx, t, s, topk, n_routed);
        if (e < 0) continue;
        // placement order inside an expert only decides which warp step a token rides
        // in; every token's arithmetic is its own, so the result does not depend on it
        const int pos = p.off[e] + atomicAdd(&p.fill[e], 1);
        p.pair_tok[pos] = t;
        p.pair_dst[pos] = i;
        p.pair_exp[pos] = e;
    }
}

__device__ __forceinline__ uint4 ld_stream(const uint8_t *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// sum_{i<32} w_i * x[i] for one packed group of 16 bytes (low nibble = even element).
template <int TC>
__device__ __forceinline__ void group_dot(float (&s)[TC], const uint4 wv, const float (&xv)[TC][32])
{
    const unsigned wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const __nv_fp4x2_storage_t byte = (__nv_fp4x2_storage_t)((wd[q] >> (8 * b)) & 0xFFu);
            const __half2_raw hr = __nv_cvt_fp4x2_to_halfraw2(byte, __NV_E2M1);
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
#pragma unroll
            for (int t = 0; t < TC; t++) {
                s[t] = fmaf(f.x, xv[t][8 * q + 2 * b], s[t]);
                s[t] = fmaf(f.y, xv[t][8 * q + 2 * b + 1], s[t]);
            }
        }
    }
}

template <int TC>
__device__ __forceinline__ void load_x(float (&xv)[TC][32], const float *const (&rows)[TC], int g)
{
#pragma unroll
    for (int t = 0; t < TC; t++) {
        const float4 *src = reinterpret_cast<const float4 *>(rows[t] + (size_t)g * 32);
#pragma unroll
        for (int v = 0; v < 8; v++) {
            const float4 f = __ldg(src + v);
            xv[t][4 * v] = f.x; xv[t][4 * v + 1] = f.y; xv[t][4 * v + 2] = f.z; xv[t][4 * v + 3] = f.w;
        }
    }
}

// Stream 16 rows (row_ptr/scale_ptr give each row's base) over K = 32*G elements for TC
// token rows; after the call lane l holds the full dot product of value index l where
// value = row*TC + token (TC == 2), or row = l >> 1 (TC == 1, both lanes of a pair).
template <int TC>
__device__ __forceinline__ float stream_rows16(const uint8_t *const (&prow)[16],
                                               const uint8_t *const (&srow)[16],
                                               const float *const (&xrows)[TC], int G, int lane)
{
    float acc[16][TC];
#pragma unroll
    for (int r = 0; r < 16; r++)
#pragma unroll
        for (int t = 0; t < TC; t++) acc[r][t] = 0.0f;
    for (int g = lane; g < G; g += 32) {
        float xv[TC][32];
        load_x<TC>(xv, xrows, g);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint4 wv[8];
            unsigned sb[8];
#pragma unroll
            for (int r = 0; r < 8; r++) {
                wv[r] = ld_stream(prow[8 * h + r] + (size_t)g * 16);
                sb[r] = __ldg(srow[8 * h + r] + g);
            }
#pragma unroll
            for (int r = 0; r < 8; r++) {
                float s[TC];
#pragma unroll
                for (int t = 0; t < TC; t++) s[t] = 0.0f;
                group_dot<TC>(s, wv[r], xv);
                const float sc = e8m0_scale(sb[r]);
#pragma unroll
                for (int t = 0; t < TC; t++) acc[8 * h + r][t] = fmaf(s[t], sc, acc[8 * h + r][t]);
            }
        }
    }
    // transposing butterfly: V = 16*TC values per lane -> lane l holds value l
    constexpr int V = 16 * TC;
    float v[V];
#pragma unroll
    for (int r = 0; r < 16; r++)
#pragma unroll
        for (int t = 0; t < TC; t++) v[r * TC + t] = acc[r][t];
    int n = V;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
            const int half = n / 2;
            const bool up = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < V / 2; i++) {
                if (i < half) {
                    const float send = up ? v[i] : v[i + half];
                    const float keep = up ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            n = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

constexpr int MOE_WARPS = 8;

__global__ void __launch_bounds__(256) moe_gateup_kernel(MoePlan p, const float *__restrict__ z,
                                                         K3GpuExpertBank bank, int act,
                                                         float b1, float b2)
{
    const int lane = threadIdx.x & 31;
    const int wg = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5);
    const int nw = gridDim.x * MOE_WARPS;
    const int L = bank.L, I = bank.I, G = L / 32;
    const int RB = I / 8;
    const int units = *p.n_active * RB;
    for (int u = wg; u < units; u += nw) {
        const int a = u / RB, r0 = (u % RB) * 8;
        const int e = p.act[a];
        const uint8_t *run = bank.base + (size_t)e * bank.stride;
        const uint8_t *prow[16];
        const uint8_t *srow[16];
#pragma unroll
        for (int r = 0; r < 8; r++) {
            prow[r] = run + bank.p1 + (size_t)(r0 + r) * (L / 2);
            srow[r] = run + bank.s1 + (size_t)(r0 + r) * G;
            prow[8 + r] = run + bank.p3 + (size_t)(r0 + r) * (L / 2);
            srow[8 + r] = run + bank.s3 + (size_t)(r0 + r) * G;
        }
        const int q0 = p.off[e], q1 = p.off[e + 1];
        for (int q = q0; q < q1;) {
            if (q1 - q >= 2) {
                const float *xr[2] = {z + (size_t)p.pair_tok[q] * L, z + (size_t)p.pair_tok[q + 1] * L};
                const float v = stream_rows16<2>(prow, srow, xr, G, lane);
                const float up = __shfl_down_sync(0xffffffffu, v, 16);
                if (lane < 16) {
                    const int r = lane >> 1, t = lane & 1;
                    const float h = act == K3GPU_ACT_SITU ? act_situ(v, up, b1, b2) : act_swiglu(v, up);
                    p.H[(size_t)(q + t) * I + r0 + r] = h;
                }
                q += 2;
            } else {
                const float *xr[1] = {z + (size_t)p.pair_tok[q] * L};
                const float v = stream_rows16<1>(prow, srow, xr, G, lane);
                const float up = __shfl_down_sync(0xffffffffu, v, 16);
                if (lane < 16 && (lane & 1) == 0) {
                    const int r = lane >> 1;
                    const float h = act == K3GPU_ACT_SITU ? act_situ(v, up, b1, b2) : act_swiglu(v, up);
                    p.H[(size_t)q * I + r0 + r] = h;
                }
                q += 1;
            }
        }
    }
}

__global__ void __launch_bounds__(256) moe_down_kernel(MoePlan p, K3GpuExpertBank bank)
{
    const int lane = threadIdx.x & 31;
    const int wg = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5);
    const int nw = gridDim.x * MOE_WARPS;
    const int L = bank.L, I = bank.I, G = I / 32;
    const int RB = L / 16;
    const int units = *p.n_active * RB;
    for (int u = wg; u < units; u += nw) {
        const int a = u / RB, r0 = (u % RB) * 16;
        const int e = p.act[a];
        const uint8_t *run = bank.base + (size_t)e * bank.stride;
        const uint8_t *prow[16];
        const uint8_t *srow[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            prow[r] = run + bank.p2 + (size_t)(r0 + r) * (I / 2);
            srow[r] = run + bank.s2 + (size_t)(r0 + r) * G;
        }
        const int q0 = p.off[e], q1 = p.off[e + 1];
        for (int q = q0; q < q1;) {
            if (q1 - q >= 2) {
                const float *xr[2] = {p.H + (size_t)q * I, p.H + (size_t)(q + 1) * I};
                const float v = stream_rows16<2>(prow, srow, xr, G, lane);
                const int r = lane >> 1, t = lane & 1;
                p.contrib[(size_t)p.pair_dst[q + t] * L + r0 + r] = v;
                q += 2;
            } else {
                const float *xr[1] = {p.H + (size_t)q * I};
                const float v = stream_rows16<1>(prow, srow, xr, G, lane);
                if ((lane & 1) == 0) p.contrib[(size_t)p.pair_dst[q] * L + r0 + (lane >> 1)] = v;
                q += 1;
            }
        }
    }
}

constexpr int CMB_THREADS = 256;
constexpr int CMB_MAXV = 32;     // L <= 8192

__global__ void __launch_bounds__(CMB_THREADS) moe_combine_kernel(
    float *__restrict__ out, const float *__restrict__ contrib, const int *__restrict__ idx,
    const float *__restrict__ wt, const float *__restrict__ latent_norm, float eps, int L,
    int topk, int n_routed, int n_shared)
{
    const int t = blockIdx.x;
    const int S = topk + n_shared;
    float a[CMB_MAXV];
#pragma unroll
    for (int k = 0; k < CMB_MAXV; k++) a[k] = 0.0f;
    for (int j = 0; j < topk; j++) {
        const int e = idx[(size_t)t * topk + j];
        if (e < 0 || e >= n_routed) continue;
        const float w = wt[(size_t)t * topk + j];
        const float *c = contrib + ((size_t)t * S + j) * L;
#pragma unroll
        for (int k = 0; k < CMB_MAXV; k++) {
            const int i = threadIdx.x + k * CMB_THREADS;
            if (i < L) a[k] = __fadd_rn(a[k], __fmul_rn(w, c[i]));
        }
    }
    if (latent_norm) {
        __shared__ double red[CMB_THREADS / 32];
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < CMB_MAXV; k++) {
            const int i = threadIdx.x + k * CMB_THREADS;
            if (i < L) ss += (double)a[k] * (double)a[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < CMB_THREADS / 32; w++) tot += red[w];
        const float inv = __double2float_rn(1.0 / sqrt(tot / (double)L + (double)eps));
#pragma unroll
        for (int k = 0; k < CMB_MAXV; k++) {
            const int i = threadIdx.x + k * CMB_THREADS;
            if (i < L) a[k] = __fmul_rn(__fmul_rn(latent_norm[i], a[k]), inv);
        }
    }
    for (int s = topk; s < S; s++) {
        const float *c = contrib + ((size_t)t * S + s) * L;
#pragma unroll
        for (int k = 0; k < CMB_MAXV; k++) {
            const int i = threadIdx.x + k * CMB_THREADS;
            if (i < L) a[k] = __fadd_rn(a[k], c[i]);
        }
    }
#pragma unroll
    for (int k = 0; k < CMB_MAXV; k++) {
        const int i = threadIdx.x + k * CMB_THREADS;
        if (i < L) out[(size_t)t * L + i] = a[k];
    }
}

// The combine without the latent RMSNorm (no row reduction): the same float operations in
// the same order as moe_combine_kernel, four columns a thread and a grid over (token,
// 1024-column block), with each batch of four slots' loads issued before their adds.
__global__ void __launch_bounds__(CMB_THREADS) moe_combine_flat_kernel(
    float *__restrict__ out, const float *__restrict__ contrib, const int *__restrict__ idx,
    const float *__restrict__ wt, int L, int topk, int n_routed, int n_shared)
{
    const int t = blockIdx.x;
    const int i = (blockIdx.y * CMB_THREADS + threadIdx.x) * 4;
    if (i >= L) return;
    const int S = topk + n_shared;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    const float *base = contrib + (size_t)t * S * L + i;
    for (int j0 = 0; j0 < topk; j0 += 4) {
        float4 c[4];
        float w[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int j = j0 + u;
            const int e = j < topk ? idx[(size_t)t * topk + j] : -1;
            ok[u] = e >= 0 && e < n_routed;
            w[u] = ok[u] ? wt[(size_t)t * topk + j] : 0.f;
            c[u] = ok[u] ? *reinterpret_cast<const float4 *>(base + (size_t)j * L) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (!ok[u]) continue;
            a.x = __fadd_rn(a.x, __fmul_rn(w[u], c[u].x));
            a.y = __fadd_rn(a.y, __fmul_rn(w[u], c[u].y));
            a.z = __fadd_rn(a.z, __fmul_rn(w[u], c[u].z));
            a.w = __fadd_rn(a.w, __fmul_rn(w[u], c[u].w));
        }
    }
    for (int sidx = topk; sidx < S; sidx++) {
        const float4 c = *reinterpret_cast<const float4 *>(base + (size_t)sidx * L);
        a.x = __fadd_rn(a.x, c.x);
        a.y = __fadd_rn(a.y, c.y);
        a.z = __fadd_rn(a.z, c.z);
        a.w = __fadd_rn(a.w, c.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)t * L + i) = a;
}

// one thread per 32-element group: the expert kernels' decode, written out as floats
__global__ void mxfp4_dequant_kernel(float *__restrict__ out, const uint8_t *__restrict__ packed,
                                     const uint8_t *__restrict__ scales, long long groups)
{
    const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= groups) return;
    const uint4 wv = *reinterpret_cast<const uint4 *>(packed + gi * 16);
    const float sc = e8m0_scale(scales[gi]);
    const unsigned wd[4] = {wv.x, wv.y, wv.z, wv.w};
    float *o = out + gi * 32;
#pragma unroll
    for (int q = 0; q < 4; q++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const __nv_fp4x2_storage_t byte = (__nv_fp4x2_storage_t)((wd[q] >> (8 * b)) & 0xFFu);
            const __half2_raw hr = __nv_cvt_fp4x2_to_halfraw2(byte, __NV_E2M1);
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
            o[8 * q + 2 * b] = f.x * sc;
            o[8 * q + 2 * b + 1] = f.y * sc;
        }
}

// the current device's SM count, looked up once per device
static std::mutex g_sms_mu;
static int g_num_sms[64] = {};

static int num_sms()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(g_sms_mu);
    if (g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    return g_num_sms[dev];
}

int moe_check(const K3GpuExpertBank *bank, int T, int topk, int n_routed, int n_shared, int act)
{
    if (!bank || !bank->base) return K3GPU_EINVAL;
    if (T <= 0 || topk < 0 || topk > 64 || n_routed <= 0 || n_shared < 0) return K3GPU_EINVAL;
    if (n_routed + n_shared != bank->n_experts || bank->n_experts > 4096) return K3GPU_EINVAL;
    if ((long long)T * (topk + n_shared) > (1 << 20) || topk + n_shared == 0) return K3GPU_EINVAL;
    const int L = bank->L, I = bank->I;
    if (L <= 0 || I <= 0 || L % 32 || I % 32 || L > 8192 || I % 8) return K3GPU_EINVAL;
    if (L % 16) return K3GPU_EINVAL;
    if (act != K3GPU_ACT_SITU && act != K3GPU_ACT_SWIGLU) return K3GPU_EINVAL;
    if (!aligned(bank->base, 16) || bank->stride % 16 || bank->p1 % 16 || bank->p2 % 16 ||
        bank->p3 % 16)
        return K3GPU_EINVAL;
    return K3GPU_OK;
}

// Optional phase timing (k3gpu_moe_phase_timing): events 0..5 bracket router, plan,
// gate/up, down, combine.
constexpr int N_PHASE_EV = 6;
// The tensor-core expert kernels (moe_mma.cu) run whenever the shapes allow; the
// CUDA-core kernels above cover the rest. k3gpu_moe_select_kernels can force the latter.
static bool g_use_mma = true;
static bool g_phase_on = false;
static bool g_phase_router = false;
static cudaEvent_t g_phase_ev[N_PHASE_EV];

static void phase_mark(int i, cudaStream_t s)
{
    if (g_phase_on) cudaEventRecord(g_phase_ev[i], s);
}

int moe_launch(float *out, const float *z, const int *idx, const float *wt,
               const K3GpuExpertBank *bank, int T, int topk, int n_routed, int n_shared,
               int act, float b1, float b2, const float *latent_norm, float eps, void *ws,
               size_t ws_bytes, cudaStream_t s)
{
    const int E = n_routed + n_shared, S = topk + n_shared;
    MoePlan p;
    const size_t need = plan_bytes(T, S, E, bank->L, bank->I, &p, static_cast<char *>(ws));
    if (ws_bytes < need) return K3GPU_ECAPACITY;
    phase_mark(1, s);
    moe_plan_kernel<<<1, 1024, sizeof(int) * E, s>>>(p, idx, T, topk, n_routed, n_shared);
    int st = launch_status();
    if (st) return st;
    if (g_use_mma && mma_bank_ok(*bank)) {
        // tensor-core paths: tcgen05 on the experts the bank scan certified, mma.sync on
        // the rest (all of them when the bank was never scanned)
        const int P = T * S, E = bank->n_experts;
        const bool tc = tc_bank_ok(*bank);
        const bool sync_path = !tc || bank->n_f16_unsafe > 0;
        if ((st = tc_pack_pairs_launch(p, z, bank->L, P, E, s))) return st;
        phase_mark(2, s);
        const double tpe = (double)T * topk / (double)(n_routed > 0 ? n_routed : 1);
        if (tc && (st = tc_phase_launch(0, p, *bank, P, act, b1, b2, s, tpe))) return st;
        if (sync_path && (st = mma_phase_launch(0, p, *bank, act, b1, b2, s))) return st;
        phase_mark(3, s);
        act_pack_rows_launch(p, bank->I, P, E, s);
        if ((st = launch_status())) return st;
        if (tc && (st = tc_phase_launch(1, p, *bank, P, act, b1, b2, s, tpe))) return st;
        if (sync_path && (st = mma_phase_launch(1, p, *bank, act, b1, b2, s))) return st;
    } else {
        const int grid = num_sms() * 2;
        phase_mark(2, s);
        moe_gateup_kernel<<<grid, 256, 0, s>>>(p, z, *bank, act, b1, b2);
        if ((st = launch_status())) return st;
        phase_mark(3, s);
        moe_down_kernel<<<grid, 256, 0, s>>>(p, *bank);
        if ((st = launch_status())) return st;
    }
    phase_mark(4, s);
    if (latent_norm || (reinterpret_cast<uintptr_t>(out) & 15u)) {
        moe_combine_kernel<<<T, CMB_THREADS, 0, s>>>(out, p.contrib, idx, wt, latent_norm, eps,
                                                     bank->L, topk, n_routed, n_shared);
    } else {
        const dim3 g(T, ceil_div(bank->L, 4 * CMB_THREADS));
        moe_combine_flat_kernel<<<g, CMB_THREADS, 0, s>>>(out, p.contrib, idx, wt, bank->L, topk,
                                                          n_routed, n_shared);
    }
    st = launch_status();
    phase_mark(5, s);
    return st;
}

size_t moe_workspace(int T, int topk, int n_shared, int L, int I, int n_routed)
{
    return plan_bytes(T, topk + n_shared, n_routed + n_shared, L, I, nullptr, nullptr);
}

int router_launch(int *idx, float *w, const float *x, const float *W, const float *bias, int T,
                  int hidden, int n, int topk, int renorm, float routed_scale, float *score,
                  cudaStream_t s);

}  // namespace k3

extern "C" int k3gpu_bank_scan(K3GpuExpertBank *bank, uint8_t *safe_dev, void *stream)
{
    if (!bank || !bank->base || !safe_dev || bank->n_experts <= 0) return K3GPU_EINVAL;
    if (bank->L <= 0 || bank->I <= 0 || bank->L % 32 || bank->I % 32) return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    int st = k3::tc_bank_scan(*bank, safe_dev, s);
    if (st) return st;
    // count on the host: a one-time, synchronous certification
    const int n = bank->n_experts;
    uint8_t *h = static_cast<uint8_t *>(malloc((size_t)n));
    if (!h) return K3GPU_ECAPACITY;
    st = k3::cuda_status(cudaMemcpyAsync(h, safe_dev, (size_t)n, cudaMemcpyDeviceToHost, s));
    if (!st) st = k3::cuda_status(cudaStreamSynchronize(s));
    if (!st) {
        int bad = 0;
        for (int e = 0; e < n; e++) bad += h[e] ? 0 : 1;
        bank->f16_safe = safe_dev;
        bank->n_f16_unsafe = bad;
    }
    free(h);
    return st;
}

extern "C" int k3gpu_moe_select_kernels(int which)
{
    if (which < 0 || which > 3) return K3GPU_EINVAL;
    k3::g_use_mma = which != 1;
    k3::g_tc_shape = which == 2 ? 2 : which == 3 ? 1 : 0;
    return K3GPU_OK;
}

extern "C" int k3gpu_moe_phase_timing(int enable)
{
    if (enable && !k3::g_phase_on) {
        for (int i = 0; i < k3::N_PHASE_EV; i++) {
            const int st = k3::cuda_status(cudaEventCreate(&k3::g_phase_ev[i]));
            if (st) return st;
        }
    }
    if (!enable && k3::g_phase_on) {
        for (int i = 0; i < k3::N_PHASE_EV; i++) cudaEventDestroy(k3::g_phase_ev[i]);
    }
    k3::g_phase_on = enable != 0;
    return K3GPU_OK;
}

extern "C" int k3gpu_moe_phase_ms(float *ms, int n)
{
    if (!ms || n <= 0) return K3GPU_EINVAL;
    if (!k3::g_phase_on) return 0;
    int st = k3::cuda_status(cudaEventSynchronize(k3::g_phase_ev[k3::N_PHASE_EV - 1]));
    if (st) return st;
    int w = 0;
    for (int i = 0; i < k3::N_PHASE_EV - 1 && w < n; i++, w++) {
        float v = 0.0f;
        if (i > 0 || k3::g_phase_router) {
            st = k3::cuda_status(cudaEventElapsedTime(&v, k3::g_phase_ev[i], k3::g_phase_ev[i + 1]));
            if (st) return st;
        }
        ms[w] = v;
    }
    return w;
}

extern "C" int k3gpu_mxfp4_dequant(float *out, const uint8_t *packed, const uint8_t *scales,
                                   int rows, int in, void *stream)
{
    if (!out || !packed || !scales || rows <= 0 || in <= 0 || in % 32) return K3GPU_EINVAL;
    if (!k3::aligned(packed, 16)) return K3GPU_EINVAL;
    const long long groups = (long long)rows * (in / 32);
    k3::mxfp4_dequant_kernel<<<k3::ceil_div(groups, 256), 256, 0, k3::as_stream(stream)>>>(
        out, packed, scales, groups);
    return k3::launch_status();
}

extern "C" size_t k3gpu_moe_workspace(int T, int topk, int n_shared, int L, int I, int n_routed)
{
    if (T <= 0 || L <= 0 || I <= 0 || n_routed <= 0) return 0;
    return k3::moe_workspace(T, topk, n_shared, L, I, n_routed) +
           k3gpu_router_workspace(T, n_routed);
}

extern "C" int k3gpu_moe_experts(float *out, const float *z, const int *idx, const float *wt,
                                 const K3GpuExpertBank *bank, int T, int topk, int n_routed,
                                 int n_shared, int act, float b1, float b2,
                                 const float *latent_norm, float eps, void *workspace,
                                 size_t ws_bytes, void *stream)
{
    if (!out || !z || (!idx && topk > 0) || (!wt && topk > 0) || !workspace) return K3GPU_EINVAL;
    const int st = k3::moe_check(bank, T, topk, n_routed, n_shared, act);
    if (st) return st;
    if (!k3::aligned(z, 16)) return K3GPU_EINVAL;
    k3::g_phase_router = false;
    return k3::moe_launch(out, z, idx, wt, bank, T, topk, n_routed, n_shared, act, b1, b2,
                          latent_norm, eps, workspace, ws_bytes, k3::as_stream(stream));
}

extern "C" int k3gpu_moe_layer(float *out, int *idx, float *wt, const float *x,
                               const float *gate_W, const float *bias,
                               const K3GpuExpertBank *bank, int T, int topk, int n_routed,
                               int n_shared, int act, float b1, float b2, int renorm,
                               float routed_scale, void *workspace, size_t ws_bytes,
                               void *stream)
{
    if (!out || !idx || !wt || !x || !gate_W || !workspace) return K3GPU_EINVAL;
    int st = k3::moe_check(bank, T, topk, n_routed, n_shared, act);
    if (st) return st;
    if (topk < 1 || topk > n_routed || !k3::aligned(x, 16)) return K3GPU_EINVAL;
    const size_t rws = k3gpu_router_workspace(T, n_routed);
    if (ws_bytes < k3gpu_moe_workspace(T, topk, n_shared, bank->L, bank->I, n_routed))
        return K3GPU_ECAPACITY;
    cudaStream_t s = k3::as_stream(stream);
    k3::g_phase_router = true;
    k3::phase_mark(0, s);
    st = k3::router_launch(idx, wt, x, gate_W, bias, T, bank->L, n_routed, topk, renorm,
                           routed_scale, static_cast<float *>(workspace), s);
    if (st) return st;
    return k3::moe_launch(out, x, idx, wt, bank, T, topk, n_routed, n_shared, act, b1, b2,
                          nullptr, 0.0f, static_cast<char *>(workspace) + rws, ws_bytes - rws, s);
}
