// router.cu -- the MoE router (k3_router, src/core/k3_ops.c:1624-1719 of the reference)
// for a whole verify batch.
//
// Scores: every (token, expert) score is ONE double chain over i = 0..hidden-1, in order
// -- the reference's chain (its 8-expert blocking changes issue order only). A float times
// a float is exact in double, so fma(w, x, acc) == acc + w*x rounded once, exactly the
// reference's `acc += (double)w * (double)x`. Which chains a thread runs side by side is
// free, so a thread owns a block of A tokens x B experts (up to 16 independent chains).
//
// What bounds the kernel on B200 is operand delivery, not the FP64 pipe (64 FMA/clock/SM):
// shared memory hands each lane at most ~128 bytes per clock per SM, one double per two
// FMAs at B = 2 if every lane read its own. So the A tokens of a thread are WARP-UNIFORM
// (every lane of a warp reads the same x doubles: broadcast loads) and only the B experts
// differ by lane; 4 warps of a CTA take 4 token groups against the same 32 B experts. K
// tiles of 32 columns arrive by cp.async as floats in [row][36] rows (conflict-free float4
// reads), as many tiles ahead as a 110 KB budget holds (two CTAs per SM): small shapes stream
// W with few CTAs, so their bytes in flight per CTA must cover the DRAM latency by
// themselves. Each tile is widened once per CTA into a [k][row] double tile; one barrier per
// tile. The tile shape per call comes from a small cost model over the SM
// count (FP64 issue per scheduler against shared-memory wavefronts per SM).
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

constexpr int RB_K = 32;          // hidden columns per tile
constexpr int RB_FLD = RB_K + 4;  // float stage row stride (16-byte rows on distinct banks)
constexpr int RB_THREADS = 128;   // 4 warps, one token group each
constexpr int RB_BUDGET = 110 * 1024;   // shared memory per CTA

// CTA tile of the scores kernel: A tokens per warp (A even), B experts per lane.
template <int A, int B>
struct RbTile {
    static constexpr int TT = 4 * A;                        // tokens per CTA
    static constexpr int TE = 32 * B;                       // experts per CTA
    static constexpr int ROWS = TT + TE;                    // rows of a tile
    static constexpr int PIECES = ROWS * RB_K / 4;          // float4 pieces per tile
    static constexpr int FSTAGE = ROWS * RB_FLD;            // floats per stage
    static constexpr int DTILE = 2 * RB_K * ROWS * 8;       // the two double tiles
    static constexpr int NS_FIT = (RB_BUDGET - DTILE) / (FSTAGE * 4);
    static constexpr int NS = NS_FIT < 3 ? 3 : (NS_FIT > 16 ? 16 : NS_FIT);   // cp.async stages
    static constexpr int SMEM = NS * FSTAGE * 4 + DTILE;
    static_assert(A % 2 == 0 && (B == 1 || B == 2), "tile shape");
};

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

template <int A, int B, int V>   // V = 4 when hidden % 4 == 0 and x, W are 16-byte aligned, else 1
__global__ void __launch_bounds__(RB_THREADS) router_scores_kernel(float *__restrict__ score,
                                                                   const float *__restrict__ x,
                                                                   const float *__restrict__ W,
                                                                   int T, int hidden, int n)
{
    using Tl = RbTile<A, B>;
    extern __shared__ __align__(16) unsigned char rsm[];
    float *fst = reinterpret_cast<float *>(rsm);                              // [NS][ROWS][FLD]
    double *dt = reinterpret_cast<double *>(rsm + Tl::NS * Tl::FSTAGE * 4);    // [2][K][ROWS]
    const int t0 = blockIdx.y * Tl::TT, e0 = blockIdx.x * Tl::TE;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int trow = warp * A;                 // this warp's first token row in the tile
    const int erow = Tl::TT + B * lane;        // this lane's first expert row
    const int nt = (hidden + RB_K - 1) / RB_K;

    // tile kt's floats into stage kt % NS (an empty group past the end keeps the count)
    auto issue = [&](int kt) {
        if (kt < nt) {
            float *f = fst + (kt % Tl::NS) * Tl::FSTAGE;
            const int k0 = kt * RB_K;
            for (int i = tid; i < Tl::ROWS * (RB_K / V); i += RB_THREADS) {
                const int r = i / (RB_K / V), c = (i % (RB_K / V)) * V;
                const bool is_x = r < Tl::TT;
                const int row = is_x ? t0 + r : e0 + (r - Tl::TT);
                const bool ok = (is_x ? row < T : row < n) && k0 + c < hidden;
                const float *src = is_x ? x : W;
                if (ok) src += (size_t)row * hidden + k0 + c;
                cp_async_f<V>(f + r * RB_FLD + c, src, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // tile kt's floats widened into double buffer kt & 1, [k][row]
    auto widen = [&](int kt) {
        const float *f = fst + (kt % Tl::NS) * Tl::FSTAGE;
        double *d = dt + (kt & 1) * RB_K * Tl::ROWS;
        for (int p = tid; p < Tl::PIECES; p += RB_THREADS) {
            const int r = p % Tl::ROWS, c = 4 * (p / Tl::ROWS);
            const float4 v = *reinterpret_cast<const float4 *>(f + r * RB_FLD + c);
            d[(c + 0) * Tl::ROWS + r] = (double)v.x;
            d[(c + 1) * Tl::ROWS + r] = (double)v.y;
            d[(c + 2) * Tl::ROWS + r] = (double)v.z;
            d[(c + 3) * Tl::ROWS + r] = (double)v.w;
        }
    };

    double acc[A][B];
#pragma unroll
    for (int a = 0; a < A; a++)
#pragma unroll
        for (int b = 0; b < B; b++) acc[a][b] = 0.0;

    auto step = [&](const double *dk) {
        double xv[A], wv[B];
#pragma unroll
        for (int i = 0; i < A; i += 2) {   // the same address in every lane: a broadcast
            const double2 v = *reinterpret_cast<const double2 *>(dk + trow + i);
            xv[i] = v.x;
            xv[i + 1] = v.y;
        }
        if (B == 2) {
            const double2 v = *reinterpret_cast<const double2 *>(dk + erow);
            wv[0] = v.x;
            wv[B - 1] = v.y;
        } else {
            wv[0] = dk[erow];
        }
#pragma unroll
        for (int a = 0; a < A; a++)
#pragma unroll
            for (int b = 0; b < B; b++) acc[a][b] = __fma_rn(wv[b], xv[a], acc[a][b]);
    };

    for (int kt = 0; kt < Tl::NS - 1; kt++) issue(kt);
    asm volatile("cp.async.wait_group %0;" ::"n"(Tl::NS - 2) : "memory");
    __syncthreads();                           // tile 0 landed for every thread's copies
    widen(0);
    for (int kt = 0; kt < nt; kt++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(Tl::NS - 3) : "memory");
        // tile kt+1 landed; widen(kt) done and compute(kt-1) finished in every warp
        __syncthreads();
        issue(kt + Tl::NS - 1);                 // into the stage tile kt-1 used
        if (kt + 1 < nt) widen(kt + 1);        // into the buffer compute(kt-1) read
        const double *d = dt + (kt & 1) * RB_K * Tl::ROWS;
        const int kn = min(RB_K, hidden - kt * RB_K);
        if (kn == RB_K) {
#pragma unroll 8
            for (int k = 0; k < RB_K; k++) step(d + k * Tl::ROWS);
        } else {
            for (int k = 0; k < kn; k++) step(d + k * Tl::ROWS);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int a = 0; a < A; a++) {
        const int t = t0 + trow + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int e = e0 + B * lane + b;
            if (e < n) score[(size_t)t * n + e] = sigmoid_cr(__double2float_rn(acc[a][b]));
        }
    }
}

// Small batches: one chain per thread. When the whole call fits one wave of CTAs (a verify
// step of a few sequences: T <= ~72 at 384 experts), every CTA walks all hidden columns
// whatever its tile shape, so the time is the per-column cost of one CTA's walk. This form
// keeps that short: a CTA owns 24 experts x 8 tokens (192 chains), 128-column K tiles (a
// quarter of the barriers of the 32-column tiles above) arrive by cp.async two tiles
// ahead and are widened to double once in shared memory, and each thread runs its chain
// from registers loaded eight columns ahead.
constexpr int RW_E = 24;     // experts per CTA
constexpr int RW_T = 8;      // tokens per CTA
constexpr int RW_R = RW_E + RW_T;
constexpr int RW_THREADS = RW_E * RW_T;
constexpr int RW_K = 128;    // hidden columns per tile
constexpr int RW_NS = 3;     // cp.async stages
constexpr int RW_LD = RW_K + 2;   // double tile row stride: rows land on distinct banks
constexpr int RW_F_TILE = RW_R * RW_K;
constexpr int RW_SMEM = RW_NS * RW_F_TILE * 4 + 2 * RW_R * RW_LD * 8;

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
__global__ void __launch_bounds__(RW_THREADS) router_scores_wave_kernel(float *__restrict__ score,
                                                                        const float *__restrict__ x,
                                                                        const float *__restrict__ W,
                                                                        int T, int hidden, int n)
{
    extern __shared__ __align__(16) unsigned char rsm[];
    float *fst = reinterpret_cast<float *>(rsm);                            // [NS][R][K]
    double *dt = reinterpret_cast<double *>(rsm + RW_NS * RW_F_TILE * 4);   // [2][R][LD]
    const int e0 = blockIdx.x * RW_E, t0 = blockIdx.y * RW_T;
    const int tid = threadIdx.x;
    const int tl = tid & 7;          // token of this thread's chain
    const int el = tid >> 3;         // expert of this thread's chain
    const int nt = (hidden + RW_K - 1) / RW_K;
    constexpr int CPR = RW_K / V;    // copies per tile row

    auto issue = [&](int kt) {
        if (kt < nt) {
            float *f = fst + (kt % RW_NS) * RW_F_TILE;
            const int k0 = kt * RW_K;
            for (int i = tid; i < RW_R * CPR; i += RW_THREADS) {
                const int r = i / CPR, c = (i % CPR) * V;
                const bool is_w = r < RW_E;
                const int row = is_w ? e0 + r : t0 + (r - RW_E);
                const bool ok = (is_w ? row < n : row < T) && k0 + c < hidden;
                const float *src = is_w ? W : x;
                if (ok) src += (size_t)row * hidden + k0 + c;
                cp_async_f<V>(f + r * RW_K + c, src, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int kt = 0; kt < RW_NS - 1; kt++) issue(kt);

    double acc = 0.0;
    for (int kt = 0; kt < nt; kt++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(RW_NS - 2) : "memory");
        __syncthreads();                       // tile kt landed for every thread's copies
        issue(kt + RW_NS - 1);                 // into the stage tile kt-1 used
        const float *f = fst + (kt % RW_NS) * RW_F_TILE;
        double *d = dt + (kt & 1) * RW_R * RW_LD;
        for (int i = tid; i < RW_F_TILE / 4; i += RW_THREADS) {   // widen once, 4 at a time
            const float4 v = reinterpret_cast<const float4 *>(f)[i];
            double *o = d + (i / (RW_K / 4)) * RW_LD + (i % (RW_K / 4)) * 4;
            reinterpret_cast<double2 *>(o)[0] = make_double2(v.x, v.y);
            reinterpret_cast<double2 *>(o)[1] = make_double2(v.z, v.w);
        }
        __syncthreads();
        const double *wr = d + el * RW_LD;
        const double *xr = d + (RW_E + tl) * RW_LD;
        const int kn = min(RW_K, hidden - kt * RW_K);
        if (kn == RW_K) {
            double2 wa[4], xa[4], wb[4], xb[4];
            load8(wa, xa, wr, xr);
#pragma unroll
            for (int c = 0; c < RW_K; c += 16) {
                load8(wb, xb, wr + c + 8, xr + c + 8);
                acc = chain8(acc, wa, xa);
                if (c + 16 < RW_K) load8(wa, xa, wr + c + 16, xr + c + 16);
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
template <int A, int B, int V>
static int router_smem_optin()
{
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        st = cuda_status(cudaFuncSetAttribute(router_scores_kernel<A, B, V>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, RbTile<A, B>::SMEM));
        if (st) return st;
        done[dev] = true;
    }
    return K3GPU_OK;
}

// The same opt-in for the one-wave kernel.
static int wave_smem_optin(bool v4)
{
    static std::mutex mu;
    static bool done[64][2] = {};
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev][v4]) {
        st = cuda_status(v4 ? cudaFuncSetAttribute(router_scores_wave_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, RW_SMEM)
                            : cudaFuncSetAttribute(router_scores_wave_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, RW_SMEM));
        if (st) return st;
        done[dev][v4] = true;
    }
    return K3GPU_OK;
}

template <int A, int B>
static int scores_launch(bool v4, float *score, const float *x, const float *W, int T, int hidden, int n,
                         cudaStream_t s)
{
    using Tl = RbTile<A, B>;
    int st = v4 ? router_smem_optin<A, B, 4>() : router_smem_optin<A, B, 1>();
    if (st) return st;
    dim3 g(ceil_div(n, Tl::TE), ceil_div(T, Tl::TT));
    if (v4) router_scores_kernel<A, B, 4><<<g, RB_THREADS, Tl::SMEM, s>>>(score, x, W, T, hidden, n);
    else router_scores_kernel<A, B, 1><<<g, RB_THREADS, Tl::SMEM, s>>>(score, x, W, T, hidden, n);
    return launch_status();
}

// Estimated clocks per hidden column of tile shape (a, b): the FP64 issue of the warps
// sharing one scheduler (2 clocks per warp FMA), the shared-memory wavefronts of the warps
// sharing one SM (a/2 broadcast loads of one wavefront, b doubles per lane at 2 wavefronts
// per 8 bytes x 32 lanes), and one chain step: an FMA latency (about 8 clocks) and its issue.
static double scores_cost(int a, int b, int T, int n, int sms)
{
    const double warps = 4.0 * ceil_div(T, 4 * a) * ceil_div(n, 32 * b);
    const double fp64 = ceil(warps / (4.0 * sms)) * 2.0 * a * b;
    const double lds = ceil(warps / sms) * (a / 2 + 2 * b);
    return fmax(fmax(fp64, lds), 10.0);
}

int router_launch(int *idx, float *w, const float *x, const float *W, const float *bias, int T,
                  int hidden, int n, int topk, int renorm, float routed_scale, float *score,
                  cudaStream_t s)
{
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const bool v4 = hidden % 4 == 0 && ((uintptr_t)x & 15u) == 0 && ((uintptr_t)W & 15u) == 0;
    const dim3 gw(ceil_div(n, RW_E), ceil_div(T, RW_T));
    if ((long long)gw.x * gw.y <= sms) {   // one wave of one-chain-per-thread CTAs
        int st = wave_smem_optin(v4);
        if (st) return st;
        if (v4) router_scores_wave_kernel<4><<<gw, RW_THREADS, RW_SMEM, s>>>(score, x, W, T, hidden, n);
        else router_scores_wave_kernel<1><<<gw, RW_THREADS, RW_SMEM, s>>>(score, x, W, T, hidden, n);
        if ((st = launch_status())) return st;
        router_topk_kernel<<<ceil_div(T, 4), 128, 0, s>>>(idx, w, score, bias, T, n, topk, renorm, routed_scale);
        return launch_status();
    }
    static const int shapes[][2] = {{8, 2}, {6, 2}, {4, 2}, {4, 1}, {2, 1}};
    int best = 0;
    double bc = 1e300;
    for (int i = 0; i < 5; i++) {
        const double c = scores_cost(shapes[i][0], shapes[i][1], T, n, sms);
        if (c < bc) { bc = c; best = i; }
    }
    int st;
    switch (best) {
    case 0: st = scores_launch<8, 2>(v4, score, x, W, T, hidden, n, s); break;
    case 1: st = scores_launch<6, 2>(v4, score, x, W, T, hidden, n, s); break;
    case 2: st = scores_launch<4, 2>(v4, score, x, W, T, hidden, n, s); break;
    case 3: st = scores_launch<4, 1>(v4, score, x, W, T, hidden, n, s); break;
    default: st = scores_launch<2, 1>(v4, score, x, W, T, hidden, n, s); break;
    }
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
