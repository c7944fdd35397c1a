// accept.cu -- on-device verify-and-accept: per-position argmax over the vocabulary,
// the longest accepted draft prefix (chain) or path (tree), the bonus token, and
// temperature sampling with the speculative rejection rule.
//
// argmax follows the reference's argmax_ (src/cli/k3_run.c:138-139): a sequential scan
// with strict '>' from index 0, i.e. the first index of the maximum over non-NaN values,
// and index 0 whenever v[0] is NaN (nothing then compares greater than it).
#include <cooperative_groups.h>
#include <math.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace k3 {

constexpr int AM_THREADS = 512;
constexpr int AM_CLUSTER = 8;      // CTAs per row: a verify sweep has too few rows to fill the GPU

__device__ __forceinline__ bool better(float ov, int oi, float bv, int bi)
{
    if (oi < 0) return false;
    if (bi < 0) return true;
    return ov > bv || (ov == bv && oi < bi);
}

__device__ __forceinline__ void warp_best(float &v, int &b)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, b, o);
        if (better(ov, oi, v, b)) { v = ov; b = oi; }
    }
}

// grid (AM_CLUSTER, min(rows, 65535)), clusters of AM_CLUSTER CTAs along x, block 512:
// arg[row] = argmax of logits[row][0..vocab). CTA r of a cluster scans chunk r of the row,
// each thread its elements in ascending order with strict '>', so within a thread the
// first index of its maximum wins; across threads and chunks ties go to the smaller index
// -- together the first index of the row maximum over non-NaN values, as the sequential
// scan finds it. Rank 0 merges the chunks' bests through distributed shared memory.
__global__ void __cluster_dims__(AM_CLUSTER, 1, 1) __launch_bounds__(AM_THREADS)
    argmax_kernel(int *__restrict__ arg, const float *__restrict__ logits, int vocab, long long rows)
{
    __shared__ float sv[AM_THREADS / 32];
    __shared__ int si[AM_THREADS / 32];
    __shared__ float cv;
    __shared__ int ci;
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    for (long long row = blockIdx.y; row < rows; row += gridDim.y) {   // uniform over the cluster
        const float *l = logits + (size_t)row * (size_t)vocab;
        float bv = -INFINITY;
        int bi = -1;
        auto take = [&](float x, int i) {
            if (x == x && (bi < 0 || x > bv)) { bv = x; bi = i; }   // NaN never a candidate
        };
        if ((vocab & 3) == 0 && (reinterpret_cast<uintptr_t>(l) & 15u) == 0) {
            const float4 *l4 = reinterpret_cast<const float4 *>(l);
            const int n4 = vocab / 4, per = (n4 + AM_CLUSTER - 1) / AM_CLUSTER;
            const int j1 = min(n4, (rank + 1) * per);
            for (int j = rank * per + (int)threadIdx.x; j < j1; j += AM_THREADS) {
                const float4 x = __ldg(l4 + j);
                take(x.x, 4 * j);
                take(x.y, 4 * j + 1);
                take(x.z, 4 * j + 2);
                take(x.w, 4 * j + 3);
            }
        } else {
            const int per = (vocab + AM_CLUSTER - 1) / AM_CLUSTER;
            const int i1 = min(vocab, (rank + 1) * per);
            for (int i = rank * per + (int)threadIdx.x; i < i1; i += AM_THREADS) take(l[i], i);
        }
        warp_best(bv, bi);
        if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < AM_THREADS / 32 ? sv[threadIdx.x] : -INFINITY;
            int b = threadIdx.x < AM_THREADS / 32 ? si[threadIdx.x] : -1;
            warp_best(v, b);
            if (threadIdx.x == 0) { cv = v; ci = b; }
        }
        cl.sync();
        if (rank == 0 && threadIdx.x < 32) {
            float v = -INFINITY;
            int b = -1;
            if (threadIdx.x < AM_CLUSTER) {
                v = *cl.map_shared_rank(&cv, threadIdx.x);
                b = *cl.map_shared_rank(&ci, threadIdx.x);
            }
            warp_best(v, b);
            if (threadIdx.x == 0) {
                // the sequential scan keeps index 0 if l[0] is NaN (no value compares greater)
                // and when every value is NaN
                if (l[0] != l[0] || b < 0) b = 0;
                arg[row] = b;
            }
        }
        cl.sync();   // the chunks' bests stay readable until rank 0 has merged them
    }
}

// one thread per sequence: m = longest prefix with arg == draft, emit draft[0..m) + arg[m]
__global__ void accept_chain_kernel(int *__restrict__ emit, int *__restrict__ n_emit,
                                    const int *__restrict__ arg, const int *__restrict__ drafts,
                                    const int *__restrict__ nd_b, int B, int nd)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int n = nd_b ? nd_b[b] : nd;
    if (n < 0 || n > nd) {
        flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : nd;
    }
    const int *a = arg + (size_t)b * (nd + 1);
    const int *d = drafts + (size_t)b * nd;
    int *e = emit + (size_t)b * (nd + 1);
    int m = 0;
    while (m < n && a[m] == d[m]) {
        e[m] = d[m];
        m++;
    }
    e[m] = a[m];
    n_emit[b] = m + 1;
}

// one thread per sequence over a tree of T nodes in topological (index) order
__global__ void accept_tree_kernel(int *__restrict__ emit, int *__restrict__ n_emit,
                                   int *__restrict__ path, const int *__restrict__ arg,
                                   const int *__restrict__ tok, const int *__restrict__ parent,
                                   int B, int T)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int *a = arg + (size_t)b * T;
    const int *tk = tok + (size_t)b * T;
    int *pth = path + (size_t)b * T;
    int *e = emit + (size_t)b * T;
    // walk down from the root: the accepted child of node c is its lowest-index child
    // whose drafted id equals argmax(c); children have larger indices than parents
    int c = 0, depth = 0;
    pth[0] = 0;
    for (;;) {
        int next = -1;
        for (int i = c + 1; i < T; i++) {
            const int pi = parent[i];
            if (pi < 0 || pi >= i) { flag(DEV_BAD_INDEX); continue; }
            if (pi == c && tk[i] == a[c]) { next = i; break; }
        }
        if (next < 0) break;
        e[depth] = tk[next];
        depth++;
        pth[depth] = next;
        c = next;
    }
    e[depth] = a[c];
    n_emit[b] = depth + 1;
}

// ---------------------------------------------------------------- sampling ------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2,
// 3", SC'11): 10 rounds of two 32x32->64 multiplies with the published multipliers and
// Weyl key increments.
__host__ __device__ inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1)
{
    for (int r = 0; r < 10; r++) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

// A uniform double in [0, 1) with 53 random bits for draw `which` of position i of
// sequence b: counter (offset lo, offset hi, b, 2*i + which), key (seed lo, seed hi).
__host__ __device__ inline double philox_uniform(uint64_t seed, uint64_t offset, int b, int i,
                                                 int which)
{
    uint32_t c[4] = {(uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)b,
                     (uint32_t)(2 * i + which)};
    philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    const uint64_t bits = ((uint64_t)(c[0] >> 5) << 26) | (uint64_t)(c[1] >> 6);
    return (double)bits * (1.0 / 9007199254740992.0);
}

constexpr int SM_THREADS = 256;

// e_v = exp((l_v - m) / temp) in float with a correctly rounded exp
__device__ __forceinline__ float samp_e(float l, float m, float temp)
{
    return expf_cr(__fdiv_rn(__fsub_rn(l, m), temp));
}

// The fixed reduction order shared with the CPU restatement: thread t owns the
// contiguous chunk [t*C, min((t+1)*C, vocab)), sums it ascending in double, and the 256
// chunk sums are added in thread order. `skip` (-1 for none) is left out of the sums.
__device__ double chunk_sum(const float *l, int vocab, float m, float temp, int skip,
                            double *csum /* [SM_THREADS] shared */)
{
    const int C = (vocab + SM_THREADS - 1) / SM_THREADS;
    const int v0 = threadIdx.x * C, v1 = min(vocab, v0 + C);
    double s = 0.0;
    for (int v = v0; v < v1; v++)
        if (v != skip && l[v] == l[v]) s += (double)samp_e(l[v], m, temp);
    csum[threadIdx.x] = s;
    __syncthreads();
    double tot = 0.0;
    for (int t = 0; t < SM_THREADS; t++) tot += csum[t];
    return tot;
}

// Inverse CDF over the same chunk order: the first v (v != skip) whose running sum
// exceeds r; if rounding leaves r at or past the total, the last v with e_v > 0.
__device__ int chunk_pick(const float *l, int vocab, float m, float temp, int skip, double r,
                          const double *csum, int *sh_pick)
{
    const int C = (vocab + SM_THREADS - 1) / SM_THREADS;
    if (threadIdx.x == 0) {
        double run = 0.0;
        int pick = -1, last = -1;
        for (int t = 0; t < SM_THREADS && pick < 0; t++) {
            if (run + csum[t] > r) {
                const int v0 = t * C, v1 = min(vocab, v0 + C);
                for (int v = v0; v < v1; v++) {
                    if (v == skip || l[v] != l[v]) continue;
                    run += (double)samp_e(l[v], m, temp);
                    if (run > r) { pick = v; break; }
                }
                break;   // not found inside the chunk (rounding): the fallback below
            } else {
                run += csum[t];
            }
        }
        if (pick < 0) {
            for (int v = vocab - 1; v >= 0; v--)
                if (v != skip && l[v] == l[v] && samp_e(l[v], m, temp) > 0.0f) { last = v; break; }
            pick = last >= 0 ? last : 0;
        }
        *sh_pick = pick;
    }
    __syncthreads();
    return *sh_pick;
}

__device__ float block_max_nonnan(const float *l, int vocab, float *red)
{
    float m = -INFINITY;
    for (int v = threadIdx.x; v < vocab; v += SM_THREADS) {
        const float x = l[v];
        if (x == x && x > m) m = x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < SM_THREADS / 32; w++) r = fmaxf(r, red[w]);
    return r;
}

// one CTA per sequence; positions are decided in order, so the kernel stops at the first
// rejection and reads no later position's logits
__global__ void __launch_bounds__(SM_THREADS) accept_sample_kernel(
    int *__restrict__ emit, int *__restrict__ n_emit, const float *__restrict__ logits,
    const int *__restrict__ drafts, const int *__restrict__ nd_b, int nd, int vocab,
    float temp, uint64_t seed, uint64_t offset)
{
    __shared__ double csum[SM_THREADS];
    __shared__ float red[SM_THREADS / 32];
    __shared__ int pick;
    const int b = blockIdx.x;
    int n = nd_b ? nd_b[b] : nd;
    if (n < 0 || n > nd) {
        if (threadIdx.x == 0) flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : nd;
    }
    int *e = emit + (size_t)b * (nd + 1);
    for (int i = 0; i <= n; i++) {
        const float *l = logits + ((size_t)b * (nd + 1) + i) * vocab;
        const float m = block_max_nonnan(l, vocab, red);
        const double Z = chunk_sum(l, vocab, m, temp, -1, csum);
        __syncthreads();
        if (i == n) {   // every draft accepted: the bonus from p_n
            const double r = philox_uniform(seed, offset, b, i, 1) * Z;
            const int v = chunk_pick(l, vocab, m, temp, -1, r, csum, &pick);
            if (threadIdx.x == 0) { e[i] = v; n_emit[b] = i + 1; }
            return;
        }
        const int d = drafts[(size_t)b * nd + i];
        const bool ok_d = d >= 0 && d < vocab && l[d] == l[d];
        const double pd = ok_d ? (double)samp_e(l[d], m, temp) / Z : 0.0;
        const double u = philox_uniform(seed, offset, b, i, 0);
        if (u < pd) {
            if (threadIdx.x == 0) e[i] = d;
            __syncthreads();
            continue;
        }
        // rejected: draw from p_i with the draft removed, renormalised
        const double Zr = chunk_sum(l, vocab, m, temp, ok_d ? d : -1, csum);
        __syncthreads();
        const double r = philox_uniform(seed, offset, b, i, 1) * Zr;
        const int v = chunk_pick(l, vocab, m, temp, ok_d ? d : -1, r, csum, &pick);
        if (threadIdx.x == 0) { e[i] = v; n_emit[b] = i + 1; }
        return;
    }
}

}  // namespace k3

extern "C" int k3gpu_accept_sample(int *emit, int *n_emit, const float *logits,
                                   const int *drafts, const int *nd_b, int B, int nd, int vocab,
                                   float temp, uint64_t seed, uint64_t offset, void *stream)
{
    if (!emit || !n_emit || !logits || (!drafts && nd > 0)) return K3GPU_EINVAL;
    if (B <= 0 || nd < 0 || nd > 1024 || vocab <= 0 || !(temp > 0.0f)) return K3GPU_EINVAL;
    k3::accept_sample_kernel<<<B, k3::SM_THREADS, 0, k3::as_stream(stream)>>>(
        emit, n_emit, logits, drafts, nd_b, nd, vocab, temp, seed, offset);
    return k3::launch_status();
}

extern "C" int k3gpu_accept_greedy(int *emit, int *n_emit, int *arg, const float *logits,
                                   const int *drafts, const int *nd_b, int B, int nd, int vocab,
                                   void *stream)
{
    if (!emit || !n_emit || !arg || (!drafts && nd > 0)) return K3GPU_EINVAL;
    if (B <= 0 || nd < 0 || nd > 1024 || (logits && vocab <= 0)) return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    const long long rows = (long long)B * (nd + 1);
    int st;
    if (logits) {   // else arg already holds every position's argmax (k3gpu_model_verify_greedy)
        k3::argmax_kernel<<<dim3(k3::AM_CLUSTER, (unsigned)std::min(rows, 65535LL)), k3::AM_THREADS, 0, s>>>(
            arg, logits, vocab, rows);
        if ((st = k3::launch_status())) return st;
    }
    k3::accept_chain_kernel<<<k3::ceil_div(B, 128), 128, 0, s>>>(emit, n_emit, arg, drafts, nd_b,
                                                                  B, nd);
    return k3::launch_status();
}

extern "C" int k3gpu_argmax(int *arg, const float *logits, int rows, int vocab, void *stream)
{
    if (!arg || !logits || rows <= 0 || vocab <= 0) return K3GPU_EINVAL;
    k3::argmax_kernel<<<dim3(k3::AM_CLUSTER, (unsigned)std::min(rows, 65535)), k3::AM_THREADS, 0,
                        k3::as_stream(stream)>>>(arg, logits, vocab, rows);
    return k3::launch_status();
}

extern "C" int k3gpu_accept_tree_greedy(int *emit, int *n_emit, int *path, int *arg,
                                        const float *logits, const int *tok, const int *parent,
                                        int B, int T, int vocab, void *stream)
{
    if (!emit || !n_emit || !path || !arg || !tok || !parent) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 4096 || (logits && vocab <= 0)) return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    const long long rows = (long long)B * T;
    int st;
    if (logits) {   // else arg already holds every node's argmax (k3gpu_model_verify_greedy)
        k3::argmax_kernel<<<dim3(k3::AM_CLUSTER, (unsigned)std::min(rows, 65535LL)), k3::AM_THREADS, 0, s>>>(
            arg, logits, vocab, rows);
        if ((st = k3::launch_status())) return st;
    }
    k3::accept_tree_kernel<<<k3::ceil_div(B, 128), 128, 0, s>>>(emit, n_emit, path, arg, tok,
                                                                 parent, B, T);
    return k3::launch_status();
}
