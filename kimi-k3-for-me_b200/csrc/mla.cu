// mla.cu -- absorbed MLA over the compressed latent cache with a chain or tree mask
// (the --mla-absorb branch of k3_mla_cached, src/core/k3_ops.c:1417-1540 of the
// reference, generalised from its causal rule s <= cached + t to per-node ancestor masks).
//
//   qabs     q_abs[h] = W_uk[h]^T q_nope[h] in fp32 (the reference forms it in double and
//            rounds to float, :1443-1461).
//   attend   split over cache positions (flash-decoding): each CTA takes 8 heads of one
//            query node and one slice of positions, streams bf16 latent+rope rows through
//            shared memory 32 at a time, and keeps an online-softmax state per head:
//            running max, running sum and u = sum p * lat. Partial states go to the
//            workspace.
//   merge    merges the slices of each (node, head) into u (over q_abs's buffer).
//   out      out = W_uv[h] u, a register-tiled product per head.
//
// Scores are fp32 dot products of fp32 queries with the bf16 cache (the cache is the
// compressed latent the reference stores in fp32; here it is held in bf16 in HBM, half
// the bytes). The softmax uses the slice maxima and fp32 exps; tolerance-level against
// the reference's double normaliser.
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace k3 {

constexpr int MLA_HT = 8;        // heads per CTA
constexpr int MLA_PT = 32;       // positions per shared-memory tile
constexpr int MLA_SPLIT = 512;   // positions per split (one CTA's slice)
constexpr int MLA_THREADS = 256;
constexpr int MLA_MAXL = 512;    // kv_lora upper bound
constexpr int MLA_MAXR = 64;     // qk_rope upper bound
constexpr int MLA_MAXSPLIT = 256;   // slices per (node, head): max_ctx <= 131072
constexpr size_t MLA_SMEM =
    sizeof(float) * ((size_t)MLA_HT * (MLA_MAXL + MLA_MAXR) + (size_t)MLA_PT * (MLA_MAXL + MLA_MAXR + 1));

struct MlaWs {
    float *qabs;   // [B][T][H][kvl]
    float *pm;     // [B][T][H][nsplit] running max
    float *pl;     // [B][T][H][nsplit] running sum
    float *pu;     // [B][T][H][nsplit][kvl]
    uint16_t *qh, *ql;   // tensor-core path: [B][T][H][kvl + qr] bf16 pieces of [q_abs | q_rope]
};

static size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

static size_t mla_ws_layout(int B, int T, int H, int kvl, int qr, int ns, MlaWs *w, char *base)
{
    const size_t rows = (size_t)B * T * H;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += a256(bytes);
        return r;
    };
    char *qa = take(rows * kvl * 4), *pm = take(rows * ns * 4), *pl = take(rows * ns * 4);
    char *pu = take(rows * ns * (size_t)kvl * 4);
    char *qh = take(rows * (size_t)(kvl + qr) * 2), *ql = take(rows * (size_t)(kvl + qr) * 2);
    if (w) {
        w->qabs = (float *)qa; w->pm = (float *)pm; w->pl = (float *)pl; w->pu = (float *)pu;
        w->qh = (uint16_t *)qh; w->ql = (uint16_t *)ql;
    }
    return o;
}

// grid (H, ceil(B*T / QB_T), ceil(kvl / QB_J)), block 256: qabs[bt][h][j] = sum_i
// W[h*kvd + i][j] * q_nope[bt][h][i], i ascending (one fma chain per output). A block
// computes 64 query nodes x 128 columns of one head, the operands staged through shared
// memory 32 values of i at a time (the next chunk's loads in flight during this chunk's
// fmas); thread (ty, tx) holds the 8 x 4 outputs of nodes 8 ty.. and columns 4 tx.. in
// registers (two broadcast float4 loads and one float4 load per 32 fmas).
constexpr int QB_T = 64, QB_J = 128, QB_K = 32, QB_AS = QB_T + 4;
__global__ void __launch_bounds__(256) mla_qabs_kernel(float *__restrict__ qabs,
                                                       const float *__restrict__ q_nope,
                                                       const float *__restrict__ kv_b, int BT, int H,
                                                       int qn, int vh, int kvl)
{
    __shared__ __align__(16) float As[QB_K][QB_AS];  // q_nope chunk [i][node], padded rows
    __shared__ __align__(16) float Bs[QB_K][QB_J];   // W_uk chunk [i][column]
    const int h = blockIdx.x, bt0 = blockIdx.y * QB_T, j0 = blockIdx.z * QB_J;
    const int kvd = qn + vh;
    const int ty = threadIdx.x >> 5, tx = threadIdx.x & 31;
    float acc[8][4];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[r][c] = 0.0f;
    // a chunk's operands: 8 values of q_nope and 16 of W_uk per thread, all loads issued
    // before any is used; the next chunk's are in flight during this chunk's fmas
    float ra[QB_K * QB_T / 256], rb[QB_K * QB_J / 256];
    auto fetch = [&](int i0) {
        const int kn = min(QB_K, qn - i0);
#pragma unroll
        for (int k = 0; k < QB_K * QB_T / 256; k++) {
            const int x = threadIdx.x + 256 * k, i = x % QB_K, t = x / QB_K;
            ra[k] = (bt0 + t < BT && i < kn) ? q_nope[((size_t)(bt0 + t) * H + h) * qn + i0 + i] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < QB_K * QB_J / 256; k++) {
            const int x = threadIdx.x + 256 * k, j = x % QB_J, i = x / QB_J;
            rb[k] = (j0 + j < kvl && i < kn) ? kv_b[((size_t)h * kvd + i0 + i) * kvl + j0 + j] : 0.0f;
        }
    };
    fetch(0);
    for (int i0 = 0; i0 < qn; i0 += QB_K) {
        const int kn = min(QB_K, qn - i0);
        __syncthreads();
        // a warp read 32 consecutive i of one node (coalesced) and stores them down a
        // column of As (the padded rows keep that at 4-way bank conflicts)
#pragma unroll
        for (int k = 0; k < QB_K * QB_T / 256; k++) {
            const int x = threadIdx.x + 256 * k;
            As[x % QB_K][x / QB_K] = ra[k];
        }
#pragma unroll
        for (int k = 0; k < QB_K * QB_J / 256; k++) {
            const int x = threadIdx.x + 256 * k;
            Bs[x / QB_J][x % QB_J] = rb[k];
        }
        __syncthreads();
        if (i0 + QB_K < qn) fetch(i0 + QB_K);
#pragma unroll 4
        for (int i = 0; i < kn; i++) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[i][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[i][ty * 8 + 4]);
            const float4 b4 = *reinterpret_cast<const float4 *>(&Bs[i][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int r = 0; r < 8; r++)
#pragma unroll
                for (int c = 0; c < 4; c++) acc[r][c] = fmaf(bv[c], av[r], acc[r][c]);
        }
    }
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const int t = bt0 + ty * 8 + r;
        if (t >= BT) break;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = j0 + tx * 4 + c;
            if (j < kvl) qabs[((size_t)t * H + h) * kvl + j] = acc[r][c];
        }
    }
}

__device__ __forceinline__ float bf2f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// grid (nsplit, B*T, H/MLA_HT): one query node, MLA_HT heads, one slice of positions
__global__ void __launch_bounds__(MLA_THREADS) mla_attend_kernel(
    MlaWs w, const float *__restrict__ q_rope, const uint16_t *__restrict__ lat,
    const uint16_t *__restrict__ rope, const int *__restrict__ cached,
    const uint64_t *__restrict__ mask, int T, int H, int qr, int kvl, int cap, int nsplit,
    float scale)
{
    extern __shared__ float mla_dyn[];
    float (*sq)[MLA_MAXL + MLA_MAXR] = reinterpret_cast<float (*)[MLA_MAXL + MLA_MAXR]>(mla_dyn);
    float (*skv)[MLA_MAXL + MLA_MAXR + 1] =
        reinterpret_cast<float (*)[MLA_MAXL + MLA_MAXR + 1]>(mla_dyn + MLA_HT * (MLA_MAXL + MLA_MAXR));
    __shared__ float ss[MLA_HT][MLA_PT];
    __shared__ float sm[MLA_HT], sl[MLA_HT], salpha[MLA_HT];
    const int split = blockIdx.x, bt = blockIdx.y, h0 = blockIdx.z * MLA_HT;
    const int b = bt / T, t = bt % T;
    const int kw = kvl + qr;
    const int c = cached[b];
    const int n_ctx = c + T;
    const int s_begin = split * MLA_SPLIT, s_end = min(n_ctx, s_begin + MLA_SPLIT);
    const size_t prow = ((size_t)bt * H) * nsplit;   // + h * nsplit + split
    if (n_ctx > cap) {   // the new rows would lie past the cache
        if (threadIdx.x == 0) flag(DEV_BAD_POSITION);
        return;
    }
    // queries: [q_abs | q_rope] per head
    for (int i = threadIdx.x; i < MLA_HT * kw; i += MLA_THREADS) {
        const int hh = i / kw, d = i % kw, h = h0 + hh;
        float v = 0.0f;
        if (h < H)
            v = d < kvl ? w.qabs[((size_t)bt * H + h) * kvl + d]
                        : q_rope[((size_t)bt * H + h) * qr + (d - kvl)];
        sq[hh][d] = v;
    }
    if (threadIdx.x < MLA_HT) {
        sm[threadIdx.x] = -INFINITY;
        sl[threadIdx.x] = 0.0f;
    }
    // u accumulators: thread owns (head hh = tid / 32, columns lane, lane+32, ...)
    const int hh_u = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float u[MLA_MAXL / 32];
#pragma unroll
    for (int k = 0; k < MLA_MAXL / 32; k++) u[k] = 0.0f;
    const uint64_t mk = mask[t];
    const uint16_t *latb = lat + (size_t)b * cap * kvl;
    const uint16_t *ropeb = rope + (size_t)b * cap * qr;
    for (int p0 = s_begin; p0 < s_end; p0 += MLA_PT) {
        const int np = min(MLA_PT, s_end - p0);
        __syncthreads();
        for (int i = threadIdx.x; i < MLA_PT * kw; i += MLA_THREADS) {
            const int r = i / kw, d = i % kw, s = p0 + r;
            float v = 0.0f;
            if (r < np) v = d < kvl ? bf2f(latb[(size_t)s * kvl + d]) : bf2f(ropeb[(size_t)s * qr + (d - kvl)]);
            skv[r][d] = v;
        }
        __syncthreads();
        // scores: 256 threads over MLA_HT x MLA_PT = 256 (head, position) pairs
        {
            const int hh = threadIdx.x / MLA_PT, r = threadIdx.x % MLA_PT, s = p0 + r;
            bool vis = r < np && (h0 + hh) < H;
            if (vis && s >= c) vis = ((mk >> (s - c)) & 1ull) != 0;
            float d = 0.0f;
            if (vis) {
                for (int i = 0; i < kw; i++) d = fmaf(sq[hh][i], skv[r][i], d);
                d *= scale;
            }
            ss[hh][r] = vis ? d : -INFINITY;
        }
        __syncthreads();
        // online softmax per head (one warp per head, lane = position)
        {
            const int hh = threadIdx.x >> 5;
            const float x = ss[hh][lane];
            float m = x;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float mold = sm[hh];
            const float mnew = fmaxf(mold, m);
            const float p = mnew == -INFINITY ? 0.0f : __expf(x - mnew);
            float sum = p;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            ss[hh][lane] = p;
            __syncwarp();
            if (lane == 0) {
                const float al = (mold == -INFINITY) ? 0.0f : __expf(mold - mnew);
                salpha[hh] = al;
                sl[hh] = sl[hh] * al + sum;
                sm[hh] = mnew;
            }
        }
        __syncthreads();
        {
            const float al = salpha[hh_u];
#pragma unroll
            for (int k = 0; k < MLA_MAXL / 32; k++) u[k] *= al;
            for (int r = 0; r < np; r++) {
                const float p = ss[hh_u][r];
                if (p == 0.0f) continue;
#pragma unroll
                for (int k = 0; k < MLA_MAXL / 32; k++) {
                    const int j = lane + 32 * k;
                    if (j < kvl) u[k] = fmaf(p, skv[r][j], u[k]);
                }
            }
        }
    }
    __syncthreads();
    const int h = h0 + hh_u;
    if (h < H) {
        const size_t pi = prow + (size_t)h * nsplit + split;
        if (lane == 0) {
            w.pm[pi] = sm[hh_u];
            w.pl[pi] = sl[hh_u];
        }
#pragma unroll
        for (int k = 0; k < MLA_MAXL / 32; k++) {
            const int j = lane + 32 * k;
            if (j < kvl) w.pu[pi * kvl + j] = u[k];
        }
    }
}

// grid (ceil(H / MG_H), B*T), block 256: merge the slices of one query node for MG_H heads
// into u[node][h][:] (written over q_abs, which the attention has consumed). The merge
// weights of each (node, head) come from one thread in slice order -- the maximum,
// exp(m_s - M), the weighted sum of the slice sums, the reciprocal -- then u[j] = sum_s
// w_s u_s[j] is one fma chain over the slices; each slice's loads for the thread's 8 heads
// x 2 columns are issued together (coalesced over j).
constexpr int MG_H = 8, MG_J = MLA_MAXL / 256;
__global__ void __launch_bounds__(256) mla_merge_kernel(float *__restrict__ u, MlaWs w,
                                                        const int *__restrict__ cached, int T, int H,
                                                        int kvl, int nsplit, int split_len)
{
    __shared__ float sw[MG_H][MLA_MAXSPLIT];
    const int bt = blockIdx.y, h0 = blockIdx.x * MG_H;
    const int n_ctx = cached[bt / T] + T;
    const int nsu = max(0, min(nsplit, (n_ctx + split_len - 1) / split_len));
    if (threadIdx.x < MG_H && h0 + (int)threadIdx.x < H) {
        const int r = threadIdx.x;
        const size_t base = ((size_t)bt * H + h0 + r) * nsplit;
        float M = -INFINITY;
        for (int s = 0; s < nsu; s++) M = fmaxf(M, w.pm[base + s]);
        float Lsum = 0.0f;
        for (int s = 0; s < nsu; s++) {
            const float f = w.pm[base + s] == -INFINITY ? 0.0f : __expf(w.pm[base + s] - M);
            sw[r][s] = f;
            Lsum += f * w.pl[base + s];
        }
        const float inv = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
        for (int s = 0; s < nsu; s++) sw[r][s] *= inv;
    }
    __syncthreads();
    float a[MG_H][MG_J];
#pragma unroll
    for (int r = 0; r < MG_H; r++)
#pragma unroll
        for (int q = 0; q < MG_J; q++) a[r][q] = 0.0f;
    for (int s = 0; s < nsu; s++) {
        float v[MG_H][MG_J];
#pragma unroll
        for (int r = 0; r < MG_H; r++)
#pragma unroll
            for (int q = 0; q < MG_J; q++) {
                const int j = threadIdx.x + 256 * q;
                v[r][q] = (h0 + r < H && j < kvl) ? w.pu[(((size_t)bt * H + h0 + r) * nsplit + s) * kvl + j] : 0.0f;
            }
#pragma unroll
        for (int r = 0; r < MG_H; r++)
#pragma unroll
            for (int q = 0; q < MG_J; q++) a[r][q] = fmaf(sw[r][s], v[r][q], a[r][q]);
    }
#pragma unroll
    for (int r = 0; r < MG_H; r++)
#pragma unroll
        for (int q = 0; q < MG_J; q++) {
            const int j = threadIdx.x + 256 * q;
            if (h0 + r < H && j < kvl) u[((size_t)bt * H + h0 + r) * kvl + j] = a[r][q];
        }
}

// grid (H, ceil(B*T / OB_T), ceil(vh / OB_R)), block 256: out[node][h][r] = sum_j
// W_uv[h][r][j] u[node][h][j], one fma chain over j ascending. A block computes 64 nodes x
// 128 rows of one head, the operands staged through shared memory 32 values of j at a time
// (the next chunk's loads in flight during this chunk's fmas, both read coalesced over j
// and stored down columns of padded rows); thread (ty, tx) holds nodes 8 ty.. x rows 4 tx..
constexpr int OB_T = 64, OB_R = 128, OB_K = 32;
constexpr int OB_AS = OB_T + 4, OB_BS = OB_R + 4;
__global__ void __launch_bounds__(256, 2) mla_out_kernel(float *__restrict__ out, const float *__restrict__ u,
                                                      const float *__restrict__ kv_b, int BT, int H, int qn,
                                                      int vh, int kvl)
{
    __shared__ __align__(16) float As[OB_K][OB_AS];   // u chunk [j][node]
    __shared__ __align__(16) float Bs[OB_K][OB_BS];   // W_uv chunk [j][row]
    const int h = blockIdx.x, bt0 = blockIdx.y * OB_T, r0 = blockIdx.z * OB_R;
    const int kvd = qn + vh;
    const int ty = threadIdx.x >> 5, tx = threadIdx.x & 31;
    float acc[8][4];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[r][c] = 0.0f;
    float ra[OB_K * OB_T / 256], rb[OB_K * OB_R / 256];
    auto fetch = [&](int j0) {
        const int kn = min(OB_K, kvl - j0);
#pragma unroll
        for (int k = 0; k < OB_K * OB_T / 256; k++) {
            const int x = threadIdx.x + 256 * k, j = x % OB_K, t = x / OB_K;
            ra[k] = (bt0 + t < BT && j < kn) ? u[((size_t)(bt0 + t) * H + h) * kvl + j0 + j] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < OB_K * OB_R / 256; k++) {
            const int x = threadIdx.x + 256 * k, j = x % OB_K, r = x / OB_K;
            rb[k] = (j < kn && r0 + r < vh) ? kv_b[((size_t)h * kvd + qn + r0 + r) * kvl + j0 + j] : 0.0f;
        }
    };
    fetch(0);
    for (int j0 = 0; j0 < kvl; j0 += OB_K) {
        const int kn = min(OB_K, kvl - j0);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < OB_K * OB_T / 256; k++) {
            const int x = threadIdx.x + 256 * k;
            As[x % OB_K][x / OB_K] = ra[k];
        }
#pragma unroll
        for (int k = 0; k < OB_K * OB_R / 256; k++) {
            const int x = threadIdx.x + 256 * k;
            Bs[x % OB_K][x / OB_K] = rb[k];
        }
        __syncthreads();
        if (j0 + OB_K < kvl) fetch(j0 + OB_K);
#pragma unroll 4
        for (int j = 0; j < kn; j++) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[j][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[j][ty * 8 + 4]);
            const float4 b4 = *reinterpret_cast<const float4 *>(&Bs[j][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int r = 0; r < 8; r++)
#pragma unroll
                for (int c = 0; c < 4; c++) acc[r][c] = fmaf(bv[c], av[r], acc[r][c]);
        }
    }
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const int t = bt0 + ty * 8 + r;
        if (t >= BT) break;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int rr = r0 + tx * 4 + c;
            if (rr < vh) out[((size_t)t * H + h) * vh + rr] = acc[r][c];
        }
    }
}

// ------------------------------------------------------------------ tensor cores -----
// The same attention on tcgen05 for kv_lora in {128, 256, 512} and qk_rope in {0, 64}. All
// H heads of a query node read the same latent rows, so one sequence's T*H query rows
// against its cache rows is a pair of GEMMs with a softmax between them:
//   S [rows x positions] = [q_abs | q_rope] . [lat | rope]^T        (K = kvl + qr)
//   u [rows x kvl]      += softmax(S) . lat                          (K = positions)
// A CTA takes 128 query rows, one half of u's kvl columns and one slice of positions
// (flash-decoding: slices merge in mla_merge_kernel), 128 positions per tile:
//   warp 0      TMA, score ring: per tile and 64-column atom, Q hi, Q lo and the cache atom
//   warp 1      TMA, value ring: the tile's latent atoms of this half, two per stage
//   warp 2      score MMAs (one thread): S = Qhi.C + Qlo.C into one of two TMEM buffers
//   warp 3      value MMAs (one thread): u += Phi.V + Plo.V with P read from TMEM and V an
//               MN-major operand straight from the cache tile (N = 128: two atoms per MMA)
//   warps 4-11  softmax, two warps per TMEM lane quarter (64 positions each), one query row
//               per lane: masked scores, a running max in log2 units that moves only when
//               a tile's max exceeds it by more than 2^11 (then the row of u in TMEM is
//               rescaled), exps summed in fp32, P split into exact-enough bf16 hi and lo
//               pieces written over the scores they came from; at the end the row's m, l
//               and u go to the workspace
// A tile's S/P buffer is reused two tiles later, once its value MMAs have completed, so
// the softmax of tile j+1 overlaps the value product of tile j. The fp32 queries enter as
// bf16 hi + lo (x = hi + lo to 2^-17 relative) and the cache is bf16, so every product is
// exact in the fp32 accumulator; P likewise. TMEM: S/P buffers at columns 0 and 128, u's
// half at 256..511 (P of 32 positions: 16 columns of hi pairs, then 16 of lo pairs, in
// place of those positions' scores). Every wait is bounded; TMEM is freed on every exit
// path; no TMA multicast.
namespace mlatc {
using namespace tc;

constexpr int NP = 128;                     // positions per tile
constexpr int ATOM = 128 * 128;             // 128 rows x 128 bytes
constexpr int QSTAGE = 3 * ATOM;            // Q hi, Q lo, cache atom
constexpr int NSQ = 3;
constexpr int VSTAGE = 2 * ATOM;            // two latent atoms (128 columns of u)
constexpr int NSV = 2;
constexpr int V_OFF = NSQ * QSTAGE;
constexpr int X_OFF = V_OFF + NSV * VSTAGE; // row max exchange [2][2][128], row sums [128]
constexpr int BAR_OFF = X_OFF + 5 * 128 * 4;
// qfull, qempty, vfull, vempty, s_full[2], p_full[2], pv_done[2], o_full, fin_q, fin_v
constexpr int NBAR = 2 * NSQ + 2 * NSV + 6 + 3;
constexpr int SMEM = BAR_OFF + NBAR * 8 + 16 + 1024;   // + room to align the base to 1024
constexpr int NSOFT = 8;
constexpr int THREADS = (4 + NSOFT) * 32;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float RESCALE_AT = 11.0f;         // log2 units
constexpr int SMS_PLAN = 148;               // the split plan assumes a full B200
static_assert(SMEM <= 227 * 1024, "shared memory");

struct Args {
    float *pm, *pl, *pu;                    // workspace partial states
    const int *cached;
    const uint64_t *mask;
    int T, H, R, kvl, qr, cap, nsplit, split_len, qa;
    float scale;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo_elem, float hi_elem)
{
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo_elem, hi_elem);
    return *reinterpret_cast<const uint32_t *>(&v);
}
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// grid B*R, block 128: [q_abs | q_rope] -> bf16 hi, lo pieces
__global__ void __launch_bounds__(128) prep_kernel(uint16_t *__restrict__ qh, uint16_t *__restrict__ ql,
                                                   const float *__restrict__ qabs,
                                                   const float *__restrict__ q_rope, int kvl, int qr)
{
    const size_t row = blockIdx.x;
    const int kq = kvl + qr;
    for (int d = threadIdx.x; d < kq; d += blockDim.x) {
        const float x = d < kvl ? qabs[row * kvl + d] : q_rope[row * qr + (d - kvl)];
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
        qh[row * kq + d] = __bfloat16_as_ushort(hi);
        ql[row * kq + d] = __bfloat16_as_ushort(lo);
    }
}

__global__ void __launch_bounds__(THREADS, 1) attend_kernel(const __grid_constant__ CUtensorMap qhmap,
                                                            const __grid_constant__ CUtensorMap qlmap,
                                                            const __grid_constant__ CUtensorMap latmap,
                                                            const __grid_constant__ CUtensorMap ropemap, Args a)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = s_addr(smem_raw);
    unsigned char *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BAR_OFF);
    uint64_t *b_qfull = bars, *b_qempty = bars + NSQ, *b_vfull = bars + 2 * NSQ, *b_vempty = b_vfull + NSV;
    uint64_t *b_sfull = b_vempty + NSV, *b_pfull = b_sfull + 2, *b_pvdone = b_pfull + 2;
    uint64_t *b_ofull = b_pvdone + 2, *b_finq = b_ofull + 1, *b_finv = b_finq + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    float *xmax = reinterpret_cast<float *>(smem + X_OFF);     // [2 tiles][2 halves][128]
    float *xsum = xmax + 4 * 128;                              // [128]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sp = blockIdx.x, qt = blockIdx.y >> 1, hf = blockIdx.y & 1, b = blockIdx.z;
    const int q0 = qt * 128;
    const int va = a.kvl / 128;                 // latent atoms of this half
    const int vw = va < 2 ? va : 2;             // atoms per value stage
    const int nvs = va / vw;                    // value stages per tile
    const int c = a.cached[b];
    const int n_ctx = c + a.T;
    const bool bad = c < 0 || n_ctx > a.cap;    // the new rows would lie outside the cache
    const int begin = sp * a.split_len;
    const int end = bad ? begin : min(n_ctx, begin + a.split_len);
    const int ntile = end > begin ? (end - begin + NP - 1) / NP : 0;
    if (bad && tid == 0 && sp == 0 && blockIdx.y == 0) flag(DEV_BAD_POSITION);

    if (tid == 0) {
        for (int s = 0; s < NSQ; s++) {
            bar_init(s_addr(&b_qfull[s]), 1);
            bar_init(s_addr(&b_qempty[s]), 1);
        }
        for (int s = 0; s < NSV; s++) {
            bar_init(s_addr(&b_vfull[s]), 1);
            bar_init(s_addr(&b_vempty[s]), 1);
        }
        for (int i = 0; i < 2; i++) {
            bar_init(s_addr(&b_sfull[i]), 1);
            bar_init(s_addr(&b_pfull[i]), NSOFT);
            bar_init(s_addr(&b_pvdone[i]), 1);
        }
        bar_init(s_addr(b_ofull), 1);
        bar_init(s_addr(b_finq), 1);
        bar_init(s_addr(b_finv), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s_addr(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;
    const int yc = b * a.cap;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA, scores
        if (lane == 0 && ntile > 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qhmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qlmap) : "memory");
            const int yq = b * a.R + q0;
            const int latoms = a.kvl / 64;
            int item = 0;
            for (int j = 0; j < ntile && !failed; j++)
                for (int at = 0; at < a.qa; at++, item++) {
                    const int st = item % NSQ;
                    if (!bar_wait(s_addr(&b_qempty[st]), (uint32_t)(((item / NSQ) & 1) ^ 1))) { failed = true; break; }
                    const uint32_t sw = s_addr(smem + (size_t)st * QSTAGE), full = s_addr(&b_qfull[st]);
                    bar_expect(full, QSTAGE);
                    tma2d(sw, &qhmap, at * 64, yq, full);
                    tma2d(sw + ATOM, &qlmap, at * 64, yq, full);
                    if (at < latoms) tma2d(sw + 2 * ATOM, &latmap, at * 64, yc + begin + j * NP, full);
                    else tma2d(sw + 2 * ATOM, &ropemap, 0, yc + begin + j * NP, full);
                }
            // let the copies in flight land before the CTA can exit
            for (int k = max(0, item - NSQ); k < item; k++)
                if (!bar_wait(s_addr(&b_qfull[k % NSQ]), (uint32_t)((k / NSQ) & 1))) failed = true;
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ TMA, values
        if (lane == 0 && ntile > 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&latmap) : "memory");
            int item = 0;
            for (int i = 0; i < ntile && !failed; i++)
                for (int vs = 0; vs < nvs; vs++, item++) {
                    const int st = item % NSV;
                    if (!bar_wait(s_addr(&b_vempty[st]), (uint32_t)(((item / NSV) & 1) ^ 1))) { failed = true; break; }
                    const uint32_t sv = s_addr(smem + V_OFF + (size_t)st * VSTAGE), full = s_addr(&b_vfull[st]);
                    bar_expect(full, (uint32_t)(vw * ATOM));
                    for (int x = 0; x < vw; x++)
                        tma2d(sv + x * ATOM, &latmap, (hf * va + vs * vw + x) * 64, yc + begin + i * NP, full);
                }
            for (int k = max(0, item - NSV); k < item; k++)
                if (!bar_wait(s_addr(&b_vfull[k % NSV]), (uint32_t)((k / NSV) & 1))) failed = true;
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------------ score MMAs
        if (ntile > 0) {
            const uint32_t idq = bf16_idesc(NP, false);
            int item = 0;
            for (int j = 0; j < ntile && !failed; j++) {
                const int sb = j & 1;
                // the buffer's previous tile (j - 2) has left it: its value MMAs are done
                if (!bar_wait(s_addr(&b_pvdone[sb]), (uint32_t)(((j >> 1) & 1) ^ 1))) { failed = true; break; }
                fence_after();
                const uint32_t s_tm = tmem + (uint32_t)(sb * NP);
                for (int at = 0; at < a.qa; at++, item++) {
                    const int st = item % NSQ;
                    if (!bar_wait(s_addr(&b_qfull[st]), (uint32_t)((item / NSQ) & 1))) { failed = true; break; }
                    fence_after();
                    if (lane == 0) {
                        const uint64_t d0 = sw128_desc(s_addr(smem + (size_t)st * QSTAGE));
                        constexpr uint32_t ql = ATOM >> 4, cc = (2 * ATOM) >> 4;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            mma_ss(s_tm, d0 + 2 * k, d0 + cc + 2 * k, idq, (at | k) ? 1u : 0u);
                            mma_ss(s_tm, d0 + ql + 2 * k, d0 + cc + 2 * k, idq, 1u);
                        }
                        mma_commit(s_addr(&b_qempty[st]));
                    }
                    __syncwarp();
                }
                if (failed) break;
                if (lane == 0) mma_commit(s_addr(&b_sfull[sb]));
                __syncwarp();
            }
            if (lane == 0) {
                mma_commit(s_addr(b_finq));
                // every MMA of this warp has completed before TMEM can be freed
                if (!bar_wait(s_addr(b_finq), 0)) failed = true;
                if (failed) flag(DEV_TIMEOUT);
            }
        }
    } else if (warp == 3) {
        // ------------------------------------------------------------------ value MMAs
        if (ntile > 0) {
            const uint32_t idv = bf16_idesc(vw * 64, true);
            int item = 0;
            for (int i = 0; i < ntile && !failed; i++) {
                const int sb = i & 1;
                if (!bar_wait(s_addr(&b_pfull[sb]), (uint32_t)((i >> 1) & 1))) { failed = true; break; }
                fence_after();
                const int nv = min(NP, end - (begin + i * NP));   // rows past it lie at or past n_ctx
                const uint32_t p_tm = tmem + (uint32_t)(sb * NP);
                for (int vs = 0; vs < nvs; vs++, item++) {
                    const int st = item % NSV;
                    if (!bar_wait(s_addr(&b_vfull[st]), (uint32_t)((item / NSV) & 1))) { failed = true; break; }
                    fence_after();
                    unsigned char *sv = smem + V_OFF + (size_t)st * VSTAGE;
                    if (nv < NP) {
                        // the cache past n_ctx is unspecified: zero it, so 0 * row stays 0
                        for (int x = 0; x < vw; x++)
                            for (int e = nv * 8 + lane; e < NP * 8; e += 32)
                                *reinterpret_cast<uint4 *>(sv + (size_t)x * ATOM + (size_t)e * 16) = make_uint4(0, 0, 0, 0);
                        fence_async_smem();
                        __syncwarp();
                    }
                    if (lane == 0) {
                        const uint32_t d_tm = tmem + 256u + (uint32_t)(vs * vw * 64);
                        const uint32_t vb = s_addr(sv);
#pragma unroll
                        for (int kk = 0; kk < NP / 16; kk++) {
                            // positions 16 kk.. : chunk kk / 2 of 32, hi pairs then lo pairs
                            const uint32_t pa = p_tm + (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8);
                            const uint64_t vd = sw128_mn_desc(vb + (uint32_t)(kk * 2048), ATOM);
                            mma_ts(d_tm, pa, vd, idv, (i > 0 || kk > 0) ? 1u : 0u);
                            mma_ts(d_tm, pa + 16u, vd, idv, 1u);
                        }
                        mma_commit(s_addr(&b_vempty[st]));
                    }
                    __syncwarp();
                }
                if (failed) break;
                if (lane == 0) mma_commit(s_addr(&b_pvdone[sb]));
                __syncwarp();
            }
            if (lane == 0) {
                mma_commit(s_addr(b_ofull));
                mma_commit(s_addr(b_finv));
                if (!bar_wait(s_addr(b_finv), 0)) failed = true;
                if (failed) flag(DEV_TIMEOUT);
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax
        const int quarter = warp & 3;
        const int half = (warp - 4) >> 2;      // which 64 positions of a tile
        const int row = quarter * 32 + lane;
        const int rg = q0 + row;
        const bool row_ok = rg < a.R;
        const int t = row_ok ? rg / a.H : 0;
        const uint64_t mk = a.mask[t];
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        const float sl2 = a.scale * LOG2E;
        const int ocols = va * 32;              // this warp's share of u's half
        float m_run = -INFINITY, l_part = 0.0f;   // log2 units
        // A warp whose wait gave up keeps stepping (without waiting) so that all eight reach
        // every named barrier; the slice is then reported through the status word only.
        for (int j = 0; j < ntile; j++) {
            const int sb = j & 1;
            const int p0 = begin + j * NP + half * 64;
            if (!failed && !bar_wait(s_addr(&b_sfull[sb]), (uint32_t)((j >> 1) & 1))) failed = true;
            fence_after();
            const uint32_t s_tm = tmem + lane_addr + (uint32_t)(sb * NP + half * 64);
            uint32_t sv[64];
            {
                uint32_t (&v0)[16] = *reinterpret_cast<uint32_t (*)[16]>(&sv[0]);
                uint32_t (&v1)[16] = *reinterpret_cast<uint32_t (*)[16]>(&sv[16]);
                uint32_t (&v2)[16] = *reinterpret_cast<uint32_t (*)[16]>(&sv[32]);
                uint32_t (&v3)[16] = *reinterpret_cast<uint32_t (*)[16]>(&sv[48]);
                tmem_ld16(s_tm, v0);
                tmem_ld16(s_tm + 16u, v1);
                tmem_ld16(s_tm + 32u, v2);
                tmem_ld16(s_tm + 48u, v3);
                tmem_wait_ld();
            }
            // a position is visible when it lies below end and is an old row or a new row
            // whose bit is set in the node's mask
            const bool all_old = p0 + 64 <= min(c, end);
            auto visible = [&](int s) -> bool {
                return s < end && (s < c || ((mk >> (s - c)) & 1ull) != 0);
            };
            float mt = -INFINITY;
            if (all_old) {
#pragma unroll
                for (int n = 0; n < 64; n++) mt = fmaxf(mt, __uint_as_float(sv[n]));
            } else {
#pragma unroll
                for (int n = 0; n < 64; n++)
                    if (visible(p0 + n)) mt = fmaxf(mt, __uint_as_float(sv[n]));
            }
            // both halves of the row agree on the tile max (scale > 0)
            xmax[((j & 1) * 2 + half) * 128 + row] = mt;
            asm volatile("bar.sync 1, %0;" ::"n"(NSOFT * 32) : "memory");
            mt = fmaxf(xmax[((j & 1) * 2) * 128 + row], xmax[((j & 1) * 2 + 1) * 128 + row]);
            const float mt2 = (row_ok && mt > -INFINITY) ? mt * sl2 : -INFINITY;
            const bool upd = mt2 > -INFINITY && (m_run == -INFINITY || mt2 > m_run + RESCALE_AT);
            const bool resc = upd && m_run != -INFINITY;
            const float al = resc ? ex2(m_run - mt2) : 1.0f;
            if (upd) m_run = mt2;
            if (__any_sync(0xffffffffu, resc)) {
                // u holds the value products up to tile j - 1: wait for them, then scale
                // this warp's columns of the row (lanes whose max stayed scale by 1)
                if (!failed && j >= 1 && !bar_wait(s_addr(&b_pvdone[(j - 1) & 1]), (uint32_t)(((j - 1) >> 1) & 1)))
                    failed = true;
                fence_after();
                for (int ch = 0; ch < ocols / 16; ch++) {
                    uint32_t v[16];
                    const uint32_t ot = tmem + lane_addr + 256u + (uint32_t)(half * ocols + ch * 16);
                    tmem_ld16(ot, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int n = 0; n < 16; n++) v[n] = __float_as_uint(__uint_as_float(v[n]) * al);
                    tmem_st16(ot, v);
                }
                tmem_wait_st();
            }
            if (resc) l_part *= al;
            const float mneg = -m_run;
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {        // two chunks of 32 positions
                uint32_t hw[16], lw[16];
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const int n0 = cc * 32 + 2 * q;
                    float x0 = 0.0f, x1 = 0.0f;
                    const bool v0 = row_ok && (all_old || visible(p0 + n0));
                    const bool v1 = row_ok && (all_old || visible(p0 + n0 + 1));
                    if (v0) x0 = ex2(fmaf(__uint_as_float(sv[n0]), sl2, mneg));
                    if (v1) x1 = ex2(fmaf(__uint_as_float(sv[n0 + 1]), sl2, mneg));
                    l_part += x0;
                    l_part += x1;
                    const uint32_t h = pack_bf16x2(x0, x1);
                    hw[q] = h;
                    lw[q] = pack_bf16x2(__fsub_rn(x0, __uint_as_float(h << 16)),
                                        __fsub_rn(x1, __uint_as_float(h & 0xFFFF0000u)));
                }
                const uint32_t pt = s_tm + (uint32_t)(cc * 32);
                tmem_st16(pt, hw);
                tmem_st16(pt + 16u, lw);
            }
            tmem_wait_st();
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(s_addr(&b_pfull[sb]));
        }
        // the row's partial state for this slice
        if (ntile > 0 && !failed) {
            if (!bar_wait(s_addr(b_ofull), 0)) failed = true;
            fence_after();
        }
        if (half == 1) xsum[row] = l_part;
        asm volatile("bar.sync 1, %0;" ::"n"(NSOFT * 32) : "memory");
        if (failed) {
            if (lane == 0) flag(DEV_TIMEOUT);
        } else {
            const size_t pi = ((size_t)b * a.R + (size_t)(row_ok ? rg : 0)) * a.nsplit + sp;
            if (row_ok && hf == 0 && half == 0) {
                a.pm[pi] = m_run == -INFINITY ? -INFINITY : m_run * LN2;
                a.pl[pi] = l_part + xsum[row];
            }
            float *dst = a.pu + pi * a.kvl + hf * va * 64 + half * ocols;
            for (int ch = 0; ch < ocols / 16; ch++) {
                uint32_t v[16];
                if (ntile > 0) {
                    tmem_ld16(tmem + lane_addr + 256u + (uint32_t)(half * ocols + ch * 16), v);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int n = 0; n < 16; n++) v[n] = 0u;
                }
                if (row_ok) {
#pragma unroll
                    for (int n = 0; n < 16; n += 4)
                        *reinterpret_cast<float4 *>(dst + ch * 16 + n) =
                            make_float4(__uint_as_float(v[n]), __uint_as_float(v[n + 1]), __uint_as_float(v[n + 2]),
                                        __uint_as_float(v[n + 3]));
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 2) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Slices: the number of 128-position tiles per slice that minimises (waves of CTAs) x
// (tiles per slice + a fixed cost per slice), on a full B200.
static int plan(int B, int R, int max_ctx, int *split_len)
{
    const int tiles = ceil_div(max_ctx, NP);
    const long long combos = (long long)B * ceil_div(R, 128) * 2;
    double best = 1e300;
    int best_tl = tiles;
    for (int ns = 1; ns <= std::min(tiles, MLA_MAXSPLIT); ns++) {
        const int tl = ceil_div(tiles, ns);
        const int nsr = ceil_div(tiles, tl);
        const long long waves = (combos * nsr + SMS_PLAN - 1) / SMS_PLAN;
        const double cost = (double)waves * (tl + 1.5);
        if (cost < best - 1e-9) { best = cost; best_tl = tl; }
    }
    *split_len = best_tl * NP;
    return ceil_div(tiles, best_tl);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(q);
    });
    return fn;
}

// bf16 [rows][cols] (row stride cols) in boxes of 64 columns x 128 rows, 128-byte swizzle
static int map_bf16(CUtensorMap *m, const void *base, long long cols, long long rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return K3GPU_ECUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {64u, 128u};
    cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        g_last_cuda_error = (int)r;
        return K3GPU_ECUDA;
    }
    return K3GPU_OK;
}

static bool usable(int kvl, int qr, const void *lat, const void *rope)
{
    return (kvl == 128 || kvl == 256 || kvl == 512) && (qr == 0 || qr == 64) && aligned(lat, 16) &&
           (qr == 0 || aligned(rope, 16));
}

static int g_attr_dev = -1;
static std::mutex g_attr_mu;

}  // namespace mlatc

}  // namespace k3

extern "C" size_t k3gpu_mla_workspace(int B, int T, int H, int kv_lora, int max_ctx)
{
    if (B <= 0 || T <= 0 || H <= 0 || kv_lora <= 0 || max_ctx <= 0) return 0;
    // room for either path: the CUDA-core slices of MLA_SPLIT positions or the
    // tensor-core plan's slices (the rope width is at most MLA_MAXR)
    int sl = 0;
    const int ns_tc = k3::mlatc::plan(B, T * H, max_ctx, &sl);
    const int ns = std::max(k3::ceil_div(max_ctx, k3::MLA_SPLIT), ns_tc);
    return k3::mla_ws_layout(B, T, H, kv_lora, k3::MLA_MAXR, ns, nullptr, nullptr);
}

extern "C" int k3gpu_mla_absorbed(float *out, const float *q_nope, const float *q_rope,
                                  const float *kv_b, const uint16_t *lat, const uint16_t *rope,
                                  const int *cached, const uint64_t *mask, int B, int T, int H,
                                  int qk_nope, int qk_rope, int v_head, int kv_lora, int cap,
                                  int max_ctx, float scale, void *workspace, size_t ws_bytes,
                                  void *stream)
{
    if (!out || !q_nope || !kv_b || !lat || !cached || !mask || !workspace ||
        (qk_rope > 0 && (!q_rope || !rope)))
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || H <= 0 || H > 4096 || qk_nope <= 0 || qk_nope > 256 ||
        qk_rope < 0 || qk_rope > k3::MLA_MAXR || v_head <= 0 || v_head > 256 ||
        (kv_lora != 128 && kv_lora != 256 && kv_lora != 512) || cap <= 0 || max_ctx <= 0 ||
        max_ctx > cap || k3::ceil_div(max_ctx, k3::MLA_SPLIT) > k3::MLA_MAXSPLIT)
        return K3GPU_EINVAL;
    const int ns_cc = k3::ceil_div(max_ctx, k3::MLA_SPLIT);
    int split_len = 0;
    const int ns_tc = k3::mlatc::plan(B, T * H, max_ctx, &split_len);
    k3::MlaWs w;
    const size_t need = k3::mla_ws_layout(B, T, H, kv_lora, k3::MLA_MAXR, std::max(ns_cc, ns_tc), &w,
                                          static_cast<char *>(workspace));
    if (ws_bytes < need) return K3GPU_ECAPACITY;
    cudaStream_t s = k3::as_stream(stream);
    k3::mla_qabs_kernel<<<dim3(H, k3::ceil_div(B * T, k3::QB_T), k3::ceil_div(kv_lora, k3::QB_J)), 256, 0, s>>>(
        w.qabs, q_nope, kv_b, B * T, H, qk_nope, v_head, kv_lora);
    int st = k3::launch_status();
    if (st) return st;
    int ns = ns_cc, sl = k3::MLA_SPLIT;
    if (k3::mlatc::usable(kv_lora, qk_rope, lat, rope)) {
        using namespace k3::mlatc;
        const int R = T * H, kq = kv_lora + qk_rope;
        prep_kernel<<<B * R, 128, 0, s>>>(w.qh, w.ql, w.qabs, q_rope, kv_lora, qk_rope);
        if ((st = k3::launch_status())) return st;
        CUtensorMap qhm, qlm, latm, ropem;
        if ((st = map_bf16(&qhm, w.qh, kq, (long long)B * R))) return st;
        if ((st = map_bf16(&qlm, w.ql, kq, (long long)B * R))) return st;
        if ((st = map_bf16(&latm, lat, kv_lora, (long long)B * cap))) return st;
        if ((st = map_bf16(&ropem, qk_rope ? (const void *)rope : (const void *)lat, qk_rope ? 64 : kv_lora,
                           (long long)B * cap)))
            return st;
        int dev = 0;
        if ((st = k3::cuda_status(cudaGetDevice(&dev)))) return st;
        {
            std::lock_guard<std::mutex> lock(g_attr_mu);
            if (g_attr_dev != dev) {
                st = k3::cuda_status(cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
                if (st) return st;
                g_attr_dev = dev;
            }
        }
        Args a;
        a.pm = w.pm; a.pl = w.pl; a.pu = w.pu;
        a.cached = cached; a.mask = mask;
        a.T = T; a.H = H; a.R = R; a.kvl = kv_lora; a.qr = qk_rope; a.cap = cap;
        a.nsplit = ns_tc; a.split_len = split_len; a.qa = kv_lora / 64 + (qk_rope ? 1 : 0);
        a.scale = scale;
        attend_kernel<<<dim3(ns_tc, k3::ceil_div(R, 128) * 2, B), THREADS, SMEM, s>>>(qhm, qlm, latm, ropem, a);
        if ((st = k3::launch_status())) return st;
        ns = ns_tc;
        sl = split_len;
    } else {
        // the opt-in to >48 KB of dynamic shared memory, once per device (a function's
        // attributes belong to each device's context)
        static std::mutex attr_mu;
        static bool attr_set[64] = {};
        int adev = 0;
        if ((st = k3::cuda_status(cudaGetDevice(&adev)))) return st;
        if (adev < 0 || adev >= 64) return K3GPU_EINVAL;
        {
            std::lock_guard<std::mutex> lock(attr_mu);
            if (!attr_set[adev]) {
                st = k3::cuda_status(cudaFuncSetAttribute(k3::mla_attend_kernel,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          (int)k3::MLA_SMEM));
                if (st) return st;
                attr_set[adev] = true;
            }
        }
        k3::mla_attend_kernel<<<dim3(ns, B * T, k3::ceil_div(H, k3::MLA_HT)), k3::MLA_THREADS,
                                k3::MLA_SMEM, s>>>(
            w, q_rope, lat, rope, cached, mask, T, H, qk_rope, kv_lora, cap, ns, scale);
        if ((st = k3::launch_status())) return st;
    }
    // the merged slices go over q_abs (its last reader, the attention, has run)
    k3::mla_merge_kernel<<<dim3(k3::ceil_div(H, k3::MG_H), B * T), 256, 0, s>>>(w.qabs, w, cached, T, H, kv_lora,
                                                                                 ns, sl);
    if ((st = k3::launch_status())) return st;
    k3::mla_out_kernel<<<dim3(H, k3::ceil_div(B * T, k3::OB_T), k3::ceil_div(v_head, k3::OB_R)), 256, 0, s>>>(
        out, w.qabs, kv_b, B * T, H, qk_nope, v_head, kv_lora);
    return k3::launch_status();
}
