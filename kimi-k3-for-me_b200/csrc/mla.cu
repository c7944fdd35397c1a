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
//   combine  merges the slices of each (node, head) and applies out = W_uv[h] u.
//
// Scores are fp32 dot products of fp32 queries with the bf16 cache (the cache is the
// compressed latent the reference stores in fp32; here it is held in bf16 in HBM, half
// the bytes). The softmax uses the slice maxima and fp32 exps; tolerance-level against
// the reference's double normaliser.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"

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
};

static size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

static size_t mla_ws_layout(int B, int T, int H, int kvl, int max_ctx, MlaWs *w, char *base)
{
    const int ns = (max_ctx + MLA_SPLIT - 1) / MLA_SPLIT;
    const size_t rows = (size_t)B * T * H;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += a256(bytes);
        return r;
    };
    char *qa = take(rows * kvl * 4), *pm = take(rows * ns * 4), *pl = take(rows * ns * 4);
    char *pu = take(rows * ns * (size_t)kvl * 4);
    if (w) { w->qabs = (float *)qa; w->pm = (float *)pm; w->pl = (float *)pl; w->pu = (float *)pu; }
    return o;
}

// grid (B*T, H), block 256: qabs[j] = sum_i W[h*kvd + i][j] * q_nope[i], i ascending
__global__ void __launch_bounds__(256) mla_qabs_kernel(float *__restrict__ qabs,
                                                       const float *__restrict__ q_nope,
                                                       const float *__restrict__ kv_b, int H,
                                                       int qn, int vh, int kvl)
{
    const int bt = blockIdx.x, h = blockIdx.y;
    const int kvd = qn + vh;
    const float *q = q_nope + ((size_t)bt * H + h) * qn;
    for (int j = threadIdx.x; j < kvl; j += blockDim.x) {
        float a = 0.0f;
        for (int i = 0; i < qn; i++) a = fmaf(kv_b[((size_t)h * kvd + i) * kvl + j], q[i], a);
        qabs[((size_t)bt * H + h) * kvl + j] = a;
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

// grid (B*T, H), block 256: merge the slices, then out = W_uv[h] u
__global__ void __launch_bounds__(256) mla_combine_kernel(float *__restrict__ out, MlaWs w,
                                                          const float *__restrict__ kv_b,
                                                          const int *__restrict__ cached, int T,
                                                          int H, int qn, int vh, int kvl,
                                                          int nsplit)
{
    __shared__ float su[MLA_MAXL];
    __shared__ float sw[MLA_MAXSPLIT];
    const int bt = blockIdx.x, h = blockIdx.y;
    const int b = bt / T;
    const int n_ctx = cached[b] + T;
    const int nsu = min(nsplit, (n_ctx + MLA_SPLIT - 1) / MLA_SPLIT);
    const size_t base = ((size_t)bt * H + h) * nsplit;
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int s = 0; s < nsu; s++) M = fmaxf(M, w.pm[base + s]);
        float Lsum = 0.0f;
        for (int s = 0; s < nsu; s++) {
            const float f = w.pm[base + s] == -INFINITY ? 0.0f : __expf(w.pm[base + s] - M);
            sw[s] = f;
            Lsum += f * w.pl[base + s];
        }
        const float inv = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
        for (int s = 0; s < nsu; s++) sw[s] *= inv;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < kvl; j += blockDim.x) {
        float a = 0.0f;
        for (int s = 0; s < nsu; s++) a = fmaf(sw[s], w.pu[(base + s) * kvl + j], a);
        su[j] = a;
    }
    __syncthreads();
    const int kvd = qn + vh;
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = wid; r < vh; r += blockDim.x / 32) {
        const float *wr = kv_b + ((size_t)h * kvd + qn + r) * kvl;
        float a = 0.0f;
        for (int j = lane; j < kvl; j += 32) a = fmaf(wr[j], su[j], a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) out[((size_t)bt * H + h) * vh + r] = a;
    }
}

}  // namespace k3

extern "C" size_t k3gpu_mla_workspace(int B, int T, int H, int kv_lora, int max_ctx)
{
    if (B <= 0 || T <= 0 || H <= 0 || kv_lora <= 0 || max_ctx <= 0) return 0;
    return k3::mla_ws_layout(B, T, H, kv_lora, max_ctx, nullptr, nullptr);
}

extern "C" int k3gpu_mla_absorbed(float *out, const float *q_nope, const float *q_rope,
                                  const float *kv_b, const uint16_t *lat, const uint16_t *rope,
                                  const int *cached, const uint64_t *mask, int B, int T, int H,
                                  int qk_nope, int qk_rope, int v_head, int kv_lora, int cap,
                                  int max_ctx, float scale, void *workspace, size_t ws_bytes,
                                  void *stream)
{
    if (!out || !q_nope || !q_rope || !kv_b || !lat || !rope || !cached || !mask || !workspace)
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || H <= 0 || H > 4096 || qk_nope <= 0 || qk_nope > 256 ||
        qk_rope < 0 || qk_rope > k3::MLA_MAXR || v_head <= 0 || v_head > 256 ||
        (kv_lora != 128 && kv_lora != 256 && kv_lora != 512) || cap <= 0 || max_ctx <= 0 ||
        max_ctx > cap || k3::ceil_div(max_ctx, k3::MLA_SPLIT) > k3::MLA_MAXSPLIT)
        return K3GPU_EINVAL;
    k3::MlaWs w;
    const size_t need = k3::mla_ws_layout(B, T, H, kv_lora, max_ctx, &w, static_cast<char *>(workspace));
    if (ws_bytes < need) return K3GPU_ECAPACITY;
    cudaStream_t s = k3::as_stream(stream);
    const int ns = k3::ceil_div(max_ctx, k3::MLA_SPLIT);
    k3::mla_qabs_kernel<<<dim3(B * T, H), 256, 0, s>>>(w.qabs, q_nope, kv_b, H, qk_nope, v_head,
                                                      kv_lora);
    int st = k3::launch_status();
    if (st) return st;
    static bool attr_set = false;   // one-time opt-in to >48 KB of dynamic shared memory
    if (!attr_set) {
        st = k3::cuda_status(cudaFuncSetAttribute(k3::mla_attend_kernel,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)k3::MLA_SMEM));
        if (st) return st;
        attr_set = true;
    }
    k3::mla_attend_kernel<<<dim3(ns, B * T, k3::ceil_div(H, k3::MLA_HT)), k3::MLA_THREADS,
                            k3::MLA_SMEM, s>>>(
        w, q_rope, lat, rope, cached, mask, T, H, qk_rope, kv_lora, cap, ns, scale);
    if ((st = k3::launch_status())) return st;
    k3::mla_combine_kernel<<<dim3(B * T, H), 256, 0, s>>>(out, w, kv_b, cached, T, H, qk_nope,
                                                         v_head, kv_lora, ns);
    return k3::launch_status();
}
