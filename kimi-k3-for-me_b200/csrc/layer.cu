// layer.cu -- a KDA + MoE decoder layer of a verify sweep, composed on the library's own
// entry points in the reference's order.
//
// k3gpu_kda_layer_verify is k3_kda_layer_log (src/core/k3_ops.c:2231-2385) for B
// sequences of T positions: the six projections (k3_mmw_batch, here
// k3gpu_matmul_bf16_batch), the prologue (ShortConv + SiLU, L2 norm, beta, decay), the
// recurrence on the read-only carried state, head RMSNorm then the sigmoid gate (the g
// projection), and the output projection. The log operands a commit replays (k, v, alpha,
// beta, pre-conv rows) are written straight into the caller's log buffers.
//
// k3gpu_mla_layer_verify is k3_mla_cached (src/core/k3_ops.c:1115-1615) in its absorbed
// latent layout: q_a, RMSNorm, q_b; kv_a, the latent's RMSNorm, the new rows appended to the
// bf16 latent and rope caches; absorbed attention (k3gpu_mla_absorbed); the sigmoid gate
// on x, then o.
//
// k3gpu_decoder_layer_kda_verify is k3_decoder_layer_core (src/core/k3_ops.c:2485-2592)
// for that layer: AttnRes before attention over each position's block-residual snapshots,
// the block-boundary snapshot (then the running residual restarts from the attention
// output), input RMSNorm, the KDA layer, AttnRes before the MLP, post RMSNorm, the MoE, and
// the residual. The MoE is either the single-layer form (router and MXFP4 experts at the
// hidden width, shared experts in the bank) or the K3 form of k3_moe_prefill
// (src/core/k3_ops.c:2008-2053, 1848-1860): routing on x, the MXFP4 experts on the latent
// down-projection, the latent RMSNorm, the up-projection, and the dense bf16 shared expert.
#include <cuda_bf16.h>

#include "common.cuh"
#include "moe.cuh"

namespace k3 {

// block_residual[t][n_blocks[t]] = pref[t]; n_blocks[t] += 1 (one CTA per position)
__global__ void __launch_bounds__(256) snapshot_kernel(float *__restrict__ block_residual,
                                                       int *__restrict__ n_blocks,
                                                       const float *__restrict__ pref, int maxb,
                                                       int E)
{
    const int t = blockIdx.x;
    const int nb = n_blocks[t];
    if (nb < 0 || nb >= maxb) {
        if (threadIdx.x == 0) flag(DEV_BAD_COUNT);
        return;
    }
    float *dst = block_residual + ((size_t)t * maxb + nb) * E;
    const float *src = pref + (size_t)t * E;
    for (int i = threadIdx.x; i < E; i += 256) dst[i] = src[i];
    __syncthreads();
    if (threadIdx.x == 0) n_blocks[t] = nb + 1;
}

// y = a + b in float (y may be a)
__global__ void __launch_bounds__(256) add_kernel(float *y, const float *a, const float *b, long long n)
{
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

static int add_launch(float *y, const float *a, const float *b, long long n, cudaStream_t s)
{
    add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, a, b, n);
    return launch_status();
}

// y = act(g, u) elementwise (the shared expert's [gate | up] -> act; y may be g)
__global__ void __launch_bounds__(256) glu_kernel(float *y, const float *g, const float *u, long long n, int act,
                                                  float b1, float b2)
{
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i < n) y[i] = act == K3GPU_ACT_SITU ? act_situ(g[i], u[i], b1, b2) : act_swiglu(g[i], u[i]);
}

struct MoeWs {
    float *z, *acc, *g, *u, *d;
    char *router, *experts, *mm;
    size_t router_bytes, experts_bytes, mm_bytes;
};

static size_t moe_ws_layout(const K3GpuMoeCfg *c, int T, MoeWs *w, char *base)
{
    const int E = c->hidden, L = c->latent, SI = c->shared_inter;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return r;
    };
    MoeWs t;
    t.z = (float *)take((size_t)T * L * 4);
    t.acc = (float *)take((size_t)T * L * 4);
    t.g = (float *)take((size_t)T * (SI > 0 ? SI : 1) * 4);
    t.u = (float *)take((size_t)T * (SI > 0 ? SI : 1) * 4);
    t.d = (float *)take((size_t)T * E * 4);
    t.router_bytes = k3gpu_router_workspace(T, c->n_routed);
    t.router = take(t.router_bytes);
    t.experts_bytes = k3gpu_moe_workspace(T, c->topk, 0, L, c->moe_inter, c->n_routed);
    t.experts = take(t.experts_bytes);
    size_t mm = std::max(k3gpu_matmul_bf16_workspace(T, E, L), k3gpu_matmul_bf16_workspace(T, L, E));
    if (SI > 0)
        mm = std::max(mm, std::max(k3gpu_matmul_bf16_workspace(T, E, SI), k3gpu_matmul_bf16_workspace(T, SI, E)));
    t.mm_bytes = mm;
    t.mm = take(mm);
    if (w) *w = t;
    return o;
}

static bool moe_cfg_ok(const K3GpuMoeCfg *c)
{
    return c && c->hidden > 0 && c->latent > 0 && c->moe_inter > 0 && c->shared_inter >= 0 && c->n_routed > 0 &&
           c->topk > 0 && c->topk <= c->n_routed;
}

struct KdaWs {
    float *q, *z, *fa, *bt, *o, *g;
    char *mm;
    size_t mm_bytes;
};

static size_t kda_ws_layout(const K3GpuLayerCfg *c, int R, KdaWs *w, char *base)
{
    const int E = c->hidden, H = c->kda_heads, D = c->kda_head_dim, P = H * D;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return r;
    };
    KdaWs t;
    t.q = (float *)take((size_t)R * P * 4);
    t.z = (float *)take((size_t)R * P * 4);
    t.fa = (float *)take((size_t)R * D * 4);
    t.bt = (float *)take((size_t)R * H * 4);
    t.o = (float *)take((size_t)R * P * 4);
    t.g = (float *)take((size_t)R * P * 4);
    size_t mm = 0;
    const int shapes[5][2] = {{E, P}, {E, H}, {E, D}, {D, P}, {P, E}};
    for (auto &sh : shapes) mm = std::max(mm, k3gpu_matmul_bf16_workspace(R, sh[0], sh[1]));
    t.mm_bytes = mm;
    t.mm = take(mm);
    if (w) *w = t;
    return o;
}

static bool cfg_ok(const K3GpuLayerCfg *c)
{
    return c && c->hidden > 0 && c->kda_heads > 0 && c->kda_head_dim > 0 && c->conv_k >= 2 && c->conv_k <= 8;
}

// ---------------------------------------------------------------------------- MLA --
static bool mla_cfg_ok(const K3GpuLayerCfg *c)
{
    return c && c->hidden > 0 && c->hidden % 8 == 0 && c->mla_heads > 0 && c->q_lora > 0 && c->q_lora % 8 == 0 &&
           (c->kv_lora == 128 || c->kv_lora == 256 || c->kv_lora == 512) && c->qk_nope > 0 && c->qk_nope <= 256 &&
           c->qk_rope >= 0 && c->qk_rope <= 64 && c->v_head > 0 && c->v_head <= 256 &&
           (c->mla_heads * c->v_head) % 8 == 0;
}

struct MlaLWs {
    float *ql, *qln, *q, *ct, *qnp, *qrp, *acc, *g;
    char *mm, *att;
    size_t mm_bytes, att_bytes;
};

static size_t mla_ws_layout(const K3GpuLayerCfg *c, int B, int T, int max_ctx, MlaLWs *w, char *base)
{
    const int E = c->hidden, H = c->mla_heads, qn = c->qk_nope, qr = c->qk_rope, vh = c->v_head;
    const int kvw = c->kv_lora + qr, R = B * T;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return r;
    };
    MlaLWs t;
    t.ql = (float *)take((size_t)R * c->q_lora * 4);
    t.qln = (float *)take((size_t)R * c->q_lora * 4);
    t.q = (float *)take((size_t)R * H * (qn + qr) * 4);
    t.ct = (float *)take((size_t)R * kvw * 4);
    t.qnp = (float *)take((size_t)R * H * qn * 4);
    t.qrp = (float *)take((size_t)R * H * std::max(qr, 1) * 4);
    t.acc = (float *)take((size_t)R * H * vh * 4);
    t.g = (float *)take((size_t)R * H * vh * 4);
    size_t mm = 0;
    const int shapes[5][2] = {{E, c->q_lora}, {c->q_lora, H * (qn + qr)}, {E, kvw}, {E, H * vh}, {H * vh, E}};
    for (auto &sh : shapes) mm = std::max(mm, k3gpu_matmul_bf16_workspace(R, sh[0], sh[1]));
    t.mm_bytes = mm;
    t.mm = take(mm);
    t.att_bytes = k3gpu_mla_workspace(B, T, H, c->kv_lora, max_ctx);
    t.att = take(t.att_bytes);
    if (w) *w = t;
    return o;
}

constexpr int AP_THREADS = 256;

__device__ __forceinline__ double ap_block_sum(double v, double *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < AP_THREADS / 32; w++) t += red[w];
    return t;
}

// One CTA per new row (b, t): the latent part of ct normalised as k3gpu_rmsnorm does (the
// reference's k3_rmsnorm: double sum of squares, float scale), both parts rounded to bf16
// and written at cache position cached[b] + t (src/core/k3_ops.c:1188-1200).
__global__ void __launch_bounds__(AP_THREADS) mla_append_kernel(uint16_t *__restrict__ lat, uint16_t *__restrict__ rope,
                                                                const float *__restrict__ ct,
                                                                const float *__restrict__ norm_w,
                                                                const int *__restrict__ cached, int T, int cap,
                                                                int kvl, int qr, float eps)
{
    __shared__ double red[AP_THREADS / 32];
    const int r = blockIdx.x, b = r / T, t = r % T;
    const int pos = cached[b] + t;
    if (cached[b] < 0 || pos >= cap) {      // uniform over the block
        if (threadIdx.x == 0) flag(DEV_BAD_POSITION);
        return;
    }
    const float *xr = ct + (size_t)r * (kvl + qr);
    double ss = 0.0;
    for (int i = threadIdx.x; i < kvl; i += AP_THREADS) ss += (double)xr[i] * (double)xr[i];
    ss = ap_block_sum(ss, red);
    const float inv = __double2float_rn(1.0 / sqrt(ss / (double)kvl + (double)eps));
    uint16_t *lr = lat + ((size_t)b * cap + pos) * kvl;
    for (int i = threadIdx.x; i < kvl; i += AP_THREADS)
        lr[i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(__fmul_rn(norm_w[i], xr[i]), inv)));
    if (qr > 0) {
        uint16_t *rr = rope + ((size_t)b * cap + pos) * qr;
        for (int i = threadIdx.x; i < qr; i += AP_THREADS) rr[i] = __bfloat16_as_ushort(__float2bfloat16_rn(xr[kvl + i]));
    }
}

// q [R][H][qn + qr] -> q_nope [R][H][qn], q_rope [R][H][qr]
__global__ void __launch_bounds__(256) mla_qsplit_kernel(float *__restrict__ qnp, float *__restrict__ qrp,
                                                        const float *__restrict__ q, long long n, int qn, int qr)
{
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i >= n) return;
    const int qh = qn + qr;
    const long long row = i / qh;
    const int d = (int)(i % qh);
    if (d < qn) qnp[row * qn + d] = q[i];
    else qrp[row * qr + (d - qn)] = q[i];
}

// acc *= 1 / (1 + exp(-g)) (src/core/k3_ops.c:1604-1608)
__global__ void __launch_bounds__(256) mla_gate_kernel(float *__restrict__ acc, const float *__restrict__ g,
                                                      long long n)
{
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    if (i < n) acc[i] = __fmul_rn(acc[i], sigmoid_cr(g[i]));
}

}  // namespace k3

extern "C" size_t k3gpu_moe_prefill_workspace(const K3GpuMoeCfg *c, int T)
{
    if (!k3::moe_cfg_ok(c) || T <= 0) return 0;
    return k3::moe_ws_layout(c, T, nullptr, nullptr);
}

extern "C" int k3gpu_moe_prefill(float *out, int *idx, float *wt, const float *x, const K3GpuMoeW *w,
                                 const K3GpuMoeCfg *c, int T, void *workspace, size_t ws_bytes, void *stream)
{
    using namespace k3;
    if (!out || !idx || !wt || !x || !w || !moe_cfg_ok(c) || !workspace || T <= 0) return K3GPU_EINVAL;
    if (!w->down || !w->up || !w->gate_W || !w->bank) return K3GPU_EINVAL;
    if (c->shared_inter > 0 && (!w->sh1 || !w->sh2 || !w->sh3)) return K3GPU_EINVAL;
    if (w->bank->L != c->latent || w->bank->I != c->moe_inter || w->bank->n_experts != c->n_routed)
        return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_moe_prefill_workspace(c, T)) return K3GPU_ECAPACITY;
    const int E = c->hidden, L = c->latent, SI = c->shared_inter;
    cudaStream_t s = as_stream(stream);
    MoeWs m;
    moe_ws_layout(c, T, &m, static_cast<char *>(workspace));
    int st;
    auto mm = [&](float *Y, const float *X, const uint16_t *W, int n_in, int n_out) {
        return k3gpu_matmul_bf16_batch(Y, n_out, X, n_in, W, n_in, n_out, T, m.mm, m.mm_bytes, stream);
    };
    // 2. down-projection (routing reads x, not z, so the order changes nothing)
    if ((st = mm(m.z, x, w->down, E, L))) return st;
    // 1. route on the full-width x
    if ((st = k3gpu_router(idx, wt, x, w->gate_W, w->gate_bias, T, E, c->n_routed, c->topk, c->renorm,
                           c->routed_scale, m.router, m.router_bytes, stream)))
        return st;
    // 3, 4. the routed experts at the latent width, summed in top-k order, then the norm
    if ((st = k3gpu_moe_experts(m.acc, m.z, idx, wt, w->bank, T, c->topk, c->n_routed, 0, c->act, c->situ_b1,
                                c->situ_b2, w->latent_norm, c->rms_eps, m.experts, m.experts_bytes, stream)))
        return st;
    // 5. up-projection
    if ((st = mm(out, m.acc, w->up, L, E))) return st;
    // 6. the dense shared expert on x, added unweighted
    if (SI > 0) {
        if ((st = mm(m.g, x, w->sh1, E, SI))) return st;
        if ((st = mm(m.u, x, w->sh3, E, SI))) return st;
        const long long n = (long long)T * SI;
        glu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m.g, m.g, m.u, n, c->act, c->situ_b1, c->situ_b2);
        if ((st = launch_status())) return st;
        if ((st = mm(m.d, m.g, w->sh2, SI, E))) return st;
        if ((st = add_launch(out, out, m.d, (long long)T * E, s))) return st;
    }
    return K3GPU_OK;
}

extern "C" size_t k3gpu_kda_layer_workspace(const K3GpuLayerCfg *c, int B, int T)
{
    if (!k3::cfg_ok(c) || B <= 0 || T <= 0) return 0;
    return k3::kda_ws_layout(c, B * T, nullptr, nullptr);
}

extern "C" int k3gpu_kda_layer_verify(float *out, const float *x, const K3GpuKdaW *w,
                                      const K3GpuLayerCfg *c, const float *state,
                                      const float *conv_hist, const K3GpuKdaLog *log, int B,
                                      int T, void *workspace, size_t ws_bytes, void *stream)
{
    return k3gpu_kda_layer_verify_tree(out, x, w, c, state, conv_hist, log, nullptr, B, T, workspace, ws_bytes,
                                       stream);
}

extern "C" int k3gpu_kda_layer_verify_tree(float *out, const float *x, const K3GpuKdaW *w,
                                           const K3GpuLayerCfg *c, const float *state,
                                           const float *conv_hist, const K3GpuKdaLog *log,
                                           const int *parent, int B, int T, void *workspace,
                                           size_t ws_bytes, void *stream)
{
    using namespace k3;
    if (!out || !x || !w || !cfg_ok(c) || !state || !conv_hist || !log || !workspace) return K3GPU_EINVAL;
    if (!log->k || !log->v || !log->alpha || !log->beta || !log->pre) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0) return K3GPU_EINVAL;
    const int E = c->hidden, H = c->kda_heads, D = c->kda_head_dim, P = H * D, R = B * T;
    if (ws_bytes < k3gpu_kda_layer_workspace(c, B, T)) return K3GPU_ECAPACITY;
    KdaWs s;
    kda_ws_layout(c, R, &s, static_cast<char *>(workspace));
    int st;
    // 1. projections, each matrix once over all B*T positions
    auto mm = [&](float *Y, const float *X, const uint16_t *W, int n_in, int n_out) {
        return k3gpu_matmul_bf16_batch(Y, n_out, X, n_in, W, n_in, n_out, R, s.mm, s.mm_bytes, stream);
    };
    if ((st = mm(s.q, x, w->q, E, P))) return st;
    if ((st = mm(log->k, x, w->k, E, P))) return st;
    if ((st = mm(log->v, x, w->v, E, P))) return st;
    if ((st = mm(s.bt, x, w->b, E, H))) return st;
    if ((st = mm(s.fa, x, w->f_a, E, D))) return st;       // the shared low-rank pair
    if ((st = mm(s.z, s.fa, w->f_b, D, P))) return st;
    // 2-5. ShortConv + SiLU, L2 norm, beta, decay; the pre-conv rows go to the log
    // (with a draft tree, along each node's ancestors)
    if ((st = k3gpu_kda_prologue_tree(s.q, log->k, log->v, log->alpha, log->beta, log->pre, s.z, s.bt, w->q_conv,
                                      w->k_conv, w->v_conv, conv_hist, w->A_log, w->dt_bias, parent, B, T, H, D,
                                      c->conv_k, c->gate_lb, stream)))
        return st;
    // 6. the recurrence on the carried state (read only), q scaled by D^-1/2 in float
    const float qscale = 1.0f / sqrtf((float)D);
    st = parent ? k3gpu_kda_verify_tree(s.o, state, s.q, log->k, log->v, log->alpha, log->beta, parent, B, T, H, D,
                                        qscale, stream)
                : k3gpu_kda_verify(s.o, state, s.q, log->k, log->v, log->alpha, log->beta, B, T, H, D, qscale,
                                   stream);
    if (st) return st;
    // 7-9. head RMSNorm, then the gate, then the output projection
    if ((st = mm(s.g, x, w->g, E, P))) return st;
    if ((st = k3gpu_kda_norm_gate(s.o, s.g, w->o_norm, R, H, D, c->rms_eps, stream))) return st;
    return mm(out, s.o, w->o, P, E);
}

extern "C" size_t k3gpu_mla_layer_workspace(const K3GpuLayerCfg *c, int B, int T, int max_ctx)
{
    if (!k3::mla_cfg_ok(c) || B <= 0 || T <= 0 || max_ctx <= 0) return 0;
    return k3::mla_ws_layout(c, B, T, max_ctx, nullptr, nullptr);
}

extern "C" int k3gpu_mla_layer_verify(float *out, const float *x, const K3GpuMlaW *w, const K3GpuLayerCfg *c,
                                      uint16_t *lat, uint16_t *rope, int cap, const int *cached,
                                      const uint64_t *mask, int max_ctx, int B, int T, void *workspace,
                                      size_t ws_bytes, void *stream)
{
    using namespace k3;
    if (!out || !x || !w || !mla_cfg_ok(c) || !lat || !cached || !mask || !workspace) return K3GPU_EINVAL;
    if (!w->q_a || !w->q_b || !w->kv_a || !w->o || !w->q_a_norm || !w->kv_a_norm || !w->kv_b) return K3GPU_EINVAL;
    if (c->qk_rope > 0 && !rope) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || cap <= 0 || max_ctx <= 0 || max_ctx > cap) return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_mla_layer_workspace(c, B, T, max_ctx)) return K3GPU_ECAPACITY;
    const int E = c->hidden, H = c->mla_heads, qn = c->qk_nope, qr = c->qk_rope, vh = c->v_head;
    const int kvl = c->kv_lora, kvw = kvl + qr, R = B * T;
    cudaStream_t s = as_stream(stream);
    MlaLWs m;
    mla_ws_layout(c, B, T, max_ctx, &m, static_cast<char *>(workspace));
    int st;
    auto mm = [&](float *Y, const float *X, const uint16_t *W, int n_in, int n_out) {
        return k3gpu_matmul_bf16_batch(Y, n_out, X, n_in, W, n_in, n_out, R, m.mm, m.mm_bytes, stream);
    };
    // projections (:1186-1200): q_a, its norm, q_b; kv_a, then the new cache rows
    if ((st = mm(m.ql, x, w->q_a, E, c->q_lora))) return st;
    if ((st = k3gpu_rmsnorm(m.qln, m.ql, w->q_a_norm, R, c->q_lora, c->rms_eps, stream))) return st;
    if ((st = mm(m.q, m.qln, w->q_b, c->q_lora, H * (qn + qr)))) return st;
    if ((st = mm(m.ct, x, w->kv_a, E, kvw))) return st;
    mla_append_kernel<<<R, AP_THREADS, 0, s>>>(lat, rope, m.ct, w->kv_a_norm, cached, T, cap, kvl, qr, c->rms_eps);
    if ((st = launch_status())) return st;
    const long long nq = (long long)R * H * (qn + qr);
    mla_qsplit_kernel<<<(unsigned)((nq + 255) / 256), 256, 0, s>>>(m.qnp, m.qrp, m.q, nq, qn, qr);
    if ((st = launch_status())) return st;
    // absorbed attention over the cache (the scale is over the full head width, :1124)
    const float scale = 1.0f / sqrtf((float)(qn + qr));
    if ((st = k3gpu_mla_absorbed(m.acc, m.qnp, qr ? m.qrp : nullptr, w->kv_b, lat, rope, cached, mask, B, T, H, qn,
                                 qr, vh, kvl, cap, max_ctx, scale, m.att, m.att_bytes, stream)))
        return st;
    // the gate before o_proj, no norm (:1603-1609)
    if (w->g) {
        if ((st = mm(m.g, x, w->g, E, H * vh))) return st;
        const long long n = (long long)R * H * vh;
        mla_gate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m.acc, m.g, n);
        if ((st = launch_status())) return st;
    }
    return mm(out, m.acc, w->o, H * vh, E);
}

namespace k3 {
struct LayerWs {
    float *pref, *tmp, *hin;
    char *attn, *moe;
    size_t attn_bytes, moe_bytes;
};

static K3GpuMoeCfg moe_cfg_of(const K3GpuLayerCfg *c)
{
    K3GpuMoeCfg m;
    m.hidden = c->hidden; m.latent = c->latent; m.moe_inter = c->moe_inter; m.shared_inter = c->shared_inter;
    m.n_routed = c->n_routed; m.topk = c->topk; m.act = c->act; m.renorm = c->renorm;
    m.routed_scale = c->routed_scale; m.situ_b1 = c->situ_b1; m.situ_b2 = c->situ_b2; m.rms_eps = c->rms_eps;
    return m;
}

static size_t layer_ws_layout(const K3GpuLayerCfg *c, int B, int T, size_t attn_bytes, LayerWs *w, char *base)
{
    const int E = c->hidden, R = B * T;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return r;
    };
    LayerWs t;
    t.pref = (float *)take((size_t)R * E * 4);
    t.tmp = (float *)take((size_t)R * E * 4);
    t.hin = (float *)take((size_t)R * E * 4);
    t.attn_bytes = attn_bytes;
    t.attn = take(t.attn_bytes);
    t.moe_bytes = k3gpu_moe_workspace(R, c->topk, c->n_shared, E, c->moe_inter, c->n_routed);
    if (c->latent > 0) {
        const K3GpuMoeCfg mc = moe_cfg_of(c);
        t.moe_bytes = std::max(t.moe_bytes, k3gpu_moe_prefill_workspace(&mc, R));
    }
    t.moe = take(t.moe_bytes);
    if (w) *w = t;
    return o;
}
}  // namespace k3

#include "layer.cuh"

namespace k3 {
static bool layer_common_ok(const K3GpuLayerCfg *c)
{
    return c && c->hidden > 0 && c->topk > 0 && c->n_routed > 0 && c->attn_res_block > 0 && c->max_blocks > 0;
}

// k3_decoder_layer_core (src/core/k3_ops.c:2485-2592) with the attention as a callable
// attn(out, in, workspace, bytes); LW is K3GpuKdaLayerW or K3GpuMlaLayerW
template <class LW, class Attn>
static int decoder_layer(float *h, float *block_residual, int *n_blocks, int *moe_idx, float *moe_wt, const LW *w,
                         const K3GpuLayerCfg *c, int layer_idx, int B, int T, const LayerWs &ws, Attn attn,
                         cudaStream_t s, void *stream, const LayerEp *ep)
{
    const int E = c->hidden, R = B * T, maxb = c->max_blocks;
    const long long n = (long long)R * E;
    int st;
    // the running residual starts as the layer input
    if ((st = cuda_status(cudaMemcpyAsync(ws.pref, h, (size_t)n * 4, cudaMemcpyDeviceToDevice, s)))) return st;
    // AttnRes before attention (src/core/k3_ops.c:2514-2525); with no snapshot a
    // position's only source is the running residual itself and h is unchanged
    if ((st = k3gpu_attn_res(h, block_residual, ws.pref, w->attn_res_fold, n_blocks, R, maxb, E, c->rms_eps,
                             stream)))
        return st;
    // block boundary: snapshot the running residual, then restart it (:2527-2533)
    const bool boundary = layer_idx % c->attn_res_block == 0;
    if (boundary) {
        snapshot_kernel<<<R, 256, 0, s>>>(block_residual, n_blocks, ws.pref, maxb, E);
        if ((st = launch_status())) return st;
    }
    // attention (:2535-2542)
    if ((st = k3gpu_rmsnorm(ws.hin, h, w->in_norm, R, E, c->rms_eps, stream))) return st;
    if ((st = attn(ws.tmp, ws.hin, ws.attn, ws.attn_bytes))) return st;
    if (boundary) st = cuda_status(cudaMemcpyAsync(ws.pref, ws.tmp, (size_t)n * 4, cudaMemcpyDeviceToDevice, s));
    else st = add_launch(ws.pref, ws.pref, ws.tmp, n, s);
    if (st) return st;
    // AttnRes before the MLP, no emptiness guard (:2544-2557), then post_norm
    if ((st = k3gpu_attn_res(h, block_residual, ws.pref, w->mlp_res_fold, n_blocks, R, maxb, E, c->rms_eps,
                             stream)))
        return st;
    if ((st = k3gpu_rmsnorm(ws.hin, h, w->post_norm, R, E, c->rms_eps, stream))) return st;
    // the MoE: the K3 form (latent projections, dense shared expert) or the single-layer
    // form (router and experts at the hidden width)
    if (ep) {        // the routed experts split over the ranks of ep->g, rows through peer memory
        st = k3gpu_moe_layer_ep(ws.tmp, moe_idx, moe_wt, ws.hin, w->gate_W, w->gate_bias, w->bank, ep->shared, ep->g,
                                ep->seq, R, c->topk, c->n_routed, c->n_shared, c->act, c->situ_b1, c->situ_b2,
                                c->renorm, c->routed_scale, ep->ok, ep->ws, ep->ws_bytes, stream);
    } else if (w->moe) {
        const K3GpuMoeCfg mc = moe_cfg_of(c);
        st = k3gpu_moe_prefill(ws.tmp, moe_idx, moe_wt, ws.hin, w->moe, &mc, R, ws.moe, ws.moe_bytes, stream);
    } else {
        st = k3gpu_moe_layer(ws.tmp, moe_idx, moe_wt, ws.hin, w->gate_W, w->gate_bias, w->bank, R, c->topk,
                             c->n_routed, c->n_shared, c->act, c->situ_b1, c->situ_b2, c->renorm, c->routed_scale,
                             ws.moe, ws.moe_bytes, stream);
    }
    if (st) return st;
    return add_launch(h, ws.pref, ws.tmp, n, s);
}

template <class LW>
static int moe_args_ok(const LW *w, const K3GpuLayerCfg *c)
{
    if (!w->moe && (!w->bank || w->bank->L != c->hidden || w->bank->I != c->moe_inter)) return 0;
    if (w->moe && c->latent <= 0) return 0;
    return 1;
}
}  // namespace k3

extern "C" size_t k3gpu_decoder_layer_workspace(const K3GpuLayerCfg *c, int B, int T)
{
    if (!k3::cfg_ok(c) || !k3::layer_common_ok(c) || B <= 0 || T <= 0) return 0;
    return k3::layer_ws_layout(c, B, T, k3gpu_kda_layer_workspace(c, B, T), nullptr, nullptr);
}

extern "C" int k3gpu_decoder_layer_kda_verify(float *h, float *block_residual, int *n_blocks,
                                              int *moe_idx, float *moe_wt, const K3GpuKdaLayerW *w,
                                              const K3GpuLayerCfg *c, int layer_idx, const float *state,
                                              const float *conv_hist, const K3GpuKdaLog *log, int B, int T,
                                              void *workspace, size_t ws_bytes, void *stream)
{
    return k3gpu_decoder_layer_kda_verify_tree(h, block_residual, n_blocks, moe_idx, moe_wt, w, c, layer_idx, state,
                                               conv_hist, log, nullptr, B, T, workspace, ws_bytes, stream);
}

extern "C" int k3gpu_decoder_layer_kda_verify_tree(float *h, float *block_residual, int *n_blocks,
                                                   int *moe_idx, float *moe_wt, const K3GpuKdaLayerW *w,
                                                   const K3GpuLayerCfg *c, int layer_idx, const float *state,
                                                   const float *conv_hist, const K3GpuKdaLog *log,
                                                   const int *parent, int B, int T, void *workspace,
                                                   size_t ws_bytes, void *stream)
{
    return k3::decoder_layer_kda(h, block_residual, n_blocks, moe_idx, moe_wt, w, c, layer_idx, state, conv_hist, log,
                                 parent, B, T, workspace, ws_bytes, stream, nullptr);
}

int k3::decoder_layer_kda(float *h, float *block_residual, int *n_blocks, int *moe_idx, float *moe_wt,
                          const K3GpuKdaLayerW *w, const K3GpuLayerCfg *c, int layer_idx, const float *state,
                          const float *conv_hist, const K3GpuKdaLog *log, const int *parent, int B, int T,
                          void *workspace, size_t ws_bytes, void *stream, const LayerEp *ep)
{
    using namespace k3;
    if (!h || !block_residual || !n_blocks || !moe_idx || !moe_wt || !w || !cfg_ok(c) || !layer_common_ok(c) ||
        !workspace)
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || layer_idx < 0 || !moe_args_ok(w, c)) return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_decoder_layer_workspace(c, B, T)) return K3GPU_ECAPACITY;
    LayerWs ws;
    layer_ws_layout(c, B, T, k3gpu_kda_layer_workspace(c, B, T), &ws, static_cast<char *>(workspace));
    auto attn = [&](float *out, const float *in, void *aws, size_t abytes) {
        return k3gpu_kda_layer_verify_tree(out, in, &w->kda, c, state, conv_hist, log, parent, B, T, aws, abytes,
                                           stream);
    };
    return decoder_layer(h, block_residual, n_blocks, moe_idx, moe_wt, w, c, layer_idx, B, T, ws, attn,
                         as_stream(stream), stream, ep);
}

extern "C" size_t k3gpu_decoder_layer_mla_workspace(const K3GpuLayerCfg *c, int B, int T, int max_ctx)
{
    if (!k3::mla_cfg_ok(c) || !k3::layer_common_ok(c) || B <= 0 || T <= 0 || max_ctx <= 0) return 0;
    return k3::layer_ws_layout(c, B, T, k3gpu_mla_layer_workspace(c, B, T, max_ctx), nullptr, nullptr);
}

extern "C" int k3gpu_decoder_layer_mla_verify(float *h, float *block_residual, int *n_blocks,
                                              int *moe_idx, float *moe_wt, const K3GpuMlaLayerW *w,
                                              const K3GpuLayerCfg *c, int layer_idx, uint16_t *lat,
                                              uint16_t *rope, int cap, const int *cached,
                                              const uint64_t *mask, int max_ctx, int B, int T,
                                              void *workspace, size_t ws_bytes, void *stream)
{
    return k3::decoder_layer_mla(h, block_residual, n_blocks, moe_idx, moe_wt, w, c, layer_idx, lat, rope, cap, cached,
                                 mask, max_ctx, B, T, workspace, ws_bytes, stream, nullptr);
}

int k3::decoder_layer_mla(float *h, float *block_residual, int *n_blocks, int *moe_idx, float *moe_wt,
                          const K3GpuMlaLayerW *w, const K3GpuLayerCfg *c, int layer_idx, uint16_t *lat,
                          uint16_t *rope, int cap, const int *cached, const uint64_t *mask, int max_ctx, int B,
                          int T, void *workspace, size_t ws_bytes, void *stream, const LayerEp *ep)
{
    using namespace k3;
    if (!h || !block_residual || !n_blocks || !moe_idx || !moe_wt || !w || !mla_cfg_ok(c) ||
        !layer_common_ok(c) || !workspace)
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || layer_idx < 0 || !moe_args_ok(w, c)) return K3GPU_EINVAL;
    const size_t need = k3gpu_decoder_layer_mla_workspace(c, B, T, max_ctx);
    if (need == 0) return K3GPU_EINVAL;
    if (ws_bytes < need) return K3GPU_ECAPACITY;
    LayerWs ws;
    layer_ws_layout(c, B, T, k3gpu_mla_layer_workspace(c, B, T, max_ctx), &ws, static_cast<char *>(workspace));
    auto attn = [&](float *out, const float *in, void *aws, size_t abytes) {
        return k3gpu_mla_layer_verify(out, in, &w->mla, c, lat, rope, cap, cached, mask, max_ctx, B, T, aws, abytes,
                                      stream);
    };
    return decoder_layer(h, block_residual, n_blocks, moe_idx, moe_wt, w, c, layer_idx, B, T, ws, attn,
                         as_stream(stream), stream, ep);
}
