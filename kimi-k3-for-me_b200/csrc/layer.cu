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
// k3gpu_decoder_layer_kda_verify is k3_decoder_layer_core (src/core/k3_ops.c:2485-2592)
// for that layer: AttnRes before attention over each position's block-residual snapshots,
// the block-boundary snapshot (then the running residual restarts from the attention
// output), input RMSNorm, the KDA layer, AttnRes before the MLP, post RMSNorm, the MoE, and
// the residual. The MoE is either the single-layer form (router and MXFP4 experts at the
// hidden width, shared experts in the bank) or the K3 form of k3_moe_prefill
// (src/core/k3_ops.c:2008-2053, 1848-1860): routing on x, the MXFP4 experts on the latent
// down-projection, the latent RMSNorm, the up-projection, and the dense bf16 shared expert.
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
    if ((st = k3gpu_kda_prologue(s.q, log->k, log->v, log->alpha, log->beta, log->pre, s.z, s.bt, w->q_conv,
                                 w->k_conv, w->v_conv, conv_hist, w->A_log, w->dt_bias, B, T, H, D, c->conv_k,
                                 c->gate_lb, stream)))
        return st;
    // 6. the recurrence on the carried state (read only), q scaled by D^-1/2 in float
    const float qscale = 1.0f / sqrtf((float)D);
    if ((st = k3gpu_kda_verify(s.o, state, s.q, log->k, log->v, log->alpha, log->beta, B, T, H, D, qscale,
                               stream)))
        return st;
    // 7-9. head RMSNorm, then the gate, then the output projection
    if ((st = mm(s.g, x, w->g, E, P))) return st;
    if ((st = k3gpu_kda_norm_gate(s.o, s.g, w->o_norm, R, H, D, c->rms_eps, stream))) return st;
    return mm(out, s.o, w->o, P, E);
}

namespace k3 {
struct LayerWs {
    float *pref, *tmp, *hin;
    char *kda, *moe;
    size_t kda_bytes, moe_bytes;
};

static K3GpuMoeCfg moe_cfg_of(const K3GpuLayerCfg *c)
{
    K3GpuMoeCfg m;
    m.hidden = c->hidden; m.latent = c->latent; m.moe_inter = c->moe_inter; m.shared_inter = c->shared_inter;
    m.n_routed = c->n_routed; m.topk = c->topk; m.act = c->act; m.renorm = c->renorm;
    m.routed_scale = c->routed_scale; m.situ_b1 = c->situ_b1; m.situ_b2 = c->situ_b2; m.rms_eps = c->rms_eps;
    return m;
}

static size_t layer_ws_layout(const K3GpuLayerCfg *c, int B, int T, LayerWs *w, char *base)
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
    t.kda_bytes = k3gpu_kda_layer_workspace(c, B, T);
    t.kda = take(t.kda_bytes);
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

extern "C" size_t k3gpu_decoder_layer_workspace(const K3GpuLayerCfg *c, int B, int T)
{
    if (!k3::cfg_ok(c) || B <= 0 || T <= 0 || c->topk <= 0 || c->n_routed <= 0) return 0;
    return k3::layer_ws_layout(c, B, T, nullptr, nullptr);
}

extern "C" int k3gpu_decoder_layer_kda_verify(float *h, float *block_residual, int *n_blocks,
                                              int *moe_idx, float *moe_wt, const K3GpuKdaLayerW *w,
                                              const K3GpuLayerCfg *c, int layer_idx, const float *state,
                                              const float *conv_hist, const K3GpuKdaLog *log, int B, int T,
                                              void *workspace, size_t ws_bytes, void *stream)
{
    using namespace k3;
    if (!h || !block_residual || !n_blocks || !moe_idx || !moe_wt || !w || !cfg_ok(c) || !workspace)
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || layer_idx < 0 || c->attn_res_block <= 0 || c->max_blocks <= 0) return K3GPU_EINVAL;
    if (!w->moe && (!w->bank || w->bank->L != c->hidden || w->bank->I != c->moe_inter)) return K3GPU_EINVAL;
    if (w->moe && c->latent <= 0) return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_decoder_layer_workspace(c, B, T)) return K3GPU_ECAPACITY;
    const int E = c->hidden, R = B * T, maxb = c->max_blocks;
    const long long n = (long long)R * E;
    cudaStream_t s = as_stream(stream);
    LayerWs ws;
    layer_ws_layout(c, B, T, &ws, static_cast<char *>(workspace));
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
    if ((st = k3gpu_kda_layer_verify(ws.tmp, ws.hin, &w->kda, c, state, conv_hist, log, B, T, ws.kda,
                                     ws.kda_bytes, stream)))
        return st;
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
    if (w->moe) {
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
