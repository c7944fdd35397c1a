// model.cu -- the verify forward of a whole model: the reference's forward() with arg_all
// (src/cli/k3_run.c:853-1138) over B sequences on the device, and the commit behind the
// speculative sweep (spec_commit, :1270-1300, plus `cached += keep`, :2941-2943).
//
// A sweep feeds T positions per sequence from each sequence's cache position: embed rows
// (k3_embed_row), every decoder layer in order (k3_decoder_layer_inc_log: KDA layers
// tentative and logged, MLA layers appending their rows to the cache at cached + t), the
// model-level AttnRes over the block snapshots (:1071-1087), the final RMSNorm, the lm_head
// over every position and the per-position argmax (:1089-1130). The KDA state is never
// touched by a sweep; the commit replays the first keep logged positions (k3_kda_advance)
// and advances cached, so rejected drafts cost nothing to roll back. With a draft tree the
// accepted path's log rows and cache rows are gathered to the front first.
//
// Memory: everything the model holds on the device sits in one caller-owned arena (the
// reference's rule that buffers are caller-owned, docs/API.md:47-64):
//   per KDA layer   state [B][H][D][D], ShortConv history [B][3][P][K-1], the sweep log
//   per MLA layer   bf16 latent cache [B][cap][kv_lora] and rope cache [B][cap][qk_rope]
//   per sweep       h, snapshots [B*T][maxb][E], normed rows, logits [B*T][vocab], the
//                   routing of the last layer, the largest layer workspace
// The host object holds only pointers and small host mirrors (cached per sequence).
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "common.cuh"
#include "layer.cuh"

namespace k3 {

// h[r] = embed[ids[r]] widened exactly from bf16; an id outside the vocabulary gives a
// zero row and is flagged
__global__ void __launch_bounds__(256) embed_kernel(float *__restrict__ h, const uint16_t *__restrict__ embed,
                                                   const int *__restrict__ ids, int E, int vocab)
{
    const int r = blockIdx.x;
    const int id = ids[r];
    float *dst = h + (size_t)r * E;
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
        for (int i = threadIdx.x; i < E; i += 256) dst[i] = 0.0f;
        return;
    }
    const uint16_t *src = embed + (size_t)id * E;
    for (int i = threadIdx.x; i < E; i += 256) dst[i] = __uint_as_float((unsigned)src[i] << 16);
}

// dst[b] = src[b * T + T - 1] (row width E): the last position of every sequence
__global__ void __launch_bounds__(256) last_rows_kernel(float *__restrict__ dst, const float *__restrict__ src, int T,
                                                       int E)
{
    const int b = blockIdx.x;
    const float *s = src + ((size_t)b * T + T - 1) * E;
    for (int i = threadIdx.x; i < E; i += 256) dst[(size_t)b * E + i] = s[i];
}

__global__ void cached_add_kernel(int *__restrict__ cached, const int *__restrict__ keep, int B, int T)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int n = keep[b];
    if (n < 0 || n > T) {
        flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : T;
    }
    cached[b] += n;
}

// One CTA per (sequence, array): rows[b][j] = rows[b][path[b][j]] for j < keep[b], in
// ascending j. A path is root first with strictly increasing node indices (parents come
// before children), so path[j] >= j and the rows read at step j are never ones written
// before it. rows: [B][T][w] floats (w a multiple of 4 when vec); path [B][T].
__global__ void __launch_bounds__(256) gather_path_f32_kernel(float *__restrict__ rows, const int *__restrict__ path,
                                                              const int *__restrict__ keep, int T, long long w)
{
    const int b = blockIdx.x;
    int n = keep[b];
    if (n < 0 || n > T) {
        if (threadIdx.x == 0) flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : T;
    }
    float *base = rows + (size_t)b * T * w;
    for (int j = 0; j < n; j++) {
        const int src = path[(size_t)b * T + j];
        if (src < j || src >= T) {             // uniform: every thread reads the same entry
            if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
            break;
        }
        if (src != j)
            for (long long i = threadIdx.x; i < w; i += 256) base[(size_t)j * w + i] = base[(size_t)src * w + i];
        __syncthreads();
    }
}

// The same gather for cache rows: rows [B][cap][w] bf16 from position cached[b] on.
__global__ void __launch_bounds__(256) gather_path_bf16_kernel(uint16_t *__restrict__ rows,
                                                               const int *__restrict__ path,
                                                               const int *__restrict__ keep,
                                                               const int *__restrict__ cached, int T, int cap, int w)
{
    const int b = blockIdx.x;
    int n = keep[b];
    if (n < 0 || n > T) {
        if (threadIdx.x == 0) flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : T;
    }
    const int c0 = cached[b];
    if (c0 < 0 || c0 + T > cap) {
        if (threadIdx.x == 0) flag(DEV_BAD_POSITION);
        return;
    }
    uint16_t *base = rows + ((size_t)b * cap + c0) * w;
    for (int j = 0; j < n; j++) {
        const int src = path[(size_t)b * T + j];
        if (src < j || src >= T) {
            if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
            break;
        }
        if (src != j)
            for (int i = threadIdx.x; i < w; i += 256) base[(size_t)j * w + i] = base[(size_t)src * w + i];
        __syncthreads();
    }
}

}  // namespace k3

struct K3GpuModel {
    K3GpuModelCfg cfg;
    std::vector<int> is_mla;
    std::vector<K3GpuKdaLayerW> kda;
    std::vector<K3GpuMlaLayerW> mla;
    K3GpuModelW w;
    int B, maxT, cap, maxb;
    void *stream;
    // device
    std::vector<float *> kstate, khist;
    std::vector<K3GpuKdaLog> klog;
    std::vector<uint16_t *> lat, rope;
    std::vector<int> slot;          // per layer: its KDA or MLA slot
    int *cached, *nb, *ids, *keep, *path, *moe_idx, *arg, *parent_dev;
    float *h, *br, *nrm, *last, *logits, *moe_wt;
    uint64_t *mask;
    char *ws;
    size_t ws_bytes;
    // host: pinned staging for the small per-call uploads (masks, keep counts, paths,
    // loop ids and args), a ring of NSTAGE slots so the host can run a few calls ahead of
    // the device; ev[i] marks the last copy that read slot i, and the host waits on it
    // before writing that slot again
    static constexpr int NSTAGE = 4;
    char *stage = nullptr;
    size_t stage_bytes = 0;
    cudaEvent_t ev[NSTAGE] = {};
    int stage_next = 0;
    std::vector<int> cached_host;
    int last_T, last_tree, pre_committed;   // the sweep awaiting its commit
    // expert parallel (k3gpu_model_set_ep): every layer's MoE step exchanges rows with the
    // other ranks; seq numbers the exchange steps, the same on every rank
    bool ep_on = false;
    K3GpuEpGroup ep_group{};
    std::vector<const K3GpuExpertBank *> ep_shared;
    int *ep_ok = nullptr;
    char *ep_ws = nullptr;
    size_t ep_ws_bytes = 0;
    unsigned ep_seq = 0;
    std::vector<int> parent_host;
    std::vector<uint64_t> mask_host;
    ~K3GpuModel()
    {
        for (cudaEvent_t e : ev)
            if (e) {
                cudaEventSynchronize(e);
                cudaEventDestroy(e);
            }
        if (stage) cudaFreeHost(stage);
    }
};


namespace k3 {

static bool model_cfg_ok(const K3GpuModelCfg *c)
{
    if (!c || c->n_layers <= 0 || c->n_layers > 4096 || c->vocab <= 0 || !c->is_mla) return false;
    const K3GpuLayerCfg &l = c->layer;
    if (l.hidden <= 0 || l.hidden % 8 != 0 || l.attn_res_block <= 0 || l.topk <= 0 || l.n_routed <= 0) return false;
    const int snaps = (c->n_layers + l.attn_res_block - 1) / l.attn_res_block;
    if (l.max_blocks < snaps || l.max_blocks + 1 > 256) return false;
    int n_kda = 0, n_mla = 0;
    for (int i = 0; i < c->n_layers; i++) (c->is_mla[i] ? n_mla : n_kda)++;
    if (n_kda && k3gpu_kda_layer_workspace(&l, 1, 1) == 0) return false;
    if (n_mla && k3gpu_mla_layer_workspace(&l, 1, 1, 1) == 0) return false;
    return true;
}

// The MLA layer's workspace for any context up to cap: the attention's slice count is not
// monotonic in the context, so take the largest over every 128-position tile count.
static size_t mla_ws_any_ctx(const K3GpuLayerCfg *l, int B, int T, int cap)
{
    size_t ws = k3gpu_decoder_layer_mla_workspace(l, B, T, cap);
    for (int ctx = 128; ctx < cap; ctx += 128) ws = std::max(ws, k3gpu_decoder_layer_mla_workspace(l, B, T, ctx));
    return ws;
}

// The arena: every region 256-byte aligned, in a fixed order; m == nullptr only sizes.
static size_t model_layout(const K3GpuModelCfg *c, int B, int maxT, int cap, K3GpuModel *m, char *base)
{
    const K3GpuLayerCfg &l = c->layer;
    const int E = l.hidden, R = B * maxT, V = c->vocab;
    const int H = l.kda_heads, D = l.kda_head_dim, P = H * D, K = l.conv_k;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return r;
    };
    size_t ws = 0, ws_mla = 0;
    bool any_mla = false;
    for (int i = 0; i < c->n_layers; i++) {
        if (c->is_mla[i]) {
            uint16_t *lt = (uint16_t *)take((size_t)B * cap * l.kv_lora * 2);
            uint16_t *rp = l.qk_rope ? (uint16_t *)take((size_t)B * cap * l.qk_rope * 2) : nullptr;
            if (m) {
                m->slot.push_back((int)m->lat.size());
                m->lat.push_back(lt);
                m->rope.push_back(rp);
            }
            any_mla = true;
        } else {
            float *st = (float *)take((size_t)B * H * D * D * 4);
            float *hi = (float *)take((size_t)B * 3 * P * (K - 1) * 4);
            K3GpuKdaLog lg;
            lg.k = (float *)take((size_t)R * P * 4);
            lg.v = (float *)take((size_t)R * P * 4);
            lg.alpha = (float *)take((size_t)R * P * 4);
            lg.beta = (float *)take((size_t)R * H * 4);
            lg.pre = (float *)take((size_t)R * 3 * P * 4);
            if (m) {
                m->slot.push_back((int)m->kstate.size());
                m->kstate.push_back(st);
                m->khist.push_back(hi);
                m->klog.push_back(lg);
            }
            ws = std::max(ws, k3gpu_decoder_layer_workspace(&l, B, maxT));
        }
    }
    if (any_mla) ws_mla = mla_ws_any_ctx(&l, B, maxT, cap);
    ws = std::max(ws, ws_mla);
    ws = std::max(ws, k3gpu_matmul_bf16_workspace(R, E, V));
    ws = std::max(ws, k3gpu_lm_head_argmax_workspace(R, E, V));
    char *cached = take((size_t)B * 4);
    char *nb = take((size_t)R * 4);
    char *ids = take((size_t)R * 4);
    char *keep = take((size_t)B * 4);
    char *path = take((size_t)R * 4);
    char *arg = take((size_t)R * 4);
    char *moe_idx = take((size_t)R * l.topk * 4);
    char *moe_wt = take((size_t)R * l.topk * 4);
    char *mask = take((size_t)maxT * 8);
    char *parent = take((size_t)maxT * 4);
    char *h = take((size_t)R * E * 4);
    char *br = take((size_t)R * l.max_blocks * E * 4);
    char *nrm = take((size_t)R * E * 4);
    char *last = take((size_t)B * E * 4);
    char *logits = take((size_t)R * V * 4);
    char *wsp = take(ws);
    if (m) {
        m->cached = (int *)cached; m->nb = (int *)nb; m->ids = (int *)ids; m->keep = (int *)keep;
        m->path = (int *)path; m->arg = (int *)arg; m->moe_idx = (int *)moe_idx; m->moe_wt = (float *)moe_wt;
        m->mask = (uint64_t *)mask; m->parent_dev = (int *)parent; m->h = (float *)h; m->br = (float *)br; m->nrm = (float *)nrm;
        m->last = (float *)last; m->logits = (float *)logits; m->ws = wsp; m->ws_bytes = ws;
    }
    return o;
}

// ancestor masks of a tree given as parents (parent[0] = -1, parent[i] < i), or of a chain
static int build_masks(const int *parent, int T, uint64_t *mask)
{
    for (int t = 0; t < T; t++) {
        if (!parent) {
            mask[t] = t == 63 ? ~0ull : ((1ull << (t + 1)) - 1);
            continue;
        }
        const int p = parent[t];
        if ((t == 0 && p != -1) || (t > 0 && (p < 0 || p >= t))) return K3GPU_EINVAL;
        mask[t] = (1ull << t) | (t ? mask[p] : 0ull);
    }
    return K3GPU_OK;
}

static bool is_chain(const int *parent, int T)
{
    if (!parent) return true;
    for (int t = 1; t < T; t++)
        if (parent[t] != t - 1) return false;
    return true;
}

// A staging slot: mask [maxT] u64 | keep [B] | path [B*maxT] | ids [B*maxT] | arg [B*maxT] |
// parent [maxT].
struct Stage {
    uint64_t *mask;
    int *keep, *path, *ids, *arg, *parent;
    int slot;
};

static size_t stage_slot_bytes(int B, int maxT)
{
    return ((size_t)maxT * 8 + ((size_t)B + 3 * (size_t)B * maxT + maxT) * 4 + 255) & ~(size_t)255;
}

// take the next slot once the copies that last read it have run
static int stage_acquire(K3GpuModel *m, Stage *st)
{
    const int i = m->stage_next;
    m->stage_next = (i + 1) % K3GpuModel::NSTAGE;
    int rc = cuda_status(cudaEventSynchronize(m->ev[i]));
    if (rc) return rc;
    char *p = m->stage + (size_t)i * stage_slot_bytes(m->B, m->maxT);
    st->mask = (uint64_t *)p;
    st->keep = (int *)(p + (size_t)m->maxT * 8);
    st->path = st->keep + m->B;
    st->ids = st->path + (size_t)m->B * m->maxT;
    st->arg = st->ids + (size_t)m->B * m->maxT;
    st->parent = st->arg + (size_t)m->B * m->maxT;
    st->slot = i;
    return K3GPU_OK;
}

// after the copies out of the slot are enqueued
static int stage_release(K3GpuModel *m, const Stage &st)
{
    return cuda_status(cudaEventRecord(m->ev[st.slot], as_stream(m->stream)));
}

// one sweep of T <= maxT positions per sequence from the device ids [B][T]; logit_rows 0:
// logits and argmax for every position, 1: for each sequence's last position only, 2: the
// argmax of every position from the lm_head fused with it (no logits written)
static int model_sweep(K3GpuModel *m, const int *ids_dev, int T, const int *parent, int logit_rows)
{
    const K3GpuLayerCfg &l = m->cfg.layer;
    const int B = m->B, E = l.hidden, R = B * T, V = m->cfg.vocab;
    cudaStream_t s = as_stream(m->stream);
    void *sp = m->stream;
    int st;
    const bool tree = !is_chain(parent, T);
    int max_ctx = 0;
    for (int b = 0; b < B; b++) max_ctx = std::max(max_ctx, m->cached_host[b] + T);
    if (max_ctx > m->cap) return K3GPU_ECAPACITY;
    Stage sg;
    if ((st = stage_acquire(m, &sg))) return st;
    if ((st = build_masks(parent, T, sg.mask))) return st;
    if ((st = cuda_status(cudaMemcpyAsync(m->mask, sg.mask, (size_t)T * 8, cudaMemcpyHostToDevice, s)))) return st;
    if (tree) {   // the KDA layers follow each node's ancestors
        std::copy(parent, parent + T, sg.parent);
        if ((st = cuda_status(cudaMemcpyAsync(m->parent_dev, sg.parent, (size_t)T * 4, cudaMemcpyHostToDevice, s))))
            return st;
    }
    if ((st = stage_release(m, sg))) return st;
    if (parent) std::copy(parent, parent + T, m->parent_host.begin());
    embed_kernel<<<R, 256, 0, s>>>(m->h, m->w.embed, ids_dev, E, V);
    if ((st = launch_status())) return st;
    if ((st = cuda_status(cudaMemsetAsync(m->nb, 0, (size_t)R * 4, s)))) return st;
    for (int i = 0; i < m->cfg.n_layers; i++) {
        const int sl = m->slot[i];
        LayerEp ep;
        if (m->ep_on) {
            ep.g = &m->ep_group;
            ep.shared = m->ep_shared[i];
            ep.seq = ++m->ep_seq;
            ep.ok = m->ep_ok;
            ep.ws = m->ep_ws;
            ep.ws_bytes = m->ep_ws_bytes;
        }
        const LayerEp *epp = m->ep_on ? &ep : nullptr;
        if (m->is_mla[i]) {
            st = decoder_layer_mla(m->h, m->br, m->nb, m->moe_idx, m->moe_wt, &m->mla[i], &l, i, m->lat[sl],
                                   m->rope[sl], m->cap, m->cached, m->mask, max_ctx, B, T, m->ws, m->ws_bytes, sp, epp);
        } else {
            st = decoder_layer_kda(m->h, m->br, m->nb, m->moe_idx, m->moe_wt, &m->kda[i], &l, i, m->kstate[sl],
                                   m->khist[sl], &m->klog[sl], tree ? m->parent_dev : nullptr, B, T, m->ws,
                                   m->ws_bytes, sp, epp);
        }
        if (st) return st;
    }
    // the model-level AttnRes over the snapshots and the final residual (:1071-1087), then
    // the final norm
    if (m->w.out_res_fold) {
        if ((st = k3gpu_attn_res(m->nrm, m->br, m->h, m->w.out_res_fold, m->nb, R, m->maxb, E, l.rms_eps, sp)))
            return st;
        if ((st = k3gpu_rmsnorm(m->nrm, m->nrm, m->w.norm, R, E, l.rms_eps, sp))) return st;
    } else if ((st = k3gpu_rmsnorm(m->nrm, m->h, m->w.norm, R, E, l.rms_eps, sp))) {
        return st;
    }
    // lm_head over every position (a verify sweep), or over each sequence's last one (a
    // read-in pass: only the next id after the pass is needed)
    if (logit_rows == 2) return k3gpu_lm_head_argmax(m->arg, m->nrm, E, m->w.lm_head, E, V, R, m->ws, m->ws_bytes, sp);
    if (logit_rows == 0) {
        if ((st = k3gpu_matmul_bf16_batch(m->logits, V, m->nrm, E, m->w.lm_head, E, V, R, m->ws, m->ws_bytes, sp)))
            return st;
        return k3gpu_argmax(m->arg, m->logits, R, V, sp);
    }
    last_rows_kernel<<<B, 256, 0, s>>>(m->last, m->nrm, T, E);
    if ((st = launch_status())) return st;
    if ((st = k3gpu_matmul_bf16_batch(m->logits, V, m->last, E, m->w.lm_head, E, V, B, m->ws, m->ws_bytes, sp)))
        return st;
    return k3gpu_argmax(m->arg, m->logits, B, V, sp);
}

// the commit of the sweep in flight: keep_dev [B] and, for a tree, path_dev [B][T]
static int model_commit_dev(K3GpuModel *m, const int *keep_dev, const int *path_dev)
{
    const K3GpuLayerCfg &l = m->cfg.layer;
    const int B = m->B, T = m->last_T, H = l.kda_heads, D = l.kda_head_dim, P = H * D, K = l.conv_k;
    cudaStream_t s = as_stream(m->stream);
    int st;
    if (path_dev) {
        for (size_t i = 0; i < m->klog.size(); i++) {
            const K3GpuKdaLog &lg = m->klog[i];
            float *arrs[5] = {lg.k, lg.v, lg.alpha, lg.beta, lg.pre};
            const long long wid[5] = {P, P, P, H, 3LL * P};
            for (int a = 0; a < 5; a++) {
                gather_path_f32_kernel<<<B, 256, 0, s>>>(arrs[a], path_dev, keep_dev, T, wid[a]);
                if ((st = launch_status())) return st;
            }
        }
        for (size_t i = 0; i < m->lat.size(); i++) {
            gather_path_bf16_kernel<<<B, 256, 0, s>>>(m->lat[i], path_dev, keep_dev, m->cached, T, m->cap, l.kv_lora);
            if ((st = launch_status())) return st;
            if (l.qk_rope) {
                gather_path_bf16_kernel<<<B, 256, 0, s>>>(m->rope[i], path_dev, keep_dev, m->cached, T, m->cap,
                                                          l.qk_rope);
                if ((st = launch_status())) return st;
            }
        }
    }
    for (size_t i = 0; i < m->kstate.size(); i++) {
        const K3GpuKdaLog &lg = m->klog[i];
        if ((st = k3gpu_kda_commit(m->kstate[i], lg.k, lg.v, lg.alpha, lg.beta, keep_dev, B, T, H, D, m->stream)))
            return st;
        if ((st = k3gpu_kda_commit_conv(m->khist[i], lg.pre, keep_dev, B, T, H, D, K, m->stream))) return st;
    }
    cached_add_kernel<<<ceil_div(B, 128), 128, 0, s>>>(m->cached, keep_dev, B, T);
    return launch_status();
}

// host checks of a commit: 0 <= keep <= T, and a tree path root first along parents
static int commit_args_ok(const K3GpuModel *m, const int *keep, const int *path)
{
    const int T = m->last_T;
    for (int b = 0; b < m->B; b++) {
        if (keep[b] < 0 || keep[b] > T) return K3GPU_EINVAL;
        if (!path) continue;
        const int *pb = path + (size_t)b * T;
        for (int j = 0; j < keep[b]; j++) {
            const int pj = pb[j];
            if (pj < 0 || pj >= T || (j == 0 && pj != 0)) return K3GPU_EINVAL;
            if (j > 0 && m->parent_host[pj] != pb[j - 1]) return K3GPU_EINVAL;
        }
    }
    return K3GPU_OK;
}

static int model_commit_host(K3GpuModel *m, const int *keep, const int *path)
{
    if (m->last_T <= 0 || (path && !m->last_tree)) return K3GPU_EINVAL;
    int st;
    if ((st = commit_args_ok(m, keep, path))) return st;
    const int B = m->B, T = m->last_T;
    cudaStream_t s = as_stream(m->stream);
    Stage sg;
    if ((st = stage_acquire(m, &sg))) return st;
    std::copy(keep, keep + B, sg.keep);
    if (path) std::copy(path, path + (size_t)B * T, sg.path);
    if ((st = cuda_status(cudaMemcpyAsync(m->keep, sg.keep, (size_t)B * 4, cudaMemcpyHostToDevice, s)))) return st;
    if (path &&
        (st = cuda_status(cudaMemcpyAsync(m->path, sg.path, (size_t)B * T * 4, cudaMemcpyHostToDevice, s))))
        return st;
    if ((st = stage_release(m, sg))) return st;
    if ((st = model_commit_dev(m, m->keep, path ? m->path : nullptr))) return st;
    for (int b = 0; b < B; b++) m->cached_host[b] += keep[b];
    m->last_T = 0;
    return K3GPU_OK;
}

}  // namespace k3

extern "C" size_t k3gpu_model_arena_bytes(const K3GpuModelCfg *c, int B, int max_T, int kv_cap)
{
    if (!k3::model_cfg_ok(c) || B <= 0 || B > 4096 || max_T <= 0 || max_T > 64 || kv_cap < max_T) return 0;
    return k3::model_layout(c, B, max_T, kv_cap, nullptr, nullptr);
}

extern "C" K3GpuModel *k3gpu_model_create(const K3GpuModelCfg *c, const K3GpuModelW *w, int B, int max_T,
                                          int kv_cap, void *arena, size_t arena_bytes, void *stream)
{
    using namespace k3;
    const size_t need = k3gpu_model_arena_bytes(c, B, max_T, kv_cap);
    if (!need || !w || !arena || arena_bytes < need || !aligned(arena, 256)) return nullptr;
    if (!w->embed || !w->lm_head || !w->norm || !w->kda || !w->mla) return nullptr;
    for (int i = 0; i < c->n_layers; i++) {
        const bool mla_l = c->is_mla[i] != 0;
        const void *core = mla_l ? (const void *)w->mla[i].mla.q_a : (const void *)w->kda[i].kda.q;
        const bool moe_ok = mla_l ? (w->mla[i].moe || w->mla[i].bank) : (w->kda[i].moe || w->kda[i].bank);
        if (!core || !moe_ok) return nullptr;
    }
    K3GpuModel *m = new (std::nothrow) K3GpuModel();
    if (!m) return nullptr;
    m->cfg = *c;
    m->is_mla.assign(c->is_mla, c->is_mla + c->n_layers);
    m->cfg.is_mla = m->is_mla.data();
    m->kda.assign(w->kda, w->kda + c->n_layers);
    m->mla.assign(w->mla, w->mla + c->n_layers);
    m->w = *w;
    m->w.kda = m->kda.data();
    m->w.mla = m->mla.data();
    m->B = B;
    m->maxT = max_T;
    m->cap = kv_cap;
    m->maxb = c->layer.max_blocks;
    m->stream = stream;
    m->cached_host.assign(B, 0);
    m->parent_host.assign(max_T, -1);
    m->last_T = m->last_tree = m->pre_committed = 0;
    m->stage_bytes = stage_slot_bytes(B, max_T) * K3GpuModel::NSTAGE;
    bool ok = cudaMallocHost((void **)&m->stage, m->stage_bytes) == cudaSuccess;
    for (int i = 0; ok && i < K3GpuModel::NSTAGE; i++)
        ok = cudaEventCreateWithFlags(&m->ev[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        delete m;
        return nullptr;
    }
    model_layout(c, B, max_T, kv_cap, m, static_cast<char *>(arena));
    if (k3gpu_model_reset(m) != K3GPU_OK) {
        delete m;
        return nullptr;
    }
    return m;
}

extern "C" void k3gpu_model_free(K3GpuModel *m) { delete m; }

extern "C" int k3gpu_model_set_stream(K3GpuModel *m, void *stream)
{
    if (!m) return K3GPU_EINVAL;
    for (cudaEvent_t e : m->ev) {   // the staging slots are released on the old stream
        int st = k3::cuda_status(cudaEventSynchronize(e));
        if (st) return st;
    }
    m->stream = stream;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_reset(K3GpuModel *m)
{
    using namespace k3;
    if (!m) return K3GPU_EINVAL;
    cudaStream_t s = as_stream(m->stream);
    const K3GpuLayerCfg &l = m->cfg.layer;
    const int H = l.kda_heads, D = l.kda_head_dim, P = H * D, K = l.conv_k;
    int st;
    for (size_t i = 0; i < m->kstate.size(); i++) {
        if ((st = cuda_status(cudaMemsetAsync(m->kstate[i], 0, (size_t)m->B * H * D * D * 4, s)))) return st;
        if ((st = cuda_status(cudaMemsetAsync(m->khist[i], 0, (size_t)m->B * 3 * P * (K - 1) * 4, s)))) return st;
    }
    if ((st = cuda_status(cudaMemsetAsync(m->cached, 0, (size_t)m->B * 4, s)))) return st;
    std::fill(m->cached_host.begin(), m->cached_host.end(), 0);
    m->last_T = 0;
    m->pre_committed = 0;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_verify(K3GpuModel *m, const int *ids, int T, const int *parent, int *arg,
                                  const float **logits)
{
    using namespace k3;
    if (!m || !ids || T <= 0 || T > m->maxT) return K3GPU_EINVAL;
    int st = model_sweep(m, ids, T, parent, 0);
    if (st) return st;
    m->last_T = T;
    m->last_tree = parent != nullptr;
    m->pre_committed = 0;
    if (logits) *logits = m->logits;
    if (!arg) return K3GPU_OK;
    return cuda_status(cudaMemcpyAsync(arg, m->arg, (size_t)m->B * T * 4, cudaMemcpyDeviceToDevice,
                                       as_stream(m->stream)));
}

extern "C" int k3gpu_model_verify_greedy(K3GpuModel *m, const int *ids, int T, const int *parent, int *arg)
{
    using namespace k3;
    if (!m || !ids || !arg || T <= 0 || T > m->maxT) return K3GPU_EINVAL;
    int st = model_sweep(m, ids, T, parent, 2);
    if (st) return st;
    m->last_T = T;
    m->last_tree = parent != nullptr;
    m->pre_committed = 0;
    return cuda_status(cudaMemcpyAsync(arg, m->arg, (size_t)m->B * T * 4, cudaMemcpyDeviceToDevice,
                                       as_stream(m->stream)));
}

extern "C" int k3gpu_model_commit(K3GpuModel *m, const int *keep, const int *path)
{
    if (!m || !keep) return K3GPU_EINVAL;
    return k3::model_commit_host(m, keep, path);
}

extern "C" int k3gpu_model_commit_device(K3GpuModel *m, const int *keep_dev, const int *keep_host)
{
    using namespace k3;
    if (!m || !keep_dev || !keep_host || m->last_T <= 0 || m->last_tree) return K3GPU_EINVAL;
    int st;
    if ((st = commit_args_ok(m, keep_host, nullptr))) return st;
    if ((st = model_commit_dev(m, keep_dev, nullptr))) return st;
    for (int b = 0; b < m->B; b++) m->cached_host[b] += keep_host[b];
    m->last_T = 0;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_prefill(K3GpuModel *m, const int *ids, int n, int *next)
{
    using namespace k3;
    if (!m || !ids || !next || n <= 0) return K3GPU_EINVAL;
    const int B = m->B;
    cudaStream_t s = as_stream(m->stream);
    int st;
    std::vector<int> keep(B);
    for (int i = 0; i < n;) {
        const int q = std::min(m->maxT, n - i);
        // ids is [B][n]; a pass takes columns i..i+q of every sequence
        if ((st = cuda_status(cudaMemcpy2DAsync(m->ids, (size_t)q * 4, ids + i, (size_t)n * 4, (size_t)q * 4, B,
                                                cudaMemcpyDeviceToDevice, s))))
            return st;
        if ((st = model_sweep(m, m->ids, q, nullptr, 1))) return st;
        m->last_T = q;
        m->last_tree = 0;
        std::fill(keep.begin(), keep.end(), q);
        if ((st = model_commit_host(m, keep.data(), nullptr))) return st;
        i += q;
    }
    return cuda_status(cudaMemcpyAsync(next, m->arg, (size_t)B * 4, cudaMemcpyDeviceToDevice, s));
}

extern "C" int k3gpu_model_set_cached(K3GpuModel *m, const int *cached)
{
    using namespace k3;
    if (!m || !cached) return K3GPU_EINVAL;
    for (int b = 0; b < m->B; b++)
        if (cached[b] < 0 || cached[b] > m->cap) return K3GPU_EINVAL;
    Stage sg;
    int st;
    if ((st = stage_acquire(m, &sg))) return st;
    std::copy(cached, cached + m->B, sg.keep);
    if ((st = cuda_status(cudaMemcpyAsync(m->cached, sg.keep, (size_t)m->B * 4, cudaMemcpyHostToDevice,
                                          as_stream(m->stream)))))
        return st;
    if ((st = stage_release(m, sg))) return st;
    std::copy(cached, cached + m->B, m->cached_host.begin());
    m->last_T = 0;
    m->pre_committed = 0;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_cached(const K3GpuModel *m, int *cached)
{
    if (!m || !cached) return K3GPU_EINVAL;
    for (int b = 0; b < m->B; b++) cached[b] = m->cached_host[b];
    return K3GPU_OK;
}

extern "C" int k3gpu_model_kda_state(const K3GpuModel *m, int layer, float **state, float **conv_hist)
{
    if (!m || layer < 0 || layer >= m->cfg.n_layers || m->is_mla[layer]) return K3GPU_EINVAL;
    if (state) *state = m->kstate[m->slot[layer]];
    if (conv_hist) *conv_hist = m->khist[m->slot[layer]];
    return K3GPU_OK;
}

extern "C" int k3gpu_model_last_routing(const K3GpuModel *m, const int **idx)
{
    if (!m || !idx) return K3GPU_EINVAL;
    *idx = m->moe_idx;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_mla_cache(const K3GpuModel *m, int layer, uint16_t **lat, uint16_t **rope)
{
    if (!m || layer < 0 || layer >= m->cfg.n_layers || !m->is_mla[layer]) return K3GPU_EINVAL;
    if (lat) *lat = m->lat[m->slot[layer]];
    if (rope) *rope = m->rope[m->slot[layer]];
    return K3GPU_OK;
}

// ---- the decode loop's callbacks over one sequence (B == 1) ----
// verify: ids host [n]; a prompt longer than max_T is read in passes, all but the last
// committed at once (a read-in keeps every position), the last left for the commit.
extern "C" int k3gpu_model_loop_verify(void *ctx, const int *ids, const int *parent, int n, int base, int *arg)
{
    using namespace k3;
    K3GpuModel *m = static_cast<K3GpuModel *>(ctx);
    if (!m || m->B != 1 || !ids || !arg || n <= 0) return K3GPU_EINVAL;
    if (base != m->cached_host[0] || (parent && n > m->maxT)) return K3GPU_EINVAL;
    cudaStream_t s = as_stream(m->stream);
    int st;
    int done = 0;
    while (n - done > 0) {
        const int q = std::min(m->maxT, n - done);
        const bool last = done + q == n;
        Stage sg;
        if ((st = stage_acquire(m, &sg))) return st;
        std::copy(ids + done, ids + done + q, sg.ids);
        if ((st = cuda_status(cudaMemcpyAsync(m->ids, sg.ids, (size_t)q * 4, cudaMemcpyHostToDevice, s)))) return st;
        if ((st = stage_release(m, sg))) return st;
        if ((st = model_sweep(m, m->ids, q, last ? parent : nullptr, last ? 0 : 1))) return st;
        m->last_T = q;
        m->last_tree = last && parent != nullptr;
        if (last) break;
        const int keep = q;   // a read-in pass keeps every position
        if ((st = model_commit_host(m, &keep, nullptr))) return st;
        done += q;
    }
    m->pre_committed = done;
    const int q = n - done;
    Stage sg;
    if ((st = stage_acquire(m, &sg))) return st;
    if ((st = cuda_status(cudaMemcpyAsync(sg.arg, m->arg, (size_t)q * 4, cudaMemcpyDeviceToHost, s)))) return st;
    if ((st = stage_release(m, sg))) return st;
    if ((st = cuda_status(cudaStreamSynchronize(s)))) return st;
    for (int i = 0; i < done; i++) arg[i] = -1;   // positions of passes already committed
    std::copy(sg.arg, sg.arg + q, arg + done);
    return K3GPU_OK;
}

extern "C" int k3gpu_model_loop_commit(void *ctx, int base, const int *path, int keep)
{
    K3GpuModel *m = static_cast<K3GpuModel *>(ctx);
    if (!m || m->B != 1 || m->last_T <= 0) return K3GPU_EINVAL;
    const int kq = keep - m->pre_committed;
    if (kq < 0 || kq > m->last_T || base + m->pre_committed != m->cached_host[0]) return K3GPU_EINVAL;
    m->pre_committed = 0;
    return k3::model_commit_host(m, &kq, path);
}

// ---- expert parallel ----
extern "C" size_t k3gpu_model_ep_workspace(const K3GpuModel *m, const K3GpuEpGroup *g)
{
    if (!m || !g) return 0;
    const K3GpuLayerCfg &l = m->cfg.layer;
    const size_t moe = k3gpu_moe_layer_ep_workspace(g, m->B * m->maxT, l.n_shared, l.moe_inter, l.n_routed);
    if (!moe) return 0;
    return ((moe + 255) & ~(size_t)255) + 256;   // + the per-owner flags
}

extern "C" int k3gpu_model_set_ep(K3GpuModel *m, const K3GpuEpGroup *g, const K3GpuExpertBank *const *shared,
                                  void *workspace, size_t ws_bytes)
{
    using namespace k3;
    if (!m || !g || !workspace || (m->cfg.layer.n_shared > 0 && !shared)) return K3GPU_EINVAL;
    const K3GpuLayerCfg &l = m->cfg.layer;
    if (g->world < 1 || g->world > K3GPU_EP_MAX_WORLD || g->cap < m->B * m->maxT || g->L != l.hidden ||
        g->K != l.topk || g->n_local * g->world != l.n_routed)
        return K3GPU_EINVAL;
    for (int i = 0; i < m->cfg.n_layers; i++) {
        const K3GpuExpertBank *b = m->is_mla[i] ? m->mla[i].bank : m->kda[i].bank;
        const bool latent = m->is_mla[i] ? m->mla[i].moe != nullptr : m->kda[i].moe != nullptr;
        if (latent || !b || b->n_experts != g->n_local) return K3GPU_EINVAL;   // the single-layer MoE form only
        if (l.n_shared > 0 && (!shared[i] || shared[i]->n_experts != l.n_shared)) return K3GPU_EINVAL;
    }
    const size_t need = k3gpu_model_ep_workspace(m, g);
    if (!need) return K3GPU_EINVAL;
    if (ws_bytes < need || !aligned(workspace, 256)) return ws_bytes < need ? K3GPU_ECAPACITY : K3GPU_EINVAL;
    m->ep_group = *g;
    m->ep_shared.assign(m->cfg.n_layers, nullptr);
    if (l.n_shared > 0) m->ep_shared.assign(shared, shared + m->cfg.n_layers);
    m->ep_ok = static_cast<int *>(workspace);
    m->ep_ws = static_cast<char *>(workspace) + 256;
    m->ep_ws_bytes = need - 256;
    m->ep_on = true;
    return K3GPU_OK;
}

extern "C" int k3gpu_model_ep_status(const K3GpuModel *m, int *ok_host)
{
    if (!m || !ok_host || !m->ep_on) return K3GPU_EINVAL;
    const int st = k3::cuda_status(cudaMemcpyAsync(ok_host, m->ep_ok, (size_t)m->ep_group.world * 4,
                                                   cudaMemcpyDeviceToHost, k3::as_stream(m->stream)));
    if (st) return st;
    return k3::cuda_status(cudaStreamSynchronize(k3::as_stream(m->stream)));
}
