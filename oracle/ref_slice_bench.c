/* ref_slice_bench.c -- the timed CPU baseline of the config-4 slice: the REFERENCE engine's
 * own attention layers at K3 dimensions on random weights.
 *
 * TEST / BENCHMARK INFRASTRUCTURE ONLY (bench.py --impl reference and its cpu_baseline
 * leg). It links the reference's k3_ops.c, compiled by oracle/Makefile into
 * _ref/libk3ref.so, and calls its public functions as a verify sweep of T positions does
 * (src/cli/k3_run.c:853-1138 through k3_decoder_layer_inc_log, src/core/k3_ops.c:2485-2602):
 *   - k3_kda_layer_log, the tentative KDA layer with its rollback log (:2231-2385);
 *   - k3_mla_cached over a cache of `ctx` earlier positions in the latent layout with the
 *     absorbed attention (the engine's --kv-latent --mla-absorb, :1115-1615);
 *   - k3_matmul_bf16_batch_ld over a sample of lm_head rows (:953).
 * The routed experts of each layer are timed separately through ref_moe_bench.c. Weights
 * are bf16 N(0, 0.02) (tagged K3_WBF16 as the released checkpoint's are), the norms 1, the
 * KDA decay parameters of the reference's tiny-model recipe, the state N(0, 0.1) and the
 * cached latents N(0, 1); the arithmetic is the reference's, unchanged and serial (this
 * image has no OpenMP runtime).
 */
#include "k3.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static uint64_t g_rng = 0x9E3779B97F4A7C15ull;

static double urand(void)
{
    g_rng ^= g_rng << 13;
    g_rng ^= g_rng >> 7;
    g_rng ^= g_rng << 17;
    return (double)(g_rng >> 11) * (1.0 / 9007199254740992.0);
}

static float nrand(void)   /* Box-Muller */
{
    double u = urand(), v = urand();
    if (u < 1e-300) u = 1e-300;
    return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

static uint16_t *bf16_mat(size_t n, float std)
{
    uint16_t *w = (uint16_t *)malloc(n * sizeof(uint16_t));
    if (!w) return NULL;
    for (size_t i = 0; i < n; i++) {
        const float f = nrand() * std;
        uint32_t u;
        memcpy(&u, &f, 4);
        w[i] = (uint16_t)(u >> 16);
    }
    return w;
}

static float *f32_vec(size_t n, float std, float mean)
{
    float *w = (float *)malloc(n * sizeof(float));
    if (!w) return NULL;
    for (size_t i = 0; i < n; i++) w[i] = mean + (std > 0 ? nrand() * std : 0.0f);
    return w;
}

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static int g_full_attn[2] = {4, 8};

static void c4_cfg(K3Cfg *c)
{
    memset(c, 0, sizeof(*c));
    c->hidden = 7168; c->n_layers = 8; c->vocab = 163840; c->rms_eps = 1e-5f;
    c->kda_heads = 32; c->kda_head_dim = 128; c->conv_k = 4; c->gate_lb = -5.0f;
    c->n_heads = 64; c->q_lora = 1536; c->kv_lora = 512; c->qk_nope = 128; c->qk_rope = 64;
    c->v_head = 128; c->mla_out_gate = 1;
    c->n_experts = 384; c->topk = 8; c->n_shared = 1; c->latent = 7168; c->moe_inter = 2048;
    c->routed_scale = 1.0f; c->moe_renorm = 1; c->latent_norm = 0;
    c->first_dense = 0; c->dense_inter = 2048; c->attn_res_block = 2;
    c->situ_b1 = 4.0f; c->situ_b2 = 25.0f;
    c->n_full_attn = 2; c->full_attn = g_full_attn;
}

/* Seconds of one KDA layer (tentative, logged) over T positions; < 0 on OOM. */
double ref_c4_kda(int T, unsigned seed)
{
    g_rng ^= (uint64_t)seed * 0x2545F4914F6CDD1Dull + 1;
    K3Cfg c;
    c4_cfg(&c);
    const size_t E = c.hidden, H = c.kda_heads, D = c.kda_head_dim, P = H * D, K = c.conv_k;
    K3KdaW w;
    memset(&w, 0, sizeof(w));
    w.q = bf16_mat(P * E, 0.02f); w.k = bf16_mat(P * E, 0.02f); w.v = bf16_mat(P * E, 0.02f);
    w.g = bf16_mat(P * E, 0.02f); w.o = bf16_mat(E * P, 0.02f);
    w.f_a = bf16_mat(D * E, 0.02f); w.f_b = bf16_mat(P * D, 0.02f); w.b = bf16_mat(H * E, 0.02f);
    float *qc = f32_vec(P * K, 0.4f, 0), *kc = f32_vec(P * K, 0.4f, 0), *vc = f32_vec(P * K, 0.4f, 0);
    float *A = f32_vec(H, 0, 0), *dt = f32_vec(P, 0.5f, 0), *on = f32_vec(D, 0, 1.0f);
    for (size_t h = 0; h < H; h++) A[h] = (float)(-0.4 + 1.6 * (double)h / (double)(H - 1));
    w.q_conv = qc; w.k_conv = kc; w.v_conv = vc; w.A_log = A; w.dt_bias = dt; w.o_norm = on;
    w.wdt = K3_WBF16;
    const size_t sf = k3_kda_state_floats(&c);
    float *state = f32_vec(sf, 0.1f, 0);
    float *scratch = (float *)malloc(k3_kda_scratch(&c, T) * sizeof(float));
    K3KdaLog lg;
    lg.rows = (float *)malloc((size_t)T * k3_kda_log_row(&c) * sizeof(float));
    lg.work = (float *)malloc(sf * sizeof(float));
    lg.cap = T;
    lg.row0 = 0;
    float *x = f32_vec((size_t)T * E, 1.0f, 0), *out = (float *)malloc((size_t)T * E * sizeof(float));
    double dtm = -1.0;
    if (w.q && w.k && w.v && w.g && w.o && w.f_a && w.f_b && w.b && state && scratch && lg.rows && lg.work && x &&
        out) {
        const double t0 = now_s();
        k3_kda_layer_log(out, x, &w, &c, T, state, scratch, &lg);
        dtm = now_s() - t0;
    }
    free((void *)w.q); free((void *)w.k); free((void *)w.v); free((void *)w.g); free((void *)w.o);
    free((void *)w.f_a); free((void *)w.f_b); free((void *)w.b);
    free(qc); free(kc); free(vc); free(A); free(dt); free(on);
    free(state); free(scratch); free(lg.rows); free(lg.work); free(x); free(out);
    return dtm;
}

/* Seconds of one MLA layer (latent cache of ctx positions, absorbed attention) over T
 * positions; < 0 on OOM. */
double ref_c4_mla(int T, int ctx, unsigned seed)
{
    g_rng ^= (uint64_t)seed * 0x2545F4914F6CDD1Dull + 3;
    K3Cfg c;
    c4_cfg(&c);
    const size_t E = c.hidden, H = c.n_heads, ql = c.q_lora, kvl = c.kv_lora;
    const size_t nope = c.qk_nope, rope = c.qk_rope, vh = c.v_head;
    K3MlaW w;
    memset(&w, 0, sizeof(w));
    w.q_a = bf16_mat(ql * E, 0.02f); w.q_b = bf16_mat(H * (nope + rope) * ql, 0.02f);
    w.kv_a = bf16_mat((kvl + rope) * E, 0.02f); w.kv_b = bf16_mat(H * (nope + vh) * kvl, 0.02f);
    w.o = bf16_mat(E * H * vh, 0.02f); w.g = bf16_mat(H * vh * E, 0.02f);
    float *qn = f32_vec(ql, 0, 1.0f), *kn = f32_vec(kvl, 0, 1.0f);
    w.q_a_norm = qn; w.kv_a_norm = kn;
    w.wdt = K3_WBF16;
    const int cap = ctx + T;
    float *kvc = f32_vec((size_t)cap * kvl, 1.0f, 0), *ropec = f32_vec((size_t)cap * rope, 1.0f, 0);
    k3_mla_absorb = 1;
    float *scratch = (float *)malloc(k3_mla_scratch_cached(&c, T, cap, 1, 1) * sizeof(float));
    float *x = f32_vec((size_t)T * E, 1.0f, 0), *out = (float *)malloc((size_t)T * E * sizeof(float));
    double dtm = -1.0;
    if (w.q_a && w.q_b && w.kv_a && w.kv_b && w.o && w.g && kvc && ropec && scratch && x && out) {
        const double t0 = now_s();
        k3_mla_cached(out, x, &w, &c, T, scratch, kvc, ropec, ctx, cap, 1);
        dtm = now_s() - t0;
    }
    free((void *)w.q_a); free((void *)w.q_b); free((void *)w.kv_a); free((void *)w.kv_b);
    free((void *)w.o); free((void *)w.g); free(qn); free(kn);
    free(kvc); free(ropec); free(scratch); free(x); free(out);
    return dtm;
}

/* Seconds of the bf16 lm_head over T positions for `rows` of its 163840 rows (the cost is
 * linear in rows); < 0 on OOM. */
double ref_c4_lm_rows(int T, int rows, unsigned seed)
{
    g_rng ^= (uint64_t)seed * 0x2545F4914F6CDD1Dull + 5;
    const int E = 7168;
    uint16_t *W = bf16_mat((size_t)rows * E, 0.02f);
    float *X = f32_vec((size_t)T * E, 1.0f, 0), *Y = (float *)malloc((size_t)T * rows * sizeof(float));
    double dtm = -1.0;
    if (W && X && Y) {
        const double t0 = now_s();
        k3_matmul_bf16_batch_ld(Y, rows, X, E, W, E, rows, T);
        dtm = now_s() - t0;
    }
    free(W); free(X); free(Y);
    return dtm;
}
