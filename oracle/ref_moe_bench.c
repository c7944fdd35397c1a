/* ref_moe_bench.c -- the timed CPU baseline: the REFERENCE engine's own kernels driven
 * over host threads for one verify batch of a MoE layer.
 *
 * TEST / BENCHMARK INFRASTRUCTURE ONLY (bench.py --impl reference and its cpu_baseline
 * leg). It links the reference's k3_ops.c, compiled by oracle/Makefile into
 * _ref/libk3ref.so, and calls its public functions exactly as k3_moe_prefill's routed
 * half does (src/core/k3_ops.c:2058-2132 of the reference): k3_router per token, then for
 * every (token, slot) k3_matmul_mxfp4 on w1 and w3, the activation, k3_matmul_mxfp4 on w2
 * (:2099-2110), and the per-token sum in the original top-k order (:2119-2128). The only
 * addition is the thread pool: the reference would use OpenMP inside each call, which this
 * image cannot link (no libgomp), so whole (token, slot) items run on separate pthreads
 * instead -- every item is the reference's own arithmetic, unchanged.
 *
 * act 0 runs the reference's k3_situ_glu; act 1 (SwiGLU, which the reference does not
 * implement) is computed here as silu(gate)*up.
 */
#include "k3.h"

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    /* shared problem */
    const float *x, *gate_W, *bias;
    const uint8_t *bank;
    int64_t stride, p1, s1, p2, s2, p3, s3;
    int T, L, I, n_routed, n_shared, topk, act;
    float b1, b2;
    int *idx;
    float *wt;
    float *contrib;   /* [T][topk + n_shared][L] */
    /* work distribution */
    int phase;        /* 0 = route, 1 = experts */
    int next;
    pthread_mutex_t mu;
} RefJob;

static int take(RefJob *j)
{
    pthread_mutex_lock(&j->mu);
    const int i = j->next++;
    pthread_mutex_unlock(&j->mu);
    return i;
}

static void run_item(RefJob *j, int item, float *gu, float *h)
{
    const int slots = j->topk + j->n_shared;
    const int t = item / slots, s = item % slots;
    const float *xt = j->x + (size_t)t * j->L;
    const int e = s < j->topk ? j->idx[(size_t)t * j->topk + s] : j->n_routed + (s - j->topk);
    float *out = j->contrib + (size_t)item * j->L;
    if (e < 0) { memset(out, 0, (size_t)j->L * sizeof(float)); return; }
    const uint8_t *run = j->bank + (size_t)e * j->stride;
    k3_matmul_mxfp4(gu, xt, run + j->p1, run + j->s1, j->L, j->I, K3_MXFP4_GROUP);
    k3_matmul_mxfp4(gu + j->I, xt, run + j->p3, run + j->s3, j->L, j->I, K3_MXFP4_GROUP);
    if (j->act == 0) {
        k3_situ_glu(h, gu, j->I, j->b1, j->b2);
    } else {
        for (int i = 0; i < j->I; i++) {
            const float g = gu[i];
            h[i] = (g * (1.0f / (1.0f + expf(-g)))) * gu[j->I + i];
        }
    }
    k3_matmul_mxfp4(out, h, run + j->p2, run + j->s2, j->I, j->L, K3_MXFP4_GROUP);
}

static void *worker(void *arg)
{
    RefJob *j = (RefJob *)arg;
    float *gu = (float *)malloc((size_t)2 * j->I * sizeof(float));
    float *h = (float *)malloc((size_t)j->I * sizeof(float));
    if (j->phase == 0) {
        for (int t; (t = take(j)) < j->T;)
            k3_router(j->idx + (size_t)t * j->topk, j->wt + (size_t)t * j->topk,
                      j->x + (size_t)t * j->L, j->gate_W, j->bias, j->L, j->n_routed,
                      j->topk, 1, 1.0f);
    } else {
        const int items = j->T * (j->topk + j->n_shared);
        for (int it; (it = take(j)) < items;) run_item(j, it, gu, h);
    }
    free(gu);
    free(h);
    return NULL;
}

static void run_phase(RefJob *j, int phase, int nthreads)
{
    pthread_t th[256];
    if (nthreads > 256) nthreads = 256;
    if (nthreads < 1) nthreads = 1;
    j->phase = phase;
    j->next = 0;
    for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, worker, j);
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
}

/* One MoE layer over T tokens (the single-layer form without latent projections):
 * out[t] = sum_j wt[t][j] * expert_idx[t][j](x_t) in top-k order, + shared experts.
 * idx/wt receive the routing decisions. Returns 0, or -1 on allocation failure. */
__attribute__((visibility("default")))
int ref_moe_layer(float *out, int *idx, float *wt, const float *x, const float *gate_W,
                  const float *bias, const uint8_t *bank, const int64_t *lay, int T, int L,
                  int I, int n_routed, int n_shared, int topk, int act, float b1, float b2,
                  int nthreads)
{
    RefJob j;
    memset(&j, 0, sizeof(j));
    j.x = x; j.gate_W = gate_W; j.bias = bias; j.bank = bank;
    j.p1 = lay[0]; j.s1 = lay[1]; j.p2 = lay[2]; j.s2 = lay[3]; j.p3 = lay[4]; j.s3 = lay[5];
    j.stride = lay[6];
    j.T = T; j.L = L; j.I = I; j.n_routed = n_routed; j.n_shared = n_shared; j.topk = topk;
    j.act = act; j.b1 = b1; j.b2 = b2; j.idx = idx; j.wt = wt;
    const int slots = topk + n_shared;
    j.contrib = (float *)malloc((size_t)T * slots * L * sizeof(float));
    if (!j.contrib) return -1;
    pthread_mutex_init(&j.mu, NULL);
    run_phase(&j, 0, nthreads);
    run_phase(&j, 1, nthreads);
    pthread_mutex_destroy(&j.mu);
    for (int t = 0; t < T; t++) {
        float *ot = out + (size_t)t * L;
        for (int i = 0; i < L; i++) ot[i] = 0.0f;
        for (int s = 0; s < topk; s++) {
            if (idx[(size_t)t * topk + s] < 0) continue;
            const float w = wt[(size_t)t * topk + s];
            const float *cb = j.contrib + ((size_t)t * slots + s) * L;
            for (int i = 0; i < L; i++) ot[i] += w * cb[i];
        }
        for (int s = topk; s < slots; s++) {
            const float *cb = j.contrib + ((size_t)t * slots + s) * L;
            for (int i = 0; i < L; i++) ot[i] += cb[i];
        }
    }
    free(j.contrib);
    return 0;
}
