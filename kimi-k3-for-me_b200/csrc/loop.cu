// loop.cu -- host C++: the engine's speculative decode loop (src/cli/k3_run.c:2812-3047)
// as a step driver over two callbacks, so the same bookkeeping runs the device forward.
//
// The loop keeps the conversation's ids (seq[0..T)), the positions the model has consumed
// (cached; the last id stays pending, cached = T - 1 between steps) and the generated ids.
// A step
//   * on the first call reads everything not yet consumed (seq[cached..T)) -- the prompt,
//     or on a resume the carried pending id plus the new prompt -- and emits the model's
//     next id (k3_run.c:2820-2854);
//   * later, drafts up to spec_n ids when the context and the cache have room for a full
//     draft (:2859, the same condition as the engine), verifies the pending id plus the
//     nd drafts in one pass, accepts the longest prefix the model agrees with and emits it
//     plus the model's own next id (:2909-2927); with nothing drafted, one serial position
//     (:2968-2975);
//   * keeps as many emitted ids as emit_keep allows (--gen, the context limit, the first
//     stop id; :1300-1317), commits exactly the positions behind them (:2941-2943), and
//     appends them (:3029-3043).
// Every verify call is followed by exactly one commit call before the next verify.
// With the tree policy the draft is a tree (k3_suffix_drafter_tree): verify gets the
// nodes' parents, acceptance follows k3gpu_accept_tree_greedy (a child is accepted when
// its parent is and its id is the parent's next id; the lowest-index such child wins),
// and commit gets the accepted path's nodes.
// With the draft-model policy (the engine's --draft, k3_run.c:2862-2905, 2956-2965) a
// second model proposes: it trails the target by dlag positions, feeds the ids it has not
// seen plus the pending one and then chains its own next ids, tentatively, and after the
// target has decided commits exactly the positions behind the kept ids it fed.
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <new>

#include "k3gpu.h"

struct K3SpecLoop {
    K3SpecLoopCfg cfg;
    int *stop;                  // a copy of cfg.stop_ids
    K3SpecVerifyFn verify;
    K3SpecCommitFn commit;
    void *ctx;
    int *seq;                   // [tmax]
    int T, cached, nout, started, done;
    int *arg;                   // [max(prefill, spec_n + 1, tree_nodes)]
    int arg_cap;
    int *tok, *parent;          // the tree draft [tree_nodes]
    K3SuffixDrafter *sam;       // P2 / P3 history
    K3SpecVerifyFn dverify;     // the draft model (K3_DRAFT_MODEL)
    K3SpecCommitFn dcommit;
    void *dctx;
    int dcached;                // positions the draft model has consumed
    K3SpecCheckpointFn ckpt;    // called at chunk boundaries of the prompt read-in
    void *ckctx;
    int ck_written;
    std::atomic<int> pause_req;
    K3SpecLoopStats st;
};

namespace {

// how many of a step's emitted ids the output keeps (src/cli/k3_run.c:1300-1317)
int emit_keep(const K3SpecLoop *L, const int *emit, int emitn)
{
    int k = 0;
    while (k < emitn && L->nout + k < L->cfg.gen && L->T + k < L->cfg.tmax) {
        const int id = emit[k++];
        for (int s = 0; s < L->cfg.n_stop; s++)
            if (id == L->stop[s]) return k;
    }
    return k;
}

int draft(K3SpecLoop *L, int *d)
{
    const K3SpecLoopCfg &c = L->cfg;
    switch (c.policy) {
        case K3_DRAFT_NGRAM: return k3_spec_draft_ngram(L->seq, L->T, c.spec_n, 4, 3, d);
        case K3_DRAFT_EAGER: return k3_spec_draft_eager(L->seq, L->T, c.spec_n, d);
        case K3_DRAFT_SUFFIX: return k3_suffix_drafter_draft(L->sam, c.spec_n, c.min_len, d, nullptr, nullptr);
        case K3_DRAFT_P3:
            return k3_suffix_drafter_draft_p3(L->sam, c.p3_q, c.p3_delta, c.p3_cost, c.p3_replay, c.spec_n, d);
        default: return 0;
    }
}

// greedy acceptance over a draft tree (k3gpu_accept_tree_greedy): path[0] = 0, the root;
// at most cap nodes (the depth limit the tree was drafted with, plus the root)
int tree_accept(const int *tok, const int *parent, int n, const int *arg, int *path, int cap)
{
    int len = 1, node = 0;
    path[0] = 0;
    while (len < cap) {
        int next = -1;
        for (int c = node + 1; c < n; c++)
            if (parent[c] == node && tok[c] == arg[node]) {
                next = c;
                break;
            }
        if (next < 0) return len;
        path[len++] = next;
        node = next;
    }
    return len;
}

// append the kept ids to the history, the output and the drafter
int append(K3SpecLoop *L, const int *emit, int keep, int *out)
{
    for (int i = 0; i < keep; i++) {
        L->seq[L->T++] = emit[i];
        if (out) out[i] = emit[i];
        L->nout++;
    }
    if (L->sam && keep > 0 && k3_suffix_drafter_push(L->sam, emit, keep) != K3GPU_OK) return K3GPU_EINVAL;
    for (int s = 0; keep > 0 && s < L->cfg.n_stop; s++)
        if (emit[keep - 1] == L->stop[s]) L->done = K3_SPEC_LOOP_STOP_ID;
    if (!L->done && L->nout >= L->cfg.gen) L->done = K3_SPEC_LOOP_GEN;
    if (!L->done && L->T >= L->cfg.tmax) L->done = K3_SPEC_LOOP_CONTEXT;
    return K3GPU_OK;
}

// read seq[from..to) into a model in passes of at most `chunk` positions (0: one pass),
// each a verify then a commit of the whole pass (k3_run.c:1189-1240); the last pass's next
// id goes to *next. With ck, a checkpoint follows every pass that leaves positions to go,
// and the read-in pauses (returns 1) once pause_after checkpoints are written or a pause
// was requested. Returns 0 when done, 1 when paused, a negative status on failure.
int read_in(K3SpecLoop *L, K3SpecVerifyFn verify, K3SpecCommitFn commit, void *ctx, int from, int to, int *done_to,
            int *next, bool ck)
{
    const int chunk = L->cfg.prefill_chunk > 0 ? L->cfg.prefill_chunk : to - from;
    int i = from;
    while (i < to) {
        const int q = to - i < chunk ? to - i : chunk;
        if (verify(ctx, L->seq + i, nullptr, q, i, L->arg) != 0) return K3GPU_ECALLBACK;
        if (commit(ctx, i, nullptr, q) != 0) return K3GPU_ECALLBACK;
        i += q;
        *done_to = i;
        if (next) *next = L->arg[q - 1];
        if (ck && L->ckpt && i < to) {
            if (L->ckpt(L->ckctx, i) != 0) return K3GPU_ECALLBACK;
            L->ck_written++;
            if ((L->cfg.pause_after && L->ck_written >= L->cfg.pause_after) || L->pause_req.load()) return 1;
        }
    }
    return 0;
}

}  // namespace

extern "C" K3SpecLoop *k3_spec_loop_create(const K3SpecLoopCfg *cfg, const int *ids, int n_ids, int cached,
                                           K3SpecVerifyFn verify, K3SpecCommitFn commit, void *ctx)
{
    if (!cfg || !ids || !verify || !commit || n_ids <= 0 || cached < 0 || cached >= n_ids) return nullptr;
    if (cfg->tmax < n_ids || cfg->gen < 0 || cfg->spec_n < 0 || cfg->spec_n > 8 || cfg->n_stop < 0 ||
        (cfg->n_stop > 0 && !cfg->stop_ids) || cfg->kv_cap < n_ids)
        return nullptr;
    if (cfg->policy < K3_DRAFT_NONE || cfg->policy > K3_DRAFT_MODEL) return nullptr;
    if (cfg->policy == K3_DRAFT_TREE && (cfg->tree_nodes < 1 || cfg->tree_nodes > 64 || cfg->tree_branch < 1))
        return nullptr;
    if (cfg->policy == K3_DRAFT_P3 && !cfg->p3_q) return nullptr;
    if (cfg->prefill_chunk < 0 || cfg->pause_after < 0) return nullptr;
    K3SpecLoop *L = new (std::nothrow) K3SpecLoop();
    if (!L) return nullptr;
    L->cfg = *cfg;
    L->verify = verify;
    L->commit = commit;
    L->ctx = ctx;
    L->arg_cap = (n_ids - cached) > (cfg->spec_n + 1) ? (n_ids - cached) : (cfg->spec_n + 1);
    if (cfg->policy == K3_DRAFT_TREE && L->arg_cap < cfg->tree_nodes) L->arg_cap = cfg->tree_nodes;
    L->seq = (int *)malloc(sizeof(int) * (size_t)cfg->tmax);
    L->arg = (int *)malloc(sizeof(int) * (size_t)L->arg_cap);
    L->stop = (int *)malloc(sizeof(int) * (size_t)(cfg->n_stop > 0 ? cfg->n_stop : 1));
    const bool sam = cfg->policy == K3_DRAFT_SUFFIX || cfg->policy == K3_DRAFT_P3 || cfg->policy == K3_DRAFT_TREE;
    if (sam) L->sam = k3_suffix_drafter_create(cfg->tmax);
    L->tok = (int *)malloc(sizeof(int) * (size_t)L->arg_cap);
    L->parent = (int *)malloc(sizeof(int) * (size_t)L->arg_cap);
    if (!L->seq || !L->arg || !L->stop || !L->tok || !L->parent || (sam && !L->sam)) {
        k3_spec_loop_free(L);
        return nullptr;
    }
    memcpy(L->seq, ids, sizeof(int) * (size_t)n_ids);
    if (cfg->n_stop > 0) memcpy(L->stop, cfg->stop_ids, sizeof(int) * (size_t)cfg->n_stop);
    L->cfg.stop_ids = L->stop;
    L->T = n_ids;
    L->cached = cached;
    if (L->sam && k3_suffix_drafter_push(L->sam, ids, n_ids) != K3GPU_OK) {
        k3_spec_loop_free(L);
        return nullptr;
    }
    return L;
}

extern "C" void k3_spec_loop_free(K3SpecLoop *L)
{
    if (!L) return;
    free(L->seq);
    free(L->arg);
    free(L->stop);
    free(L->tok);
    free(L->parent);
    k3_suffix_drafter_free(L->sam);
    delete L;
}

extern "C" int k3_spec_loop_step(K3SpecLoop *L, int *out, int *n_out, K3SpecStepTrace *trace)
{
    if (n_out) *n_out = 0;
    if (trace) memset(trace, 0, sizeof *trace);
    if (!L) return K3GPU_EINVAL;
    if (L->done) return L->done;
    if (L->cfg.policy == K3_DRAFT_MODEL && !L->dverify) return K3GPU_EINVAL;
    int emit[9], emitn = 0, keep = 0;
    const int base = L->cached;
    if (!L->started) {
        // the first step: every position not yet consumed, never tentative in the engine,
        // in passes of at most prefill_chunk positions with checkpoints between them
        const int n = L->T - base;
        int next = 0, upto = base;
        const int r = read_in(L, L->verify, L->commit, L->ctx, base, L->T, &upto, &next, true);
        L->cached = upto;
        if (r < 0) return r;
        if (r == 1) {                 // paused: positions base..upto read, nothing emitted
            L->done = K3_SPEC_LOOP_PAUSED;
            if (trace) *trace = K3SpecStepTrace{0, 0, 0, upto - base};
            return L->done;
        }
        L->started = 1;
        emit[emitn++] = next;
        if (L->cfg.policy == K3_DRAFT_MODEL) {
            // the draft model reads the whole conversation once, in the same passes (its
            // state is never saved, so a resumed run replays everything through it,
            // :2847-2853)
            int dupto = 0;
            const int rd = read_in(L, L->dverify, L->dcommit, L->dctx, 0, L->T, &dupto, nullptr, false);
            if (rd < 0) return rd;
            L->dcached = L->T;
        }
        keep = emit_keep(L, emit, emitn);
        if (trace) *trace = K3SpecStepTrace{0, 0, keep, n};
    } else if (L->cfg.policy == K3_DRAFT_TREE) {
        const K3SpecLoopCfg &c = L->cfg;
        int n = 1;
        L->tok[0] = L->seq[base];
        L->parent[0] = -1;
        if (L->T + c.spec_n + 1 < c.tmax && base + c.tree_nodes <= c.kv_cap)
            n = k3_suffix_drafter_tree(L->sam, c.tree_nodes, c.tree_branch, c.spec_n, c.min_len, L->tok, L->parent);
        if (n < 1) return K3GPU_EINVAL;
        if (L->verify(L->ctx, L->tok, L->parent, n, base, L->arg) != 0) return K3GPU_ECALLBACK;
        int path[9];
        const int plen = tree_accept(L->tok, L->parent, n, L->arg, path, c.spec_n + 1);
        const int m = plen - 1, nd = n - 1;
        for (int i = 1; i < plen; i++) emit[emitn++] = L->tok[path[i]];
        emit[emitn++] = L->arg[path[plen - 1]];
        keep = emit_keep(L, emit, emitn);
        const int used = nd > 0 ? keep : 1;
        if (L->commit(L->ctx, base, path, used) != 0) return K3GPU_ECALLBACK;
        L->cached = base + used;
        if (nd > 0) {
            L->st.sweeps++;
            L->st.drafted += nd;
            L->st.accepted += m;
            L->st.dropped += nd + 1 - keep;
            bool leaf = true;   // full: the accepted path ran to the end of its branch
            for (int i = path[plen - 1] + 1; i < n && leaf; i++) leaf = L->parent[i] != path[plen - 1];
            if (leaf) L->st.full++;
            else L->st.partial++;
            if (keep < m + 1) L->st.cut++;
            L->st.hist[m]++;
        }
        if (trace) *trace = K3SpecStepTrace{nd, m, keep, n};
    } else {
        int d[8], nd = 0, dlag = 0;
        const K3SpecLoopCfg &c = L->cfg;
        const bool room = L->T + c.spec_n + 1 < c.tmax && base + c.spec_n + 1 <= c.kv_cap;
        if (c.policy == K3_DRAFT_MODEL && room && c.spec_n > 0) {
            dlag = base - L->dcached;
            if (dlag < 0) return K3GPU_EINVAL;                 // the draft model is ahead
            if (dlag + c.spec_n > c.spec_n + 1) {              // a backlog past its log: absorb it
                if (L->dverify(L->dctx, L->seq + L->dcached, nullptr, dlag, L->dcached, L->arg) != 0 ||
                    L->dcommit(L->dctx, L->dcached, nullptr, dlag) != 0)
                    return K3GPU_ECALLBACK;
                L->dcached = base;
                dlag = 0;
            }
            // the unseen ids plus the pending one, then its own next ids, one at a time
            if (L->dverify(L->dctx, L->seq + L->dcached, nullptr, dlag + 1, L->dcached, L->arg) != 0)
                return K3GPU_ECALLBACK;
            d[nd++] = L->arg[dlag];
            while (nd < c.spec_n) {
                if (L->dverify(L->dctx, &d[nd - 1], nullptr, 1, base + nd, L->arg) != 0) return K3GPU_ECALLBACK;
                d[nd] = L->arg[0];
                nd++;
            }
            L->st.draft_rounds++;
            L->st.draft_drafted += nd;
        } else if (c.policy != K3_DRAFT_NONE && c.policy != K3_DRAFT_MODEL && room) {
            nd = draft(L, d);
        }
        int ids[9];
        ids[0] = L->seq[base];
        for (int i = 0; i < nd; i++) ids[1 + i] = d[i];
        if (L->verify(L->ctx, ids, nullptr, nd + 1, base, L->arg) != 0) return K3GPU_ECALLBACK;
        int m = 0;
        while (m < nd && L->arg[m] == d[m]) m++;
        for (int i = 0; i < m; i++) emit[emitn++] = d[i];
        emit[emitn++] = L->arg[m];
        keep = emit_keep(L, emit, emitn);
        // a serial step consumes its one position whatever the output keeps (:2972)
        const int used = nd > 0 ? keep : 1;
        if (L->commit(L->ctx, base, nullptr, used) != 0) return K3GPU_ECALLBACK;
        L->cached = base + used;
        if (nd > 0) {
            L->st.sweeps++;
            L->st.drafted += nd;
            L->st.accepted += m;
            L->st.dropped += nd + 1 - keep;
            if (m == nd) L->st.full++;
            else L->st.partial++;
            if (keep < m + 1) L->st.cut++;
            L->st.hist[m]++;
        }
        if (c.policy == K3_DRAFT_MODEL && nd > 0) {
            // the draft model keeps what the target kept of what it fed (:2956-2965)
            const int dkeep = keep < nd ? keep : nd;
            if (L->dcommit(L->dctx, base - dlag, nullptr, dlag + dkeep) != 0) return K3GPU_ECALLBACK;
            L->dcached = base + dkeep;
            L->st.draft_accepted += m;
            L->st.draft_dropped += nd - dkeep;
        }
        if (trace) *trace = K3SpecStepTrace{nd, m, keep, nd + 1};
    }
    L->st.steps++;
    if (append(L, emit, keep, out) != K3GPU_OK) return K3GPU_EINVAL;
    if (n_out) *n_out = keep;
    return K3GPU_OK;
}

extern "C" int k3_spec_loop_set_checkpoint(K3SpecLoop *L, K3SpecCheckpointFn fn, void *ctx)
{
    if (!L || L->started) return K3GPU_EINVAL;
    L->ckpt = fn;
    L->ckctx = ctx;
    return K3GPU_OK;
}

extern "C" void k3_spec_loop_request_pause(K3SpecLoop *L)
{
    if (L) L->pause_req.store(1);
}

extern "C" int k3_spec_loop_set_draft_model(K3SpecLoop *L, K3SpecVerifyFn dverify, K3SpecCommitFn dcommit,
                                            void *dctx)
{
    if (!L || !dverify || !dcommit || L->started || L->cfg.policy != K3_DRAFT_MODEL) return K3GPU_EINVAL;
    L->dverify = dverify;
    L->dcommit = dcommit;
    L->dctx = dctx;
    return K3GPU_OK;
}

extern "C" int k3_spec_loop_state(const K3SpecLoop *L, int *T, int *cached, int *nout, K3SpecLoopStats *stats)
{
    if (!L) return K3GPU_EINVAL;
    if (T) *T = L->T;
    if (cached) *cached = L->cached;
    if (nout) *nout = L->nout;
    if (stats) *stats = L->st;
    return L->done;
}

extern "C" int k3_spec_loop_ids(const K3SpecLoop *L, int *ids, int cap)
{
    if (!L || !ids || cap < L->T) return K3GPU_EINVAL;
    memcpy(ids, L->seq, sizeof(int) * (size_t)L->T);
    return L->T;
}

// ---- the layer loop's execution order (--loop / --loop-layers / --loop-count) --------
extern "C" int k3_layer_loop_plan(int n_layers, int attn_res_block, int preset, int loop_a, int loop_b,
                                  int loop_count, int *vmap, int vmap_cap, int *span_out, int *attn_res_extra)
{
    if (n_layers <= 0 || attn_res_block <= 0 || loop_count < 1 || loop_count > 8 || !vmap) return K3GPU_EINVAL;
    const int NL = n_layers, blk = attn_res_block;
    if (preset) {   // the whole block holding the middle layer (k3_run.c:2148-2152)
        const int mid = NL / 2;
        loop_a = mid - mid % blk;
        loop_b = loop_a + blk - 1 < NL - 1 ? loop_a + blk - 1 : NL - 1;
    }
    // whole AttnRes blocks within the stack, so every executed layer keeps its position in
    // its block and the block-boundary snapshots stay where they were trained (:2153-2160)
    if (loop_a < 0 || loop_b < loop_a || loop_b >= NL || loop_a % blk != 0 ||
        ((loop_b + 1) % blk != 0 && loop_b != NL - 1))
        return K3GPU_EINVAL;
    const int span = loop_b - loop_a + 1, NV = NL + (loop_count - 1) * span;
    if (vmap_cap < NV) return K3GPU_ECAPACITY;
    int nv = 0;
    for (int L = 0; L <= loop_b; L++) vmap[nv++] = L;
    for (int r = 1; r < loop_count; r++)
        for (int L = loop_a; L <= loop_b; L++) vmap[nv++] = L;
    for (int L = loop_b + 1; L < NL; L++) vmap[nv++] = L;
    if (span_out) {
        span_out[0] = loop_a;
        span_out[1] = loop_b;
    }
    if (attn_res_extra) *attn_res_extra = (loop_count - 1) * ((span + blk - 1) / blk);
    return NV;
}
