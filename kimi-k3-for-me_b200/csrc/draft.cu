// draft.cu -- host drafters beyond the engine's n-gram rule (host C++, no device code).
//
// The reference's drafting study (tools/spec_replay.py) defines two deterministic
// policies besides the engine's spec_draft:
//
//   P1  eager most-recent match (:174-184): the most recent earlier occurrence of the
//       history's suffix 4-gram, else 3-gram, else 2-gram; the ids that followed it, up to
//       the cap and the end of the history; no agreement gate.
//   P2  longest suffix match (:256-336, used at :442-449): the longest suffix of the
//       history that also ends earlier, its most recent earlier end e, and the ids after e
//       continued with period g = (T - 1) - e past the end of the history (an LZ77-style
//       overlapping copy); it fires when the match is at least min_len ids.
//
// P2 keeps an online suffix automaton over the token ids. Every state carries its
// largest end position and occurrence count; those are advanced along the suffix-link
// path one position late (the tool's commit after reading), so at a draft point they
// describe the history before its last id. Transitions live in one open-addressing hash
// table keyed by (state, id), with each state's transitions also chained in a list for the
// clone step.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "k3gpu.h"

namespace {

constexpr int SPEC_MAX = 8;   // K3_SPEC_MAX, the engine's draft cap

struct Trans {
    uint64_t key;   // (state << 32) | id
    int to;
    int next;       // next transition of the same state, -1 ends the list
};

}  // namespace

struct K3SuffixDrafter {
    int cap;             // most ids
    int n;               // ids pushed
    int pending;         // 1 when the last id's commit is still due
    int last;            // state of the whole history
    int n_states;
    int *seq, *len, *link, *last_end, *cnt, *head;   // head: first transition of a state
    Trans *tr;
    int n_tr, tr_cap;
    int *table;          // hash slot -> transition index, -1 empty
    uint64_t mask;
};

namespace {

uint64_t key_of(int state, int id) { return ((uint64_t)(uint32_t)state << 32) | (uint32_t)id; }

uint64_t hash64(uint64_t k)
{
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdULL;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ULL;
    k ^= k >> 33;
    return k;
}

// slot of key (its transition, or the empty slot where it would go)
uint64_t find_slot(const K3SuffixDrafter *d, uint64_t key)
{
    uint64_t s = hash64(key) & d->mask;
    while (d->table[s] >= 0 && d->tr[d->table[s]].key != key) s = (s + 1) & d->mask;
    return s;
}

int get(const K3SuffixDrafter *d, int state, int id)
{
    const uint64_t s = find_slot(d, key_of(state, id));
    return d->table[s] >= 0 ? d->tr[d->table[s]].to : -1;
}

// a new transition (the key is known to be absent); capacity was reserved up front
void add(K3SuffixDrafter *d, int state, int id, int to)
{
    const uint64_t key = key_of(state, id);
    const uint64_t s = find_slot(d, key);
    const int t = d->n_tr++;
    d->tr[t].key = key;
    d->tr[t].to = to;
    d->tr[t].next = d->head[state];
    d->head[state] = t;
    d->table[s] = t;
}

void redirect(K3SuffixDrafter *d, int state, int id, int to)
{
    const uint64_t s = find_slot(d, key_of(state, id));
    d->tr[d->table[s]].to = to;
}

// the tool's commit(pos): occurrence figures of every proper suffix state of the history
void commit(K3SuffixDrafter *d, int pos)
{
    int v = d->link[d->last];
    while (v > 0) {
        d->last_end[v] = pos;
        d->cnt[v] += 1;
        v = d->link[v];
    }
}

// the tool's extend(c, pos)
void extend(K3SuffixDrafter *d, int c, int pos)
{
    const int cur = d->n_states++;
    d->len[cur] = d->len[d->last] + 1;
    d->link[cur] = 0;
    d->head[cur] = -1;
    d->last_end[cur] = pos;
    d->cnt[cur] = 1;
    int p = d->last;
    while (p != -1 && get(d, p, c) < 0) {
        add(d, p, c, cur);
        p = d->link[p];
    }
    if (p != -1) {
        const int q = get(d, p, c);
        if (d->len[p] + 1 == d->len[q]) {
            d->link[cur] = q;
        } else {
            const int clone = d->n_states++;
            d->len[clone] = d->len[p] + 1;
            d->link[clone] = d->link[q];
            d->head[clone] = -1;
            for (int t = d->head[q]; t >= 0; t = d->tr[t].next)
                add(d, clone, (int)(uint32_t)(d->tr[t].key & 0xffffffffu), d->tr[t].to);
            d->last_end[clone] = d->last_end[q];
            d->cnt[clone] = d->cnt[q];
            while (p != -1 && get(d, p, c) == q) {
                redirect(d, p, c, clone);
                p = d->link[p];
            }
            d->link[q] = clone;
            d->link[cur] = clone;
        }
    }
    d->last = cur;
}

}  // namespace

extern "C" int k3_spec_draft_eager(const int *seq, int T, int cap, int *out)
{
    if (!seq || T < 0 || cap < 0 || (cap > 0 && !out)) return 0;
    if (cap > SPEC_MAX) cap = SPEC_MAX;
    for (int n = 4; n >= 2; n--) {
        if (T < n + 1) continue;
        for (int j = T - n - 1; j >= 0; j--) {
            int hit = 1;
            for (int i = 0; i < n && hit; i++) hit = seq[j + i] == seq[T - n + i];
            if (!hit) continue;
            int nd = 0;
            while (nd < cap && j + n + nd < T) {
                out[nd] = seq[j + n + nd];
                nd++;
            }
            return nd;
        }
    }
    return 0;
}

extern "C" K3SuffixDrafter *k3_suffix_drafter_create(int capacity)
{
    if (capacity <= 0 || capacity > (1 << 28)) return nullptr;
    K3SuffixDrafter *d = (K3SuffixDrafter *)calloc(1, sizeof(K3SuffixDrafter));
    if (!d) return nullptr;
    const int ns = 2 * capacity + 2;            // a suffix automaton has < 2n states
    d->cap = capacity;
    d->tr_cap = 3 * capacity + 4;               // and < 3n transitions
    uint64_t slots = 16;
    while (slots < (uint64_t)2 * d->tr_cap) slots <<= 1;
    d->mask = slots - 1;
    d->seq = (int *)malloc(sizeof(int) * (size_t)capacity);
    d->len = (int *)malloc(sizeof(int) * (size_t)ns);
    d->link = (int *)malloc(sizeof(int) * (size_t)ns);
    d->last_end = (int *)malloc(sizeof(int) * (size_t)ns);
    d->cnt = (int *)malloc(sizeof(int) * (size_t)ns);
    d->head = (int *)malloc(sizeof(int) * (size_t)ns);
    d->tr = (Trans *)malloc(sizeof(Trans) * (size_t)d->tr_cap);
    d->table = (int *)malloc(sizeof(int) * (size_t)slots);
    if (!d->seq || !d->len || !d->link || !d->last_end || !d->cnt || !d->head || !d->tr || !d->table) {
        k3_suffix_drafter_free(d);
        return nullptr;
    }
    memset(d->table, 0xff, sizeof(int) * (size_t)slots);
    d->n_states = 1;                            // the root
    d->len[0] = 0;
    d->link[0] = -1;
    d->last_end[0] = -1;
    d->cnt[0] = 0;
    d->head[0] = -1;
    return d;
}

extern "C" void k3_suffix_drafter_free(K3SuffixDrafter *d)
{
    if (!d) return;
    free(d->seq);
    free(d->len);
    free(d->link);
    free(d->last_end);
    free(d->cnt);
    free(d->head);
    free(d->tr);
    free(d->table);
    free(d);
}

extern "C" int k3_suffix_drafter_push(K3SuffixDrafter *d, const int *ids, int n)
{
    if (!d || n < 0 || (n > 0 && !ids)) return K3GPU_EINVAL;
    if (n > d->cap - d->n) return K3GPU_ECAPACITY;
    for (int i = 0; i < n; i++) {
        if (d->pending) commit(d, d->n - 1);
        d->seq[d->n] = ids[i];
        extend(d, ids[i], d->n);
        d->n++;
        d->pending = 1;
    }
    return K3GPU_OK;
}

extern "C" int k3_suffix_drafter_length(const K3SuffixDrafter *d) { return d ? d->n : 0; }

extern "C" int k3_suffix_drafter_draft(const K3SuffixDrafter *d, int cap, int min_len, int *out, int *match_len,
                                       int *period)
{
    if (match_len) *match_len = 0;
    if (period) *period = 0;
    if (!d || d->n == 0 || cap <= 0 || !out) return 0;
    if (cap > SPEC_MAX) cap = SPEC_MAX;
    // the longest suffix that also ends earlier: the whole history's suffix link
    const int v = d->link[d->last];
    if (v <= 0) return 0;
    const int L = d->len[v], e = d->last_end[v], pos = d->n - 1;
    if (match_len) *match_len = L;
    const int g = pos - e;
    if (period) *period = g;
    if (L < min_len || g <= 0) return 0;
    for (int i = 0; i < cap; i++) out[i] = d->seq[e + 1 + (i % g)];
    return cap;
}

// ---- P3: P2's draft with an adaptive length (tools/spec_replay.py:340-397, 525-568) ----
// Each draft position j (1-based) gets a feature code from its depth, the effective match
// length L + j - 1 and the agreement counts of its context (the matched suffix followed
// by the draft's first j - 1 ids): n, the context's occurrences, and k, those followed by
// the proposed id, as the automaton's occurrence counts read between extend and commit
// (the state this drafter keeps between pushes). A table q[code] of acceptance estimates,
// fitted offline, turns the codes into a length.

namespace {

constexpr int P3_N_ELL = 13, P3_N_AGREE = 6, P3_NO_DRAFT = 255;

int p3_ell_bucket(int ell)
{
    static const int edges[P3_N_ELL] = {1, 2, 3, 4, 5, 6, 7, 9, 12, 16, 24, 32, 64};
    if (ell >= 64) return P3_N_ELL - 1;
    int b = 0;
    for (int i = 0; i < P3_N_ELL; i++)
        if (edges[i] <= ell) b = i;
    return b;
}

int p3_agree_bucket(int n, int k)
{
    if (k <= 0) return 0;                 // never followed
    if (n <= 1) return 1;                 // one occurrence
    if (k >= n) return n <= 3 ? 2 : 3;    // unanimous
    return 2 * k >= n ? 4 : 5;            // majority / minority
}

int p3_depth_bucket(int j) { return j == 1 ? 0 : (j <= 3 ? 1 : 2); }

// the cost of a verify step over nd drafts in units of one plain decode step
// (tools/spec_replay.py:85-96): a_T + a_E * u(nd + 1) + a_C * (nd + 1) + eps, with
// u(n) = r * (1 - ((r - 1) / r)^n) the expected distinct experts over n positions in units
// of one position's top-k (r = experts / top-k); a step without drafts costs 1
double p3_verify_cost(int nd, const K3SpecCost *c, double eps)
{
    if (nd <= 0) return 1.0;
    const int n = nd + 1;
    const double u = c->expert_ratio * (1.0 - pow((c->expert_ratio - 1.0) / c->expert_ratio, (double)n));
    return c->a_T + c->a_E * u + c->a_C * n + eps;
}

// the second pass that restores and replays m + 1 positions after a partial acceptance
double p3_replay_cost(int m, const K3SpecCost *c)
{
    const int n = m + 1;
    const double u = c->expert_ratio * (1.0 - pow((c->expert_ratio - 1.0) / c->expert_ratio, (double)n));
    return c->a_T + c->a_E * u + c->a_C * n;
}

}  // namespace

extern "C" int k3_suffix_drafter_features(const K3SuffixDrafter *d, const int *draft, int nd, uint8_t *codes)
{
    if (!d || nd < 0 || nd > SPEC_MAX || (nd > 0 && (!draft || !codes))) return K3GPU_EINVAL;
    const int v = d->n ? d->link[d->last] : 0;
    if (v <= 0) {
        for (int j = 0; j < nd; j++) codes[j] = (uint8_t)P3_NO_DRAFT;
        return K3GPU_OK;
    }
    const int L = d->len[v];
    int w = v;
    for (int j = 0; j < nd; j++) {
        int n = 0, k = 0, w2 = -1;
        if (w >= 0) {
            n = d->cnt[w];
            w2 = get(d, w, draft[j]);
            k = w2 >= 0 ? d->cnt[w2] : 0;
        }
        codes[j] = (uint8_t)((p3_depth_bucket(j + 1) * P3_N_ELL + p3_ell_bucket(L + j)) * P3_N_AGREE +
                             p3_agree_bucket(n, k));
        w = w2;
    }
    return K3GPU_OK;
}

extern "C" int k3_spec_p3_length(const uint8_t *codes, int nd, const double *q, double delta, int cumulative)
{
    if (!codes || !q || nd <= 0 || codes[0] == P3_NO_DRAFT) return 0;
    if (nd > SPEC_MAX) nd = SPEC_MAX;
    int len = 0;
    double P = 1.0;
    bool run = true;
    for (int j = 0; j < nd; j++) {
        if (codes[j] >= K3_SPEC_P3_CODES) return 0;
        const double qj = q[codes[j]];
        if (cumulative) {
            P = j == 0 ? qj : P * qj;   // positions whose cumulative estimate exceeds delta
            len += P > delta;
        } else {
            run = run && qj > delta;    // the leading positions each above delta
            len += run;
        }
    }
    return len;
}

extern "C" int k3_spec_p3_cost_length(const uint8_t *codes, int nd, const double *q, const K3SpecCost *cost,
                                      int replay)
{
    if (!codes || !q || !cost || nd <= 0 || codes[0] == P3_NO_DRAFT) return 0;
    if (!(cost->expert_ratio >= 1.0)) return 0;
    if (nd > SPEC_MAX) nd = SPEC_MAX;
    double prev = 1.0, P = 1.0;
    for (int j = 1; j <= nd; j++) {
        if (codes[j - 1] >= K3_SPEC_P3_CODES) return 0;
        P = j == 1 ? q[codes[0]] : P * q[codes[j - 1]];
        double extra = p3_verify_cost(j, cost, cost->eps) - p3_verify_cost(j - 1, cost, cost->eps);
        if (replay) extra = extra + (prev - P) * p3_replay_cost(j - 1, cost);
        if (!(P > extra)) return j - 1;
        prev = P;
    }
    return nd;
}

extern "C" int k3_suffix_drafter_draft_p3(const K3SuffixDrafter *d, const double *q, double delta,
                                          const K3SpecCost *cost, int replay, int cap, int *out)
{
    if (!d || !q || cap <= 0 || !out) return 0;
    if (cap > SPEC_MAX) cap = SPEC_MAX;
    int draft[SPEC_MAX];
    uint8_t codes[SPEC_MAX];
    if (k3_suffix_drafter_draft(d, SPEC_MAX, 1, draft, nullptr, nullptr) != SPEC_MAX) return 0;
    if (k3_suffix_drafter_features(d, draft, SPEC_MAX, codes) != K3GPU_OK) return 0;
    int len = cost ? k3_spec_p3_cost_length(codes, SPEC_MAX, q, cost, replay)
                   : k3_spec_p3_length(codes, SPEC_MAX, q, delta, 1);
    if (len > cap) len = cap;
    for (int i = 0; i < len; i++) out[i] = draft[i];
    return len;
}

// A draft tree for tree verification. Node 0 is the pending id (the last of the history);
// its context is the longest suffix that occurred before (state link[last]). A node's
// children are the ids that followed its context in the history, most often first (ties:
// the smaller id), at most `branch` of them, each with probability k / n: k the times the
// context was followed by that id, n the times it was followed by anything. A context
// that was never followed backs off to its longest suffix with more occurrences (its
// suffix link) while that suffix keeps >= min_len ids. Nodes are added best-first by the
// product of the probabilities along their path (ties: the earliest candidate), up to
// max_nodes nodes and max_depth below the root. tok/parent [max_nodes]; parents precede
// their children; parent[0] = -1. Returns the node count (1: the root alone).
//
// Occurrence counts: cnt[] of a state counts its end positions up to the last commit; the
// commit for the newest position is deferred to the next push, so the proper suffix
// states of the history (the link path from link[last]) each lack that one occurrence.
// It is added back here, which makes k exact.
extern "C" int k3_suffix_drafter_tree(const K3SuffixDrafter *d, int max_nodes, int branch, int max_depth,
                                      int min_len, int *tok, int *parent)
{
    if (!d || d->n == 0 || max_nodes < 1 || max_nodes > 65536 || !tok || !parent) return 0;
    if (branch < 1) branch = 1;
    if (branch > 16) branch = 16;
    tok[0] = d->seq[d->n - 1];
    parent[0] = -1;
    int n = 1;
    const int v0 = d->link[d->last];
    if (v0 <= 0 || d->len[v0] < min_len || max_depth < 1 || max_nodes == 1) return n;
    // the link path from v0 (strictly decreasing len): the states owed the deferred commit
    int np = 0;
    for (int v = v0; v > 0; v = d->link[v]) np++;
    int *path = (int *)malloc(sizeof(int) * (size_t)np);
    struct Cand {
        double p;
        int par, id, state, depth;
    };
    const int max_c = max_nodes * branch + 1;
    Cand *cand = (Cand *)malloc(sizeof(Cand) * (size_t)max_c);
    if (!path || !cand) {
        free(path);
        free(cand);
        return n;
    }
    np = 0;
    for (int v = v0; v > 0; v = d->link[v]) path[np++] = v;
    auto count = [&](int w) {
        int lo = 0, hi = np;   // binary search by len (decreasing along the path)
        while (lo < hi) {
            const int mid = (lo + hi) / 2;
            if (d->len[path[mid]] > d->len[w]) lo = mid + 1;
            else hi = mid;
        }
        return d->cnt[w] + ((d->pending && lo < np && path[lo] == w) ? 1 : 0);
    };
    int nc = 0;
    // the continuations of node `node` (context state `st`, path probability `pp`)
    auto expand = [&](int node, int st, double pp, int depth) {
        while (st > 0 && d->head[st] < 0 && d->link[st] > 0 && d->len[d->link[st]] >= min_len) st = d->link[st];
        if (st <= 0 || d->head[st] < 0) return;
        int ids[16], tos[16], ks[16], k = 0;
        long long total = 0;
        for (int t = d->head[st]; t >= 0; t = d->tr[t].next) {
            const int id = (int)(uint32_t)(d->tr[t].key & 0xffffffffu), to = d->tr[t].to, c = count(to);
            total += c;
            int pos = k;
            while (pos > 0 && (ks[pos - 1] < c || (ks[pos - 1] == c && ids[pos - 1] > id))) pos--;
            if (pos >= branch) continue;
            for (int q = (k < branch ? k : branch - 1); q > pos; q--) {
                ids[q] = ids[q - 1];
                tos[q] = tos[q - 1];
                ks[q] = ks[q - 1];
            }
            ids[pos] = id;
            tos[pos] = to;
            ks[pos] = c;
            if (k < branch) k++;
        }
        for (int q = 0; q < k && nc < max_c; q++)
            cand[nc++] = Cand{pp * ((double)ks[q] / (double)total), node, ids[q], tos[q], depth + 1};
    };
    expand(0, v0, 1.0, 0);
    while (n < max_nodes && nc > 0) {
        int best = 0;
        for (int i = 1; i < nc; i++)
            if (cand[i].p > cand[best].p) best = i;
        const Cand c = cand[best];
        for (int i = best; i + 1 < nc; i++) cand[i] = cand[i + 1];
        nc--;
        tok[n] = c.id;
        parent[n] = c.par;
        const int node = n++;
        if (c.depth < max_depth) expand(node, c.state, c.p, c.depth);
    }
    free(path);
    free(cand);
    return n;
}
