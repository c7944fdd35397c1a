// state.cu -- host C++: the conversation state file (K3ST version 2), byte for byte the
// format of the reference's k3_state_save / k3_state_peek / k3_state_load
// (src/cli/k3_run.c:162-407), so a session saved by either engine resumes on the other.
//
// Layout: the 96-byte header {magic "K3ST", int32 version 2, int32 fp[12], int32 n_bound,
// n_mla, cached, nseq, int64 kper, kvpp, ropepp}, the 24-byte layer-loop record {int32 a,
// b, count, nv; double eps}, then int32 ids[nseq]; with a loop (count > 0) int32
// pcached[count + 1] and int32 passes[nseq]; then float ks[kper * slots] (slots = nv with a
// loop, else n_bound: per layer the KDA matrices [H][D][D] then the ShortConv history
// [3][P][K-1]); then per MLA layer cached * kvpp cache floats, then per MLA layer cached *
// ropepp rope floats, position-major. Loading refuses what the reference refuses: another
// loop, another fingerprint, other layer counts, another cache width, more positions than
// the destination holds, or an id count other than cached or cached + 1.
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "k3gpu.h"

namespace {

#pragma pack(push, 1)
struct Hdr {
    char magic[4];
    int32_t version;
    int32_t fp[12];
    int32_t n_bound, n_mla, cached, nseq;
    int64_t kper;
    int64_t kvpp, ropepp;
};
struct Loop {
    int32_t a, b, count, nv;
    double eps;
};
#pragma pack(pop)
static_assert(sizeof(Hdr) == 96, "K3ST header");
static_assert(sizeof(Loop) == 24, "K3ST loop record");

bool wr(FILE *f, const void *p, size_t size, size_t n) { return n == 0 || fwrite(p, size, n, f) == n; }
bool rd(FILE *f, void *p, size_t size, size_t n) { return n == 0 || fread(p, size, n, f) == n; }

void to_layout(const Hdr &h, const Loop &l, K3StateLayout *s)
{
    memcpy(s->fp, h.fp, sizeof h.fp);
    s->n_bound = h.n_bound;
    s->n_mla = h.n_mla;
    s->kper = h.kper;
    s->kvpp = h.kvpp;
    s->ropepp = h.ropepp;
    s->loop_a = l.a;
    s->loop_b = l.b;
    s->loop_count = l.count;
    s->loop_nv = l.nv;
    s->loop_eps = l.eps;
}

// the header and loop record (version 1 reads as "no loop"); 0 or K3GPU_EINVAL
int peek(FILE *f, Hdr *h, Loop *l)
{
    if (!rd(f, h, sizeof *h, 1) || memcmp(h->magic, "K3ST", 4) != 0) return K3GPU_EINVAL;
    if (h->version != 1 && h->version != 2) return K3GPU_EINVAL;
    memset(l, 0, sizeof *l);
    l->a = l->b = -1;
    l->nv = h->n_bound;
    l->eps = -1.0;
    if (h->version == 2 && !rd(f, l, sizeof *l, 1)) return K3GPU_EINVAL;
    return K3GPU_OK;
}

size_t slots_of(int count, int nv, int n_bound) { return (size_t)(count ? nv : n_bound); }

}  // namespace

extern "C" int k3_state_save(const char *path, const K3StateLayout *s, const int *seq, int nseq, int cached,
                             const float *ks, const float *kvc, const float *ropec, int kv_cap, const int *pcached,
                             const int *passes)
{
    if (!path || !s || nseq < 0 || cached < 0 || cached > kv_cap || nseq < cached || nseq > cached + 1)
        return K3GPU_EINVAL;
    if (s->kper < 0 || s->kvpp < 0 || s->ropepp < 0 || s->n_bound < 0 || s->n_mla < 0 || s->loop_count < 0 ||
        s->loop_count > 8 || (s->loop_count && s->loop_nv < 0))
        return K3GPU_EINVAL;
    if ((nseq && !seq) || (s->kper && !ks) || (s->n_mla && cached && ((s->kvpp && !kvc) || (s->ropepp && !ropec))))
        return K3GPU_EINVAL;
    FILE *f = fopen(path, "wb");
    if (!f) return K3GPU_EINVAL;
    Hdr h;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "K3ST", 4);
    h.version = 2;
    memcpy(h.fp, s->fp, sizeof h.fp);
    h.n_bound = s->n_bound;
    h.n_mla = s->n_mla;
    h.cached = cached;
    h.nseq = nseq;
    h.kper = s->kper;
    h.kvpp = s->kvpp;
    h.ropepp = s->ropepp;
    Loop l;
    memset(&l, 0, sizeof l);
    l.a = s->loop_a;
    l.b = s->loop_b;
    l.count = s->loop_count;
    l.nv = s->loop_nv;
    l.eps = s->loop_eps;
    bool ok = wr(f, &h, sizeof h, 1) && wr(f, &l, sizeof l, 1) && wr(f, seq, sizeof(int), (size_t)nseq);
    if (ok && l.count) {
        static const int zero[9] = {0};
        ok = wr(f, pcached ? pcached : zero, sizeof(int), (size_t)l.count + 1);
        for (int i = 0; ok && i < nseq; i++) {
            const int v = passes ? passes[i] : 0;
            ok = wr(f, &v, sizeof v, 1);
        }
    }
    const size_t slots = slots_of(l.count, l.nv, h.n_bound);
    ok = ok && wr(f, ks, sizeof(float), (size_t)h.kper * slots);
    for (int mi = 0; ok && mi < h.n_mla; mi++)
        ok = wr(f, kvc + (size_t)mi * kv_cap * h.kvpp, sizeof(float), (size_t)cached * h.kvpp);
    for (int mi = 0; ok && mi < h.n_mla; mi++)
        ok = wr(f, ropec + (size_t)mi * kv_cap * h.ropepp, sizeof(float), (size_t)cached * h.ropepp);
    if (fclose(f) != 0) ok = false;
    return ok ? K3GPU_OK : K3GPU_EINVAL;
}

extern "C" int k3_state_peek(const char *path, K3StateLayout *s, int *cached, int *nseq)
{
    if (!path || !s) return K3GPU_EINVAL;
    FILE *f = fopen(path, "rb");
    if (!f) return K3GPU_EINVAL;
    Hdr h;
    Loop l;
    const int st = peek(f, &h, &l);
    fclose(f);
    if (st) return st;
    to_layout(h, l, s);
    if (cached) *cached = h.cached;
    if (nseq) *nseq = h.nseq;
    return K3GPU_OK;
}

extern "C" int k3_state_load(const char *path, const K3StateLayout *expect, int *seq, int seq_cap, float *ks,
                             float *kvc, float *ropec, int kv_cap, int *pcached, int *passes, int *cached, int *nseq)
{
    if (!path || !expect || !seq || !ks) return K3GPU_EINVAL;
    FILE *f = fopen(path, "rb");
    if (!f) return K3GPU_EINVAL;
    Hdr h;
    Loop l;
    int st = peek(f, &h, &l);
    if (st) { fclose(f); return st; }
    // the refusals of k3_state_load (src/cli/k3_run.c:268-325)
    const bool loop_ok = l.count == expect->loop_count &&
                         (!l.count || (l.a == expect->loop_a && l.b == expect->loop_b && l.nv == expect->loop_nv &&
                                       memcmp(&l.eps, &expect->loop_eps, sizeof l.eps) == 0));
    if (!loop_ok || memcmp(h.fp, expect->fp, sizeof h.fp) != 0 || h.n_bound != expect->n_bound ||
        h.n_mla != expect->n_mla || h.kvpp != expect->kvpp || h.ropepp != expect->ropepp || h.kper != expect->kper ||
        h.cached < 0 || h.nseq < h.cached || h.nseq > h.cached + 1) {
        fclose(f);
        return K3GPU_EINVAL;
    }
    // sizes the rest of the file is read with: never trusted past these bounds, whatever
    // the caller expects (the loop arrays hold at most 9 counters)
    if (l.count < 0 || l.count > 8 || (l.count && l.nv < 0) || h.n_bound < 0 || h.n_mla < 0 || h.kper < 0 ||
        h.kvpp < 0 || h.ropepp < 0) {
        fclose(f);
        return K3GPU_EINVAL;
    }
    if (h.cached > kv_cap || h.nseq > seq_cap) { fclose(f); return K3GPU_ECAPACITY; }
    if (h.n_mla && h.cached && ((h.kvpp && !kvc) || (h.ropepp && !ropec))) { fclose(f); return K3GPU_EINVAL; }
    bool ok = rd(f, seq, sizeof(int), (size_t)h.nseq);
    if (ok && l.count) {
        int scratch[9];
        ok = rd(f, pcached ? pcached : scratch, sizeof(int), (size_t)l.count + 1);
        for (int i = 0; ok && i < h.nseq; i++) {
            int v;
            ok = rd(f, &v, sizeof v, 1);
            if (ok && passes) passes[i] = v;
        }
    }
    const size_t slots = slots_of(l.count, l.nv, h.n_bound);
    ok = ok && rd(f, ks, sizeof(float), (size_t)h.kper * slots);
    for (int mi = 0; ok && mi < h.n_mla; mi++)
        ok = rd(f, kvc + (size_t)mi * kv_cap * h.kvpp, sizeof(float), (size_t)h.cached * h.kvpp);
    for (int mi = 0; ok && mi < h.n_mla; mi++)
        ok = rd(f, ropec + (size_t)mi * kv_cap * h.ropepp, sizeof(float), (size_t)h.cached * h.ropepp);
    fclose(f);
    if (!ok) return K3GPU_EINVAL;   // truncated
    if (cached) *cached = h.cached;
    if (nseq) *nseq = h.nseq;
    return K3GPU_OK;
}
