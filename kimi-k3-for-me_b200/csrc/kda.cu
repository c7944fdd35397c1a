// kda.cu -- Kimi Delta Attention for the verify sweep: the tentative recurrence, the
// bit-exact commit of the kept prefix, the fused prologue and the norm/gate epilogue.
//
// The recurrence (k3_kda_step, src/core/k3_ops.c:303-360 of the reference) is
// column-separable: column j of S evolves from k, q, alpha, beta and v[j] alone. So one
// CTA runs one (sequence, head) with one thread per column, the column held in
// registers for the whole chunk: decay, u_j = sum_i k_i S_ij (i ascending, float,
// separately rounded), the delta write, o_j = sum_i q_i S_ij -- the same float
// operations in the same order as the reference, hence bit-identical state and output.
// The carried state is only read during verify; commit replays the logged operands.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace k3 {

template <int D>
__device__ __forceinline__ void kda_steps(float (&Sc)[D], float *__restrict__ o,
                                          const float *__restrict__ q,
                                          const float *__restrict__ k,
                                          const float *__restrict__ v,
                                          const float *__restrict__ al,
                                          const float *__restrict__ beta, int T, int H,
                                          float qscale, float *sm /* 3*D */)
{
    const int j = threadIdx.x;
    const int h = blockIdx.x;
    float *sk = sm, *sq = sm + D, *sa = sm + 2 * D;
    for (int t = 0; t < T; t++) {
        const size_t off = ((size_t)t * H + h) * D;
        __syncthreads();
        sk[j] = k[off + j];
        sa[j] = al[off + j];
        if (o) sq[j] = __fmul_rn(q[off + j], qscale);
        __syncthreads();
        const float bt = beta[(size_t)t * H + h];
        // 1. decay every row
#pragma unroll
        for (int i = 0; i < D; i++) Sc[i] = __fmul_rn(Sc[i], sa[i]);
        // 2. u = S^T k, rows with k_i == 0 skipped (k3_ops.c:333)
        float u = 0.0f;
#pragma unroll
        for (int i = 0; i < D; i++) {
            const float ki = sk[i];
            if (ki != 0.0f) u = __fadd_rn(u, __fmul_rn(ki, Sc[i]));
        }
        // 3. S += k (beta (v - u))^T, evaluated as (k_i * beta) * (v_j - u_j)
        const float err = __fsub_rn(v[off + j], u);
#pragma unroll
        for (int i = 0; i < D; i++) {
            const float ki = sk[i];
            if (ki != 0.0f) Sc[i] = __fadd_rn(Sc[i], __fmul_rn(__fmul_rn(ki, bt), err));
        }
        // 4. o = S^T q from the updated state, rows with q_i == 0 skipped
        if (o) {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < D; i++) {
                const float qi = sq[i];
                if (qi != 0.0f) acc = __fadd_rn(acc, __fmul_rn(qi, Sc[i]));
            }
            o[off + j] = acc;
        }
    }
}

// grid (H, B), block D. state [B][H][D][D]; rows [B][T][H][D]; beta [B][T][H].
template <int D>
__global__ void __launch_bounds__(D) kda_verify_kernel(float *__restrict__ o,
                                                      const float *__restrict__ state,
                                                      const float *__restrict__ q,
                                                      const float *__restrict__ k,
                                                      const float *__restrict__ v,
                                                      const float *__restrict__ al,
                                                      const float *__restrict__ beta, int T,
                                                      int H, float qscale)
{
    __shared__ float sm[3 * D];
    const int h = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
    const float *Sh = state + (((size_t)b * H + h) * D) * D;
    float Sc[D];
#pragma unroll
    for (int i = 0; i < D; i++) Sc[i] = Sh[(size_t)i * D + j];
    const size_t rb = (size_t)b * T * H * D;
    kda_steps<D>(Sc, o + rb, q + rb, k + rb, v + rb, al + rb, beta + (size_t)b * T * H, T, H,
                 qscale, sm);
}

template <int D>
__global__ void __launch_bounds__(D) kda_commit_kernel(float *__restrict__ state,
                                                      const float *__restrict__ k,
                                                      const float *__restrict__ v,
                                                      const float *__restrict__ al,
                                                      const float *__restrict__ beta,
                                                      const int *__restrict__ nkeep, int T,
                                                      int H)
{
    __shared__ float sm[3 * D];
    const int h = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
    int n = nkeep[b];
    if (n < 0 || n > T) {
        if (j == 0 && h == 0) flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : T;
    }
    if (n == 0) return;
    float *Sh = state + (((size_t)b * H + h) * D) * D;
    float Sc[D];
#pragma unroll
    for (int i = 0; i < D; i++) Sc[i] = Sh[(size_t)i * D + j];
    const size_t rb = (size_t)b * T * H * D;
    kda_steps<D>(Sc, nullptr, nullptr, k + rb, v + rb, al + rb, beta + (size_t)b * T * H, n, H,
                 0.0f, sm);
#pragma unroll
    for (int i = 0; i < D; i++) Sh[(size_t)i * D + j] = Sc[i];
}

// grid (H, B), block D: node t of a draft tree (parent[0] = -1, parent[t] < t; a parent of
// -1 means the carried state) reads the state after its own ancestors, with the same float
// operations in the same order as the chain kernel, so every node's output is bit-identical
// to a chain verify of its ancestor path. parent is a device array [T] shared by the B
// sequences.
//
// Most nodes of a draft tree are leaves, and a leaf's output needs its parent's state, not
// its own: o = (decay(S) + k (beta (v - u))^T)^T q is two passes over the parent's column
// (u first, then o, the updated entries recomputed on the fly and never stored). So only
// the INTERNAL nodes step the register-held column forward, visited in depth-first preorder
// (a child of the node just stepped costs one step; any other internal node re-runs its
// path from the carried state), and after each one its leaf children are evaluated from
// its state, KT_LEAVES at a time side by side (independent chains in one thread). A
// 64-node tree of branching 4 and depth 4 then costs ~20 steps and 12 leaf passes instead
// of one chain of depth + 1 steps per node.
constexpr int KT_LEAVES_MAX = 4;

template <int D>
__global__ void __launch_bounds__(D) kda_verify_tree_kernel(float *__restrict__ o,
                                                           const float *__restrict__ state,
                                                           const float *__restrict__ q,
                                                           const float *__restrict__ k,
                                                           const float *__restrict__ v,
                                                           const float *__restrict__ al,
                                                           const float *__restrict__ beta,
                                                           const int *__restrict__ parent, int T,
                                                           int H, float qscale)
{
    constexpr int KT_LEAVES = KT_LEAVES_MAX;
    extern __shared__ float Ss[];                       // [D][D]: a parked state column per thread
    __shared__ float sm[3 * D];                         // one stepped node: k, q * qscale, alpha
    __shared__ __align__(16) float lk[KT_LEAVES][D], la[KT_LEAVES][D], lq[KT_LEAVES][D];
    __shared__ int par[64], nch[64];
    __shared__ int items[66], n_items;                  // internal nodes in preorder (-1: the carried state)
    __shared__ int leaf[64], leaf0[66];                 // leaves grouped by item
    __shared__ int path[64], plen;
    const int h = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
    const float *Sh = state + (((size_t)b * H + h) * D) * D;
    const size_t rb = (size_t)b * T * H * D;
    const float *qb = q + rb, *kb = k + rb, *vb = v + rb, *ab = al + rb;
    const float *bb = beta + (size_t)b * T * H;
    float *sk = sm, *sq = sm + D, *sa = sm + 2 * D;

    if (j == 0) {
        // parents checked once (a bad one is flagged and read as the carried state)
        for (int t = 0; t < T; t++) {
            int pa = parent[t];
            if (pa >= t || pa < -1) {
                flag(DEV_BAD_INDEX);
                pa = -1;
            }
            par[t] = pa;
            nch[t] = 0;
        }
        for (int t = 0; t < T; t++)
            if (par[t] >= 0) nch[par[t]]++;
        // depth-first preorder over the nodes, children in ascending order (an explicit
        // stack: every node is pushed once); internal nodes become items, each followed by
        // its leaf children. The carried state is item 0 when some root is a leaf.
        int stack[64], sp = 0, ni = 0, nl = 0;
        bool root_leaf = false;
        for (int t = 0; t < T; t++) root_leaf |= par[t] < 0 && nch[t] == 0;
        if (root_leaf) {
            items[ni] = -1;
            leaf0[ni++] = nl;
            for (int t = 0; t < T; t++)
                if (par[t] < 0 && nch[t] == 0) leaf[nl++] = t;
        }
        for (int t = T - 1; t >= 0; t--)
            if (par[t] < 0 && nch[t] > 0) stack[sp++] = t;
        while (sp > 0) {
            const int n = stack[--sp];
            items[ni] = n;
            leaf0[ni++] = nl;
            for (int c = n + 1; c < T; c++)
                if (par[c] == n && nch[c] == 0) leaf[nl++] = c;
            for (int c = T - 1; c > n; c--)
                if (par[c] == n && nch[c] > 0) stack[sp++] = c;
        }
        leaf0[ni] = nl;
        n_items = ni;
    }
    __syncthreads();

    float Sc[D];
    int cur = -2;   // the node whose state Sc holds (-1: the carried state, -2: none yet)
    const int ni = n_items;
    for (int it = 0; it < ni; it++) {
        const int n = items[it];
        // the nodes to step, root-most first: n alone when Sc holds its parent's state, else
        // n's whole path from the carried state (its ancestors were emitted when visited)
        const bool reload = n < 0 || par[n] != cur;
        __syncthreads();
        if (j == 0) {
            int len = 0;
            if (n >= 0 && !reload) path[len++] = n;
            else
                for (int a = n; a >= 0 && len < 64; a = par[a]) path[len++] = a;
            for (int x = 0; x < len / 2; x++) {   // root-most first
                const int tmp = path[x];
                path[x] = path[len - 1 - x];
                path[len - 1 - x] = tmp;
            }
            plen = len;
        }
        __syncthreads();
        if (reload) {
#pragma unroll
            for (int i = 0; i < D; i++) Sc[i] = Sh[(size_t)i * D + j];
        }
        const int pl = plen;
        for (int pi = 0; pi < pl; pi++) {   // one k3_kda_step per node; the last one emits
            const int node = path[pi];
            const bool emit = pi == pl - 1;
            const size_t off = ((size_t)node * H + h) * D;
            __syncthreads();
            sk[j] = kb[off + j];
            sa[j] = ab[off + j];
            if (emit) sq[j] = __fmul_rn(qb[off + j], qscale);
            __syncthreads();
            const float bt = bb[(size_t)node * H + h];
#pragma unroll
            for (int i = 0; i < D; i++) Sc[i] = __fmul_rn(Sc[i], sa[i]);
            float u = 0.0f;
#pragma unroll
            for (int i = 0; i < D; i++) {
                const float ki = sk[i];
                if (ki != 0.0f) u = __fadd_rn(u, __fmul_rn(ki, Sc[i]));
            }
            const float err = __fsub_rn(vb[off + j], u);
#pragma unroll
            for (int i = 0; i < D; i++) {
                const float ki = sk[i];
                if (ki != 0.0f) Sc[i] = __fadd_rn(Sc[i], __fmul_rn(__fmul_rn(ki, bt), err));
            }
            if (emit) {
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < D; i++) {
                    const float qi = sq[i];
                    if (qi != 0.0f) acc = __fadd_rn(acc, __fmul_rn(qi, Sc[i]));
                }
                o[rb + off + j] = acc;
            }
        }
        cur = n;
        if (leaf0[it] == leaf0[it + 1]) continue;
        // this item's leaf children, KT_LEAVES side by side. The column is parked in shared
        // memory ([i][j]: conflict-free) for the leaf passes, which then hold no 128-entry
        // register array, and taken back afterwards (the barriers between make the reload
        // real, so Sc is dead while the leaves run)
#pragma unroll
        for (int i = 0; i < D; i++) Ss[i * D + j] = Sc[i];
        for (int l0 = leaf0[it]; l0 < leaf0[it + 1]; l0 += KT_LEAVES) {
            const int nl = min(KT_LEAVES, leaf0[it + 1] - l0);
            __syncthreads();
#pragma unroll
            for (int c = 0; c < KT_LEAVES; c++) {
                if (c < nl) {
                    const size_t off = ((size_t)leaf[l0 + c] * H + h) * D;
                    lk[c][j] = kb[off + j];
                    la[c][j] = ab[off + j];
                    lq[c][j] = __fmul_rn(qb[off + j], qscale);
                } else {   // an absent leaf: zero k and q rows (no update, no output)
                    lk[c][j] = 0.0f;
                    la[c][j] = 1.0f;
                    lq[c][j] = 0.0f;
                }
            }
            __syncthreads();
            float u[KT_LEAVES], bt[KT_LEAVES], vj[KT_LEAVES];
#pragma unroll
            for (int c = 0; c < KT_LEAVES; c++) {
                const int node = c < nl ? leaf[l0 + c] : 0;
                u[c] = 0.0f;
                bt[c] = c < nl ? bb[(size_t)node * H + h] : 0.0f;
                vj[c] = c < nl ? vb[((size_t)node * H + h) * D + j] : 0.0f;
            }
            // u = (decayed S)^T k, the decayed entries recomputed; four rows at a time, the
            // leaves' k and alpha as float4 broadcasts
#pragma unroll 2
            for (int i0 = 0; i0 < D; i0 += 4) {
                float sv[4];
#pragma unroll
                for (int r = 0; r < 4; r++) sv[r] = Ss[(i0 + r) * D + j];
#pragma unroll
                for (int c = 0; c < KT_LEAVES; c++) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(&lk[c][i0]);
                    const float4 a4 = *reinterpret_cast<const float4 *>(&la[c][i0]);
                    const float kv[4] = {k4.x, k4.y, k4.z, k4.w}, av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                    for (int r = 0; r < 4; r++)
                        if (kv[r] != 0.0f) u[c] = __fadd_rn(u[c], __fmul_rn(kv[r], __fmul_rn(sv[r], av[r])));
                }
            }
            float err[KT_LEAVES], acc[KT_LEAVES];
#pragma unroll
            for (int c = 0; c < KT_LEAVES; c++) {
                err[c] = __fsub_rn(vj[c], u[c]);
                acc[c] = 0.0f;
            }
            // o = (updated S)^T q, each updated entry formed as the chain forms it
#pragma unroll 2
            for (int i0 = 0; i0 < D; i0 += 4) {
                float sv[4];
#pragma unroll
                for (int r = 0; r < 4; r++) sv[r] = Ss[(i0 + r) * D + j];
#pragma unroll
                for (int c = 0; c < KT_LEAVES; c++) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(&lk[c][i0]);
                    const float4 a4 = *reinterpret_cast<const float4 *>(&la[c][i0]);
                    const float4 q4 = *reinterpret_cast<const float4 *>(&lq[c][i0]);
                    const float kv[4] = {k4.x, k4.y, k4.z, k4.w}, av[4] = {a4.x, a4.y, a4.z, a4.w};
                    const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                    for (int r = 0; r < 4; r++) {
                        float sx = __fmul_rn(sv[r], av[r]);
                        if (kv[r] != 0.0f) sx = __fadd_rn(sx, __fmul_rn(__fmul_rn(kv[r], bt[c]), err[c]));
                        if (qv[r] != 0.0f) acc[c] = __fadd_rn(acc[c], __fmul_rn(qv[r], sx));
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < KT_LEAVES; c++)
                if (c < nl) o[rb + ((size_t)leaf[l0 + c] * H + h) * D + j] = acc[c];
        }
#pragma unroll
        for (int i = 0; i < D; i++) Sc[i] = Ss[i * D + j];
    }
}

__device__ __forceinline__ float silu_f(float a) { return a * sigmoid_cr(a); }

// Block-wide double sum over blockDim.x (a multiple of 32, <= 1024) threads.
__device__ __forceinline__ double block_sum_d(double v, double *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// grid (H, B), block D (thread = channel d of head h). Runs the three ShortConvs of the
// head's channels over T, L2-normalises q and k per (t, head), computes alpha and beta.
__global__ void __launch_bounds__(256) kda_prologue_kernel(
    float *__restrict__ q, float *__restrict__ k, float *__restrict__ v,
    float *__restrict__ alpha, float *__restrict__ beta, float *__restrict__ pre,
    const float *__restrict__ z, const float *__restrict__ bproj, const float *__restrict__ qc,
    const float *__restrict__ kc, const float *__restrict__ vc, const float *__restrict__ hist,
    const float *__restrict__ A_log, const float *__restrict__ dt_bias, int T, int H, int D,
    int K, float lb, const int *__restrict__ parent)
{
    __shared__ double red[32];
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const int P = H * D, c = h * D + d, hl = K - 1;
    float *rows[3] = {q, k, v};
    const float *w[3] = {qc, kc, vc};
    float buf[3][8];
    float hist0[3][8];
    float wt[3][8];
#pragma unroll
    for (int m = 0; m < 3; m++) {
        for (int j = 0; j < hl; j++) {
            hist0[m][j] = hist ? hist[(((size_t)b * 3 + m) * P + c) * hl + j] : 0.0f;
            buf[m][j] = hist0[m][j];
        }
        for (int j = 0; j < K; j++) wt[m][j] = w[m][(size_t)c * K + j];
    }
    const float a = expf_cr(A_log[h]);
    for (int t = 0; t < T; t++) {
        const size_t rc = ((size_t)b * T + t) * P + c;
        if (parent) {
            // a draft tree: the window is the node's ancestors (newest first: its parent),
            // then the carried history, as a chain along the node's own path would see it;
            // the ancestors' pre-conv rows were written by this thread at earlier t
            int an = parent[t];
            int hh = hl - 1;
            for (int j = hl - 1; j >= 0; j--) {
                if (an >= 0 && an < t) {
#pragma unroll
                    for (int m = 0; m < 3; m++) buf[m][j] = pre[(((size_t)b * T + an) * 3 + m) * P + c];
                    const int pa = parent[an];
                    if (pa >= an) flag(DEV_BAD_INDEX);
                    an = pa < an ? pa : -1;
                } else {
#pragma unroll
                    for (int m = 0; m < 3; m++) buf[m][j] = hist0[m][hh];
                    hh--;
                    an = -1;
                }
            }
        }
        float y[3];
#pragma unroll
        for (int m = 0; m < 3; m++) {
            const float cur = rows[m][rc];
            pre[(((size_t)b * T + t) * 3 + m) * P + c] = cur;
            // taps oldest..newest, w[K-1] on the current input (k3_ops.c:185-195)
            float acc = __fmul_rn(wt[m][hl], cur);
            for (int j = 0; j < hl; j++) acc = __fadd_rn(acc, __fmul_rn(wt[m][j], buf[m][j]));
            if (!parent) {
                for (int j = 0; j + 1 < hl; j++) buf[m][j] = buf[m][j + 1];
                if (hl > 0) buf[m][hl - 1] = cur;
            }
            y[m] = __fmul_rn(acc, sigmoid_cr(acc));
        }
        // L2 norm of q and k over the head's D channels: SUM of squares, eps 1e-6
        const double sq = block_sum_d((double)y[0] * (double)y[0], red);
        const double sk = block_sum_d((double)y[1] * (double)y[1], red);
        const float iq = __double2float_rn(1.0 / sqrt(sq + 1e-6));
        const float ik = __double2float_rn(1.0 / sqrt(sk + 1e-6));
        q[rc] = __fmul_rn(y[0], iq);
        k[rc] = __fmul_rn(y[1], ik);
        v[rc] = y[2];
        // decay chain, A_log PER HEAD (k3_ops.c:206-221)
        const float u = __fmul_rn(a, __fadd_rn(z[rc], dt_bias[c]));
        const float g = __fmul_rn(lb, sigmoid_cr(u));
        alpha[rc] = expf_cr(g);
        if (d == 0) {
            const size_t bi = ((size_t)b * T + t) * H + h;
            beta[bi] = sigmoid_cr(bproj[bi]);
        }
    }
}

__global__ void kda_commit_conv_kernel(float *__restrict__ hist, const float *__restrict__ pre,
                                       const int *__restrict__ nkeep, int T, int P, int K)
{
    const int b = blockIdx.y;
    const int hl = K - 1;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // over 3*P
    if (idx >= 3LL * P) return;
    const int m = (int)(idx / P), ch = (int)(idx % P);
    int n = nkeep[b];
    if (n < 0 || n > T) {
        if (idx == 0) flag(DEV_BAD_COUNT);
        n = n < 0 ? 0 : T;
    }
    float *hc = hist + (((size_t)b * 3 + m) * P + ch) * hl;
    float old[8];
    for (int j = 0; j < hl; j++) old[j] = hc[j];
    for (int j = 0; j < hl; j++) {
        const int i = n + j;
        hc[j] = i < hl ? old[i] : pre[(((size_t)b * T + (i - hl)) * 3 + m) * P + ch];
    }
}

// grid R*H, block D: y = o_norm * o * inv (double sum of squares), then * sigmoid(gate).
__global__ void __launch_bounds__(256) kda_norm_gate_kernel(float *__restrict__ o,
                                                           const float *__restrict__ gate,
                                                           const float *__restrict__ w,
                                                           int D, float eps)
{
    __shared__ double red[32];
    const size_t row = blockIdx.x;
    const int d = threadIdx.x;
    const float x = o[row * D + d];
    const double ss = block_sum_d((double)x * (double)x, red);
    const float inv = __double2float_rn(1.0 / sqrt(ss / (double)D + (double)eps));
    const float y = __fmul_rn(__fmul_rn(w[d], x), inv);
    o[row * D + d] = __fmul_rn(y, sigmoid_cr(gate[row * D + d]));
}

}  // namespace k3

#define K3_KDA_DISPATCH(D, KERNEL, ...)                                                   \
    switch (D) {                                                                          \
    case 16: k3::KERNEL<16><<<grid, 16, 0, s>>>(__VA_ARGS__); break;                       \
    case 32: k3::KERNEL<32><<<grid, 32, 0, s>>>(__VA_ARGS__); break;                       \
    case 64: k3::KERNEL<64><<<grid, 64, 0, s>>>(__VA_ARGS__); break;                       \
    case 128: k3::KERNEL<128><<<grid, 128, 0, s>>>(__VA_ARGS__); break;                    \
    default: return K3GPU_EINVAL;                                                         \
    }

static bool kda_dim_ok(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

extern "C" int k3gpu_kda_verify(float *o, const float *state, const float *q, const float *k,
                                const float *v, const float *alpha, const float *beta, int B,
                                int T, int H, int D, float qscale, void *stream)
{
    if (!o || !state || !q || !k || !v || !alpha || !beta) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || H <= 0 || H > 65535 || B > 65535 || !kda_dim_ok(D))
        return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    dim3 grid(H, B);
    K3_KDA_DISPATCH(D, kda_verify_kernel, o, state, q, k, v, alpha, beta, T, H, qscale);
    return k3::launch_status();
}

extern "C" int k3gpu_kda_verify_tree(float *o, const float *state, const float *q, const float *k,
                                     const float *v, const float *alpha, const float *beta, const int *parent,
                                     int B, int T, int H, int D, float qscale, void *stream)
{
    if (!o || !state || !q || !k || !v || !alpha || !beta || !parent) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || H <= 0 || H > 65535 || B > 65535 || !kda_dim_ok(D))
        return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    dim3 grid(H, B);
    const size_t smem = (size_t)D * D * sizeof(float);   // the parked state columns
    if (D == 128) {   // 64 KB: above the default dynamic shared-memory limit, opted in once per device
        static std::mutex mu;
        static bool done[64] = {};
        int dev = 0;
        int st = k3::cuda_status(cudaGetDevice(&dev));
        if (st) return st;
        if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
        std::lock_guard<std::mutex> lock(mu);
        if (!done[dev]) {
            st = k3::cuda_status(cudaFuncSetAttribute(k3::kda_verify_tree_kernel<128>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (st) return st;
            done[dev] = true;
        }
    }
    switch (D) {
    case 16: k3::kda_verify_tree_kernel<16><<<grid, 16, smem, s>>>(o, state, q, k, v, alpha, beta, parent, T, H, qscale); break;
    case 32: k3::kda_verify_tree_kernel<32><<<grid, 32, smem, s>>>(o, state, q, k, v, alpha, beta, parent, T, H, qscale); break;
    case 64: k3::kda_verify_tree_kernel<64><<<grid, 64, smem, s>>>(o, state, q, k, v, alpha, beta, parent, T, H, qscale); break;
    default: k3::kda_verify_tree_kernel<128><<<grid, 128, smem, s>>>(o, state, q, k, v, alpha, beta, parent, T, H, qscale); break;
    }
    return k3::launch_status();
}

extern "C" int k3gpu_kda_commit(float *state, const float *k, const float *v,
                                const float *alpha, const float *beta, const int *n, int B,
                                int T, int H, int D, void *stream)
{
    if (!state || !k || !v || !alpha || !beta || !n) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || T > 64 || H <= 0 || H > 65535 || B > 65535 || !kda_dim_ok(D))
        return K3GPU_EINVAL;
    cudaStream_t s = k3::as_stream(stream);
    dim3 grid(H, B);
    K3_KDA_DISPATCH(D, kda_commit_kernel, state, k, v, alpha, beta, n, T, H);
    return k3::launch_status();
}

extern "C" int k3gpu_kda_prologue_tree(float *q, float *k, float *v, float *alpha, float *beta,
                                       float *pre, const float *z, const float *b,
                                       const float *q_conv, const float *k_conv,
                                       const float *v_conv, const float *hist, const float *A_log,
                                       const float *dt_bias, const int *parent, int B, int T, int H,
                                       int D, int K, float lb, void *stream)
{
    if (!q || !k || !v || !alpha || !beta || !pre || !z || !b || !q_conv || !k_conv ||
        !v_conv || !A_log || !dt_bias)
        return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || H <= 0 || D < 32 || D > 256 || D % 32 || K < 2 || K > 8 ||
        H > 65535 || B > 65535)
        return K3GPU_EINVAL;
    dim3 grid(H, B);
    k3::kda_prologue_kernel<<<grid, D, 0, k3::as_stream(stream)>>>(
        q, k, v, alpha, beta, pre, z, b, q_conv, k_conv, v_conv, hist, A_log, dt_bias, T, H, D,
        K, lb, parent);
    return k3::launch_status();
}

extern "C" int k3gpu_kda_prologue(float *q, float *k, float *v, float *alpha, float *beta,
                                  float *pre, const float *z, const float *b,
                                  const float *q_conv, const float *k_conv,
                                  const float *v_conv, const float *hist, const float *A_log,
                                  const float *dt_bias, int B, int T, int H, int D, int K,
                                  float lb, void *stream)
{
    return k3gpu_kda_prologue_tree(q, k, v, alpha, beta, pre, z, b, q_conv, k_conv, v_conv, hist, A_log,
                                   dt_bias, nullptr, B, T, H, D, K, lb, stream);
}

extern "C" int k3gpu_kda_commit_conv(float *hist, const float *pre, const int *n, int B, int T,
                                     int H, int D, int K, void *stream)
{
    if (!hist || !pre || !n) return K3GPU_EINVAL;
    if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || K < 2 || K > 8 || B > 65535) return K3GPU_EINVAL;
    const int P = H * D;
    dim3 grid(k3::ceil_div(3LL * P, 256), B);
    k3::kda_commit_conv_kernel<<<grid, 256, 0, k3::as_stream(stream)>>>(hist, pre, n, T, P, K);
    return k3::launch_status();
}

extern "C" int k3gpu_kda_norm_gate(float *o, const float *gate, const float *o_norm, int R,
                                   int H, int D, float eps, void *stream)
{
    if (!o || !gate || !o_norm) return K3GPU_EINVAL;
    if (R <= 0 || H <= 0 || D < 32 || D > 256 || D % 32) return K3GPU_EINVAL;
    k3::kda_norm_gate_kernel<<<(unsigned)((long long)R * H), D, 0, k3::as_stream(stream)>>>(
        o, gate, o_norm, D, eps);
    return k3::launch_status();
}
