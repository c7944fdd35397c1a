/* k3gpu.h -- the C ABI of the B200 speculative-verification library (libk3gpu.so).
 *
 * This is the drop-in boundary between the reference engine's C99 host (its k3_* API,
 * include/k3/k3.h of andrewd780/kimi-k3-for-me, and its CLI's verify sweep,
 * src/cli/k3_run.c:2860-2966) and hand-written sm_100a CUDA kernels. Each entry point
 * names the reference function it replaces (file:line in the reference tree).
 *
 * Conventions, for every k3gpu_* function that takes a `stream`:
 *   - pointers are DEVICE pointers unless the comment says "host";
 *   - `stream` is a cudaStream_t passed as void * (NULL = the legacy default stream), so
 *     this header needs no CUDA include; work is enqueued, never synchronised, unless the
 *     comment says otherwise;
 *   - the return value is a status: K3GPU_OK, or a negative code. Arguments are checked
 *     on the host before anything is enqueued; a failed check enqueues nothing and
 *     leaves every output untouched. Nothing aborts and nothing traps on the device:
 *     where a kernel itself detects a bad index it records it in the library's device
 *     status word (k3gpu_device_status) and skips the access;
 *   - all buffers, scratch included, are caller-owned; *_workspace() returns the bytes
 *     a call needs (the reference's own ownership rule, docs/API.md:47-64, with
 *     k3_*_scratch() sizing);
 *   - calls are reentrant; concurrent calls on different streams must not share a
 *     workspace.
 */
#ifndef K3GPU_H
#define K3GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status ---- */
enum {
    K3GPU_OK = 0,
    K3GPU_EINVAL = -1,     /* null pointer, size out of range, misaligned buffer        */
    K3GPU_ECAPACITY = -2,  /* workspace, log or cache capacity too small                */
    K3GPU_ECUDA = -3,      /* a CUDA launch/runtime error; see k3gpu_last_cuda_error()  */
    K3GPU_EDEVICE = -4,    /* a device-side check failed; see k3gpu_device_status()     */
    K3GPU_ECALLBACK = -5   /* a caller-supplied callback returned non-zero              */
};

const char *k3gpu_strerror(int status);
/* The cudaError_t behind the last K3GPU_ECUDA returned on this thread. */
int k3gpu_last_cuda_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int k3gpu_version(void);
/* Kernels this process has enqueued through the library so far (all threads, all
 * devices): the difference across a region is the number of the library's launches in it. */
long long k3gpu_launch_count(void);
/* Read (host, synchronous on the given device's default stream) and clear the device
 * status word: 0 when no kernel has flagged an out-of-range index since the last call.
 * Bits: 1 an index outside its range was skipped, 2 a count outside its range was
 * clamped, 4 a cache position outside its range was skipped, 8 a bounded device wait
 * ran out. */
int k3gpu_device_status(int device, int *status_out);

/* ------------------------------------------------------------------ router ---- */
/* Replaces k3_router (include/k3/k3.h:311-313, src/core/k3_ops.c:1624-1719) for T tokens
 * in one call. x [T][hidden] fp32, W [n_experts][hidden] fp32 row-major, bias
 * [n_experts] fp32 or NULL -> idx [T][topk] int32 and w [T][topk] fp32 in descending
 * selection order. Same arithmetic as the reference: one double chain per (token,
 * expert) in ascending i, score = 1/(1+exp(-(float)acc)) with a correctly rounded exp,
 * selection on score+bias by repeated max with first-index ties, weights from the
 * UNBIASED scores, double renormaliser 1/(sum+1e-20) rounded to float, * routed_scale.
 * Limits: 1 <= topk <= 64, topk <= n_experts <= 1024, hidden >= 1. The workspace holds
 * the [T][n_experts] scores (k3gpu_router_workspace bytes). */
size_t k3gpu_router_workspace(int T, int n_experts);
int k3gpu_router(int *idx, float *w, const float *x, const float *W, const float *bias,
                 int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                 void *workspace, size_t ws_bytes, void *stream);

/* The router for callers that cannot allocate device memory. No counterpart in the
 * reference (its k3_router mallocs its score arrays on the host per call); this entry
 * point exists for hosts that own all device memory up front -- a serving process whose
 * allocator has already reserved the HBM, or a caller on a latency-critical thread where
 * cudaMalloc, which may synchronise the device, is not allowed -- and so cannot provide
 * the workspace k3gpu_router needs. Same inputs, outputs and arithmetic as
 * k3gpu_router; the [T][n_experts] scores live instead in a fixed array inside the
 * library (K3GPU_ROUTER_NOALLOC_MAX_SCORES floats, 2 MiB, held by every GPU that loads
 * the library until the process exits).
 *   - T * n_experts above the maximum returns K3GPU_ECAPACITY and enqueues nothing.
 *   - The first call on a device looks up that device's copy of the array (set-up, once
 *     per device); make that first call before any stream capture. After a device reset
 *     (cudaDeviceReset) the array has a new address: the next call on that device sees
 *     the new context and repeats the set-up, so make it before any capture too.
 *   - Every call shares the one array: two calls whose kernels overlap on the same GPU
 *     (different streams, or host threads) race and may return wrong results. Calls on
 *     one stream are ordered and safe. Nothing in the array needs clearing: each call
 *     writes every score it reads before reading it.
 * It allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine. */
#define K3GPU_ROUTER_NOALLOC_MAX_SCORES 524288
int k3gpu_router_noalloc(int *idx, float *w, const float *x, const float *W,
                         const float *bias, int T, int hidden, int n_experts, int topk,
                         int renorm, float routed_scale, void *stream);

/* ------------------------------------------------------------ expert bank ---- */
/* Device-resident MXFP4 experts. Expert e is the byte run base + e*stride holding, at
 * the given offsets, the six tensors the reference's loader reads as one contiguous run
 * (src/io/k3_load.h:1-22; K3ExpertQ, include/k3/k3.h:512-516):
 *   p1 [I][L/2]  s1 [I][L/32]   w1, gate    (low nibble = EVEN element, E8M0 per 32)
 *   p2 [L][I/2]  s2 [L][I/32]   w2, down
 *   p3 [I][L/2]  s3 [I][L/32]   w3, up
 * Runs n_routed .. n_routed+n_shared-1 are the shared experts. L and I are multiples of
 * 32; base, stride and every offset are multiples of 16 bytes. */
typedef struct {
    const uint8_t *base;
    int64_t stride;
    int64_t p1, s1, p2, s2, p3, s3;
    int n_experts;          /* runs in the bank: routed + shared */
    int L, I;               /* expert input/output width, intermediate width */
    /* Filled by k3gpu_bank_scan (NULL / 0 until then): a device array [n_experts], 1 where
     * every E8M0 byte of the expert lies in 104..140 (or is the NaN byte 255), so that
     * scale * E2M1 is exact in f16 and the expert can run on the tcgen05 kernels; and the
     * number of experts that are not. */
    const uint8_t *f16_safe;
    int n_f16_unsafe;
} K3GpuExpertBank;

/* One-time certification of a bank for the tcgen05 expert kernels (host, synchronous on
 * `stream`): writes safe_dev [n_experts] (device) and sets bank->f16_safe and
 * bank->n_f16_unsafe. Experts that fail the check keep running on the mma.sync kernels;
 * a bank never scanned runs entirely on those. */
int k3gpu_bank_scan(K3GpuExpertBank *bank, uint8_t *safe_dev, void *stream);

/* Host C: routed experts [e0, e0 + n) of MoE layer `layer` from the checkpoint's
 * safetensors shards (files: the shard paths, any order; the format of the reference's
 * src/io/k3_st.h:7-13) into host_bank laid out as this bank (k3gpu_bank_layout(L, I): run
 * e - e0 at (e - e0) * stride), ready for one copy to the device. Reads the six U8 tensors
 * language_model.model.layers.<layer>.block_sparse_moe.experts.<e>.<w1|w2|w3>.<weight_packed|
 * weight_scale> (src/io/k3_load.c:11) after checking their dtype and shapes ([I][L/2],
 * [I][L/32] for w1 and w3; [L][I/2], [L][I/32] for w2). K3GPU_EINVAL for a missing,
 * mis-shaped or unreadable tensor or a malformed header, K3GPU_ECAPACITY when host_bytes
 * is short of n * stride. */
/* Host C: a tensor index over a checkpoint's safetensors shards, the reference's
 * k3_st_open / k3_st_find / k3_st_read (src/io/k3_st.h:60-80) for any tensor -- the
 * trunk's bf16 and fp32 weights as well as the experts' U8 runs. Open reads every
 * shard's header once (the reference's open takes a directory: every *.safetensors in
 * it, by name; k3_st_open_files takes the paths); a malformed header, data past a file's
 * end or a tensor name appearing twice in the set fails the open (NULL). Find is O(1);
 * read copies the raw stored bytes with pread. Dtype codes are the reference's K3Dtype
 * (src/io/k3_st.h:36-37). */
enum { K3_ST_UNKNOWN = 0, K3_ST_U8 = 1, K3_ST_BF16 = 2, K3_ST_F16 = 3, K3_ST_F32 = 4 };
typedef struct K3StIndex K3StIndex;
typedef struct K3StTensorInfo {
    int dtype;                 /* K3_ST_*; K3_ST_UNKNOWN for any other dtype string */
    char dtype_name[16];       /* the header's dtype string, NUL-terminated          */
    int ndim;                  /* <= 8                                               */
    int64_t shape[8];
    int shard;                 /* index of the file holding it                       */
    int64_t nbytes;
} K3StTensorInfo;
K3StIndex *k3_st_open(const char *dir);
K3StIndex *k3_st_open_files(const char *const *files, int n_files);
void k3_st_close(K3StIndex *s);
/* the indexed tensors (metadata excluded), shard by shard in header order */
int k3_st_count(const K3StIndex *s);
const char *k3_st_name(const K3StIndex *s, int i);
/* K3GPU_OK, or K3GPU_EINVAL for an absent name (a missing weight must stop a load). */
int k3_st_find(const K3StIndex *s, const char *name, K3StTensorInfo *info);
/* bytes read (the tensor's nbytes), K3GPU_EINVAL (absent, unreadable) or
 * K3GPU_ECAPACITY (buf_bytes short of nbytes). */
int64_t k3_st_read(const K3StIndex *s, const char *name, void *buf, size_t buf_bytes);

int k3_bank_read_safetensors(const char *const *files, int n_files, int layer, int e0, int n,
                             int L, int I, uint8_t *host_bank, size_t host_bytes);

/* Fill the offsets and stride of the packed run layout above (the stride is the run
 * rounded up to a multiple of lcm(L/2, I/2, 256) bytes, so every matrix starts on a whole
 * row of the expert kernels' tensor maps); leaves base and n_experts to the caller.
 * Host only. */
void k3gpu_bank_layout(K3GpuExpertBank *bank, int L, int I);

/* Replaces k3_mxfp4_dequant (include/k3/k3.h:863-864) for group 32: out [rows][in] fp32
 * from packed [rows][in/2] and scales [rows][in/32]; the same nibble decode and E8M0
 * scaling the expert kernels apply in registers (exact: no rounding anywhere).
 * in % 32 == 0; packed 16-byte aligned. */
int k3gpu_mxfp4_dequant(float *out, const uint8_t *packed, const uint8_t *scales, int rows,
                        int in, void *stream);

/* Activation of the expert FFN, applied to [gate | up]. */
enum { K3GPU_ACT_SITU = 0, K3GPU_ACT_SWIGLU = 1 };

/* ------------------------------------------------------------------- MoE ----- */
/* Workspace bytes for k3gpu_moe_experts / k3gpu_moe_layer. */
size_t k3gpu_moe_workspace(int T, int topk, int n_shared, int L, int I, int n_routed);

/* Replaces the routed half of k3_moe_prefill (src/core/k3_ops.c:2058-2132) plus the
 * shared experts, on device-resident MXFP4 experts. z [T][L] fp32 expert inputs,
 * idx/wt [T][topk] from k3gpu_router -> out [T][L] fp32:
 *   out[t] = RMSNorm?( sum_j wt[t][j] * expert_{idx[t][j]}(z[t]) )  (sum in top-k order)
 *          + sum_s shared_s(z[t])                                     (unweighted)
 * expert(z) = W2 . act(W1 z, W3 z). latent_norm [L] or NULL skips the RMSNorm (eps).
 * idx < 0 drops that slot, as the reference does for a failed expert. b1, b2 are the
 * SiTU caps (ignored for SwiGLU). Each unique expert's weights are read once per call.
 * Limits: T*(topk+n_shared) <= 1<<20, n_routed+n_shared == bank->n_experts <= 4096. */
int k3gpu_moe_experts(float *out, const float *z, const int *idx, const float *wt,
                      const K3GpuExpertBank *bank, int T, int topk, int n_routed,
                      int n_shared, int act, float b1, float b2, const float *latent_norm,
                      float eps, void *workspace, size_t ws_bytes, void *stream);

/* One MoE layer of the single-layer verify configuration (no latent projections, so
 * L == hidden): k3gpu_router on x, then k3gpu_moe_experts with z = x and no latent
 * norm. idx/wt [T][topk] receive the routing decisions. */
int k3gpu_moe_layer(float *out, int *idx, float *wt, const float *x, const float *gate_W,
                    const float *bias, const K3GpuExpertBank *bank, int T, int topk,
                    int n_routed, int n_shared, int act, float b1, float b2, int renorm,
                    float routed_scale, void *workspace, size_t ws_bytes, void *stream);

/* Expert-kernel selection (host, per process): 0 (default) runs the tensor-core expert
 * stream wherever L and I are multiples of 512 and the CUDA-core stream elsewhere, the
 * tcgen05 kernels in the pass shape the call's routed tokens per expert select (8 tokens a
 * pass while experts see few, 32 once they see 12 or more on average); 1 forces the
 * CUDA-core stream everywhere; 2 and 3 force the tcgen05 dense (32-token) and sparse
 * (8-token) pass shapes. All agree to fp32 rounding. */
int k3gpu_moe_select_kernels(int which);

/* Per-phase timing of the MoE calls, for roofline reporting. When enabled (host, per
 * process), every k3gpu_moe_experts / k3gpu_moe_layer call records CUDA events on its
 * stream around its kernels; k3gpu_moe_phase_ms then waits for the last call and writes
 * the device milliseconds of its phases into ms[0..n): 0 router (0 for
 * k3gpu_moe_experts), 1 plan, 2 gate/up expert stream, 3 down expert stream, 4 combine.
 * Returns the number written. Not for concurrent calls. */
int k3gpu_moe_phase_timing(int enable);
int k3gpu_moe_phase_ms(float *ms, int n);

/* --------------------------------------------------------------------- KDA ----- */
/* The KDA recurrence of a tentative verify sweep, k3_kda_layer_log's step 6
 * (src/core/k3_ops.c:2342-2364) for B sequences. state [B][H][D][D] fp32 is READ ONLY
 * (the sweep never touches the carried state; include/k3/k3.h:662-700). q, k, v, alpha
 * [B][T][H][D], beta [B][T][H] -> o [B][T][H][D]; q is multiplied by qscale in float
 * first. Bit-identical to k3_kda_step chained over t (same float operations in the same
 * order, zero rows of k and q skipped as the reference skips them). The operands k, v,
 * alpha, beta ARE the log a commit replays. D in {16, 32, 64, 128}; 1 <= T <= 64. */
int k3gpu_kda_verify(float *o, const float *state, const float *q, const float *k,
                     const float *v, const float *alpha, const float *beta, int B, int T,
                     int H, int D, float qscale, void *stream);

/* Replaces k3_kda_advance's recurrence (src/core/k3_ops.c:2391-2409): commit the first
 * n[b] logged positions of sequence b into state[b] in place, bit-identical to feeding
 * those positions alone. n is a DEVICE array [B] (so an on-device accept can feed it
 * without a host round trip); entries outside 0..T are clamped to that range and
 * flagged in the device status word. The log operands are those given to
 * k3gpu_kda_verify, [B][T][H][D] (beta [B][T][H]). */
/* A prompt's positions read into the carried state in one launch: the KDA recurrence in
 * its chunked (UT-transform) form, 32 positions per chunk, for B sequences of T positions
 * (any T >= 1). state [B][H][D][D] is updated in place to the state after position T-1;
 * o [B][T][H][D] (may be NULL) receives the outputs; q, k, v, alpha [B][T][H][D], beta
 * [B][T][H]; q is multiplied by qscale first. Equal to k3_kda_step chained over t to
 * fp32 rounding (the sums are reordered). D in {32, 64, 128}. The reference has no
 * chunked path (include/k3/k3.h:51-60); it reads prompts with the sequential step. */
int k3gpu_kda_prefill(float *state, float *o, const float *q, const float *k, const float *v,
                      const float *alpha, const float *beta, int B, int T, int H, int D, float qscale,
                      void *stream);

int k3gpu_kda_commit(float *state, const float *k, const float *v, const float *alpha,
                     const float *beta, const int *n, int B, int T, int H, int D,
                     void *stream);

/* k3gpu_kda_verify over a draft TREE of T nodes (no counterpart in the reference, whose
 * sweeps are chains): parent DEVICE [T] (parent[0] = -1, parent[t] < t), one tree shape for
 * the B sequences. Node t reads the state after its own ancestors -- the chain of
 * k3_kda_step over root .. t on the read-only carried state, recomputed per node with the
 * chain's float operations, so each output is bit-identical to a chain verify of the
 * node's path. Committing an accepted path: gather its log rows to the front, then
 * k3gpu_kda_commit / k3gpu_kda_commit_conv with n = the path length. */
int k3gpu_kda_verify_tree(float *o, const float *state, const float *q, const float *k,
                          const float *v, const float *alpha, const float *beta, const int *parent,
                          int B, int T, int H, int D, float qscale, void *stream);

/* The KDA prologue, src/core/k3_ops.c:2286-2303 for B sequences: from the projection
 * outputs q, k, v [B][T][P] (P = H*D), z [B][T][P] (f_b output, before dt_bias) and
 * b [B][T][H], with the carried ShortConv history hist [B][3][P][K-1] (read only):
 * ShortConv+SiLU on q, k, v in place, L2 norm of q and k per head (sum of squares in
 * double, eps 1e-6), alpha = exp(lb*sigmoid(exp(A_log[h])*(z+dt_bias))) [B][T][P] and
 * beta = sigmoid(b) [B][T][H]. pre [B][T][3][P] receives the PRE-conv q, k, v, the rows
 * the conv-history commit replays (K3KdaLog rows, include/k3/k3.h:716-724).
 * 2 <= K <= 8. */
int k3gpu_kda_prologue(float *q, float *k, float *v, float *alpha, float *beta, float *pre,
                       const float *z, const float *b, const float *q_conv,
                       const float *k_conv, const float *v_conv, const float *hist,
                       const float *A_log, const float *dt_bias, int B, int T, int H, int D,
                       int K, float lb, void *stream);

/* k3gpu_kda_prologue over a draft tree (parent DEVICE [T], as k3gpu_kda_verify_tree; NULL:
 * the chain): each node's ShortConv window is its ancestors' pre-conv rows (its parent
 * newest) and then the carried history. */
int k3gpu_kda_prologue_tree(float *q, float *k, float *v, float *alpha, float *beta, float *pre,
                            const float *z, const float *b, const float *q_conv,
                            const float *k_conv, const float *v_conv, const float *hist,
                            const float *A_log, const float *dt_bias, const int *parent, int B,
                            int T, int H, int D, int K, float lb, void *stream);

/* Replaces kda_replay_conv_ (src/core/k3_ops.c:2207-2223): advance the ShortConv history
 * hist [B][3][P][K-1] in place by the first n[b] pre-conv rows of pre [B][T][3][P].
 * n is a device array [B], clamped to 0..T. */
int k3gpu_kda_commit_conv(float *hist, const float *pre, const int *n, int B, int T, int H,
                          int D, int K, void *stream);

/* src/core/k3_ops.c:2375-2379: per-head RMSNorm over D (double sum) then the sigmoid
 * gate, in place on o [R][H][D] with gate [R][H*D], R = B*T rows. */
int k3gpu_kda_norm_gate(float *o, const float *gate, const float *o_norm, int R, int H,
                        int D, float eps, void *stream);

/* --------------------------------------------------------------------- MLA ----- */
/* Workspace bytes for k3gpu_mla_absorbed. */
size_t k3gpu_mla_workspace(int B, int T, int H, int kv_lora, int max_ctx);

/* Absorbed MLA over the compressed cache with a chain or tree mask, the --mla-absorb
 * branch of k3_mla_cached (src/core/k3_ops.c:1417-1540) for B sequences of T query
 * nodes each:
 *   q_abs[h] = W_uk[h]^T q_nope[h]
 *   score[s] = scale * (q_abs[h] . lat[s] + q_rope[h] . rope[s])   for visible s
 *   u[h]     = sum_s softmax(score)[s] * lat[s]
 *   out[h]   = W_uv[h] u[h]
 * q_nope [B][T][H][qk_nope], q_rope [B][T][H][qk_rope] fp32; kv_b [H*(qk_nope+v_head)]
 * [kv_lora] fp32 (the reference's kv_b rows: key rows then value rows per head);
 * lat [B][cap][kv_lora] and rope [B][cap][qk_rope] bf16 (uint16 bit patterns) hold
 * positions 0..cached[b]+T-1 (the T new rows already appended at cached[b]..);
 * cached is a DEVICE array [B]; mask [T] uint64 (host-side meaning, device array):
 * query t sees every row below cached[b] and new row j iff bit j of mask[t] is set
 * (chain: bits 0..t; tree: the node's ancestors and itself). out [B][T][H][v_head] fp32
 * is the attention output before the output gate. T <= 64, kv_lora in {128, 256, 512},
 * qk_rope <= 64 (q_rope and rope may be NULL when it is 0), qk_nope and v_head <= 256.
 * kv_lora in {128, 256, 512} with qk_rope in {0, 64} and 16-byte aligned lat/rope run on
 * the tensor cores (tcgen05); other shapes on a CUDA-core kernel. */
int k3gpu_mla_absorbed(float *out, const float *q_nope, const float *q_rope,
                       const float *kv_b, const uint16_t *lat, const uint16_t *rope,
                       const int *cached, const uint64_t *mask, int B, int T, int H,
                       int qk_nope, int qk_rope, int v_head, int kv_lora, int cap,
                       int max_ctx, float scale, void *workspace, size_t ws_bytes,
                       void *stream);

/* ----------------------------------------------------------------- accept ------ */
/* The greedy verify-and-accept of the CLI's sweep (src/cli/k3_run.c:2924-2928 with
 * argmax_ :138-139) for B sequences on the device: arg[b][i] = first index of the
 * maximum of logits [B][nd+1][vocab]; m = longest prefix with arg[b][i] == d[b][i]
 * (drafts [B][nd]); emit[b][0..m) = d, emit[b][m] = arg[b][m] (the bonus token);
 * n_emit[b] = m + 1. nd_b [B] (device, may be NULL = nd for all) limits each sequence's
 * draft count. emit/arg are [B][nd+1]. logits may be NULL when arg already holds every
 * position's argmax (k3gpu_model_verify_greedy). */
int k3gpu_accept_greedy(int *emit, int *n_emit, int *arg, const float *logits,
                        const int *drafts, const int *nd_b, int B, int nd, int vocab,
                        void *stream);

/* argmax_ (src/cli/k3_run.c:138-139) per row: arg [rows] = first index of the maximum of
 * logits [rows][vocab] over non-NaN values (0 when logits[row][0] is NaN). */
int k3gpu_argmax(int *arg, const float *logits, int rows, int vocab, void *stream);

/* Greedy acceptance over a draft TREE of T nodes (node 0 = the pending token, parent[0]
 * = -1, parent[i] < i; tok[i] the drafted id of node i, tok[0] unused). A child i is
 * accepted when its parent is accepted and tok[i] == argmax of the parent's logits;
 * among accepted children of one node the lowest index wins. The accepted path is
 * emitted in order, then the bonus argmax of its last node. logits [B][T][vocab];
 * parent/tok are device arrays [T] and [B][T]; path [B][T] receives the accepted node
 * indices (root first), emit [B][T] the emitted ids, n_emit [B] their count. logits may be
 * NULL when arg [B][T] already holds every node's argmax (k3gpu_model_verify_greedy). */
int k3gpu_accept_tree_greedy(int *emit, int *n_emit, int *path, int *arg,
                             const float *logits, const int *tok, const int *parent, int B,
                             int T, int vocab, void *stream);

/* Temperature sampling with the speculative rejection rule for point-mass drafts (the
 * n-gram drafter proposes one id per position with probability 1): position i's draft
 * d is accepted with probability p_i(d) = softmax(logits_i / temp)(d), drawn with
 * Philox4x32-10 (Salmon et al., SC'11) keyed by seed and counter (offset, b, i); on the
 * first rejection the replacement is drawn from p_i with d removed and renormalised, and
 * after a full acceptance the bonus is drawn from p_nd. Shapes as k3gpu_accept_greedy.
 * temp > 0. */
int k3gpu_accept_sample(int *emit, int *n_emit, const float *logits, const int *drafts,
                        const int *nd_b, int B, int nd, int vocab, float temp,
                        uint64_t seed, uint64_t offset, void *stream);

/* ------------------------------------------------------- trunk matmul ---------- */
/* Workspace bytes for k3gpu_matmul_bf16_batch (independent of T beyond 256). */
size_t k3gpu_matmul_bf16_workspace(int T, int in, int out);

/* k3_matmul_bf16_batch_ld (src/core/k3_ops.c:953; the k3_mmw_batch_ld bf16 case,
 * include/k3/k3.h:449-484) on tcgen05: Y[t*ldy + o] = sum_i W[o*in + i] * X[t*ldx + i]
 * for t < T, o < out. W bf16 bits [out][in] (16-byte aligned, in % 8 == 0), X fp32, Y fp32;
 * Y must not overlap X. The activations enter the tensor cores as two bf16 pieces
 * (x = hi + lo to 2^-17), the products are exact and the sums fp32, so Y matches the
 * reference's double sums to about 1e-5 relative, not bit for bit. */
int k3gpu_matmul_bf16_batch(float *Y, int ldy, const float *X, int ldx, const uint16_t *W,
                            int in, int out, int T, void *workspace, size_t ws_bytes,
                            void *stream);

/* The lm_head fused with the greedy argmax (the verify sweep's logits and argmax_,
 * src/cli/k3_run.c:1089-1130 and :138-139): arg[t] = first index of the maximum over
 * o < vocab of sum_i W[o*in + i] * X[t*ldx + i] among non-NaN values, 0 when the value at
 * o = 0 is NaN (the sequential scan finds nothing greater than NaN), for t < T, without
 * writing the [T][vocab] logits. The products are those of k3gpu_matmul_bf16_batch run
 * with one K split; each 128-row block's epilogue keeps its best (value, row) per position
 * and a second kernel merges the blocks in order. W bf16 bits [vocab][in] as there. */
size_t k3gpu_lm_head_argmax_workspace(int T, int in, int vocab);
int k3gpu_lm_head_argmax(int *arg, const float *X, int ldx, const uint16_t *W, int in, int vocab, int T,
                         void *workspace, size_t ws_bytes, void *stream);

/* ------------------------------------------------------- norms and AttnRes ------ */
/* k3_rmsnorm (src/core/k3_ops.c:132-140) over T rows: x, y [T][n] (y may be x), w [n];
 * double sum of squares, 1/sqrt(ss/n + eps) rounded to float, y = (w * x) * inv. */
int k3gpu_rmsnorm(float *y, const float *x, const float *w, int T, int n, float eps,
                  void *stream);

/* k3_attn_res (src/core/k3_ops.c:1722-1753) for the T positions of a sweep, with the
 * decoder layer's source stack (src/core/k3_ops.c:2514-2557) read in place: position t's
 * sources are block_residual[t][0..n_blocks[t]) ([T][maxb][n]) and then cur[t] ([T][n]);
 * fold [n] = norm weight * scoring projection; out [T][n]. n_blocks is a device array [T];
 * a count outside 0..maxb is clamped and flagged (device status bit 2). maxb + 1 <= 256.
 * The double sums run as block reductions, so results agree with the reference to an
 * ulp of float. */
int k3gpu_attn_res(float *out, const float *block_residual, const float *cur,
                   const float *fold, const int *n_blocks, int T, int maxb, int n, float eps,
                   void *stream);

/* ------------------------------------------------------------ K3 MoE (latent) ---- */
/* The K3 MoE block (k3_moe_prefill, src/core/k3_ops.c:2008-2053 with moe_shared
 * :1848-1860): routing on the full-width x, the routed MXFP4 experts on the latent
 * down-projection z, their top-k-ordered sum RMS-normalised over the latent, the
 * up-projection, plus the dense bf16 shared expert on x. */
typedef struct {
    int hidden, latent, moe_inter;   /* E, L, I (routed experts: L -> I -> L) */
    int shared_inter;                /* SI = moe_inter * n_shared; 0 = no shared expert */
    int n_routed, topk, act, renorm;
    float routed_scale, situ_b1, situ_b2, rms_eps;
} K3GpuMoeCfg;

/* bf16 [out][in]: down [L][E], up [E][L], sh1, sh3 [SI][E], sh2 [E][SI]; gate_W
 * [n_routed][E] fp32 and gate_bias [n_routed]; latent_norm [L] or NULL; the routed
 * experts' bank at L, I (n_experts == n_routed). */
typedef struct {
    const uint16_t *down, *up, *sh1, *sh3, *sh2;
    const float *gate_W, *gate_bias, *latent_norm;
    const K3GpuExpertBank *bank;
} K3GpuMoeW;

size_t k3gpu_moe_prefill_workspace(const K3GpuMoeCfg *c, int T);

/* out [T][E] = up(RMSNorm(sum_j wt_j expert_j(down(x)))) + sh2(act(sh1 x, sh3 x)) for
 * x [T][E]; idx/wt [T][topk] receive the routing (indices bit-exact). */
int k3gpu_moe_prefill(float *out, int *idx, float *wt, const float *x, const K3GpuMoeW *w,
                      const K3GpuMoeCfg *c, int T, void *workspace, size_t ws_bytes,
                      void *stream);

/* ------------------------------------------------------------ decoder layer ------ */
/* The configuration a layer needs (the K3Cfg fields it reads, include/k3/k3.h). */
typedef struct {
    int hidden;          /* E */
    int kda_heads;       /* H */
    int kda_head_dim;    /* D */
    int conv_k;          /* ShortConv width, 2..8 */
    float gate_lb;       /* KDA decay lower bound */
    float rms_eps;
    int attn_res_block;  /* a layer with layer_idx % attn_res_block == 0 snapshots */
    int max_blocks;      /* maxb: the block_residual stride */
    int n_routed, n_shared, topk, moe_inter, act, renorm;
    float routed_scale, situ_b1, situ_b2;
    int latent, shared_inter;   /* the K3 MoE form (K3GpuKdaLayerW.moe): L and SI */
    /* MLA layers (K3Cfg n_heads, q_lora, kv_lora, qk_nope, qk_rope, v_head) */
    int mla_heads, q_lora, kv_lora, qk_nope, qk_rope, v_head;
} K3GpuLayerCfg;

/* KDA weights (K3KdaW, include/k3/k3.h): projections bf16 [out][in]; q, k, v, g: [P][E];
 * b: [H][E]; f_a: [D][E]; f_b: [P][D]; o: [E][P] (P = H*D). q_conv, k_conv, v_conv
 * [P][K]; A_log [H]; dt_bias [P]; o_norm [D]. All device pointers. */
typedef struct {
    const uint16_t *q, *k, *v, *b, *f_a, *f_b, *g, *o;
    const float *q_conv, *k_conv, *v_conv, *A_log, *dt_bias, *o_norm;
} K3GpuKdaW;

/* The log of a tentative KDA sweep (K3KdaLog, include/k3/k3.h:716-732, as arrays): the
 * layer writes the recurrence operands k, v, alpha [B][T][P], beta [B][T][H] and the
 * pre-conv rows pre [B][T][3][P]; k3gpu_kda_commit / k3gpu_kda_commit_conv replay them. */
typedef struct {
    float *k, *v, *alpha, *beta, *pre;
} K3GpuKdaLog;

/* A KDA + MoE decoder layer (K3LayerW): the AttnRes folds [E] (norm weight times
 * scoring projection, folded at load as the reference does per call,
 * src/core/k3_ops.c:2504-2507), the input and post norms [E], the KDA weights, and the
 * MoE in its single-layer form (router gate_W [n_routed][E], gate_bias [n_routed]; the
 * expert bank at L = E, I = moe_inter, routed then shared) or, with moe set, the K3 form. */
typedef struct {
    const float *attn_res_fold, *mlp_res_fold, *in_norm, *post_norm;
    K3GpuKdaW kda;
    const float *gate_W, *gate_bias;
    const K3GpuExpertBank *bank;
    const K3GpuMoeW *moe;   /* non-NULL: the K3 MoE form (latent, k3gpu_moe_prefill) instead */
} K3GpuKdaLayerW;

size_t k3gpu_kda_layer_workspace(const K3GpuLayerCfg *c, int B, int T);

/* MLA weights (K3MlaW, include/k3/k3.h): projections bf16 [out][in]: q_a [q_lora][E],
 * q_b [H*(qk_nope+qk_rope)][q_lora], kv_a [kv_lora+qk_rope][E], g [H*v_head][E] (NULL: no
 * output gate), o [E][H*v_head]; norms q_a_norm [q_lora], kv_a_norm [kv_lora] fp32; kv_b
 * [H*(qk_nope+v_head)][kv_lora] fp32 (the absorbed attention reads its key and value rows
 * whole, widened once at load). All device pointers. */
typedef struct {
    const uint16_t *q_a, *q_b, *kv_a, *g, *o;
    const float *q_a_norm, *kv_a_norm, *kv_b;
} K3GpuMlaW;

size_t k3gpu_mla_layer_workspace(const K3GpuLayerCfg *c, int B, int T, int max_ctx);

/* k3_mla_cached (src/core/k3_ops.c:1115-1615; the --mla-absorb latent layout) for B
 * sequences of T query nodes, x [B*T][E] -> out [B*T][E]: q_a, its RMSNorm, q_b; kv_a, the
 * RMSNorm of its latent part; the new rows (latent, then the unrotated rope slot) appended
 * to the bf16 caches lat [B][cap][kv_lora] and rope [B][cap][qk_rope] at positions
 * cached[b] + t; absorbed attention with the node masks (k3gpu_mla_absorbed, scale
 * (qk_nope+qk_rope)^-1/2); the sigmoid gate g x, then o. cached [B] and mask [T] are device
 * arrays; cached[b] + T <= max_ctx <= cap. A verify sweep writes its T rows where the
 * reference writes them; the accepted ones are already in place for a chain, and a tree's
 * accepted path is compacted by the caller before the next sweep. */
int k3gpu_mla_layer_verify(float *out, const float *x, const K3GpuMlaW *w, const K3GpuLayerCfg *c,
                           uint16_t *lat, uint16_t *rope, int cap, const int *cached,
                           const uint64_t *mask, int max_ctx, int B, int T, void *workspace,
                           size_t ws_bytes, void *stream);

/* k3_kda_layer_log (src/core/k3_ops.c:2231-2385) for B sequences of T positions:
 * x [B*T][E] -> out [B*T][E]. state [B][H][D][D] and conv_hist [B][3][P][K-1] are the
 * carried state, read only (the sweep is tentative); the log receives the operands a
 * commit replays. Projections run on k3gpu_matmul_bf16_batch (agreement ~1e-5 relative);
 * the recurrence is bit-identical to the reference's kernel on the same operands. */
int k3gpu_kda_layer_verify(float *out, const float *x, const K3GpuKdaW *w,
                           const K3GpuLayerCfg *c, const float *state, const float *conv_hist,
                           const K3GpuKdaLog *log, int B, int T, void *workspace,
                           size_t ws_bytes, void *stream);

/* k3gpu_kda_layer_verify over a draft tree of T nodes (parent DEVICE [T]; NULL: a chain):
 * the ShortConv and the recurrence follow each node's ancestors. */
int k3gpu_kda_layer_verify_tree(float *out, const float *x, const K3GpuKdaW *w,
                                const K3GpuLayerCfg *c, const float *state, const float *conv_hist,
                                const K3GpuKdaLog *log, const int *parent, int B, int T,
                                void *workspace, size_t ws_bytes, void *stream);

size_t k3gpu_decoder_layer_workspace(const K3GpuLayerCfg *c, int B, int T);

/* k3_decoder_layer_inc_log (src/core/k3_ops.c:2594-2602 -> core :2485-2592) for a KDA +
 * MoE layer over B sequences of T positions, in place on h [B*T][E]: AttnRes before
 * attention over block_residual [B*T][max_blocks][E] with per-position counts n_blocks
 * [B*T] (device); on a block-boundary layer the running residual is snapshotted and
 * n_blocks incremented on the device; input RMSNorm, the KDA layer (tentative, logged),
 * AttnRes before the MLP, post RMSNorm, the MoE layer (moe_idx/moe_wt [B*T][topk]
 * receive the routing), and the residual. */
int k3gpu_decoder_layer_kda_verify(float *h, float *block_residual, int *n_blocks, int *moe_idx,
                                   float *moe_wt, const K3GpuKdaLayerW *w,
                                   const K3GpuLayerCfg *c, int layer_idx, const float *state,
                                   const float *conv_hist, const K3GpuKdaLog *log, int B, int T,
                                   void *workspace, size_t ws_bytes, void *stream);

/* k3gpu_decoder_layer_kda_verify over a draft tree (parent DEVICE [T]; NULL: a chain). */
int k3gpu_decoder_layer_kda_verify_tree(float *h, float *block_residual, int *n_blocks, int *moe_idx,
                                        float *moe_wt, const K3GpuKdaLayerW *w,
                                        const K3GpuLayerCfg *c, int layer_idx, const float *state,
                                        const float *conv_hist, const K3GpuKdaLog *log,
                                        const int *parent, int B, int T, void *workspace,
                                        size_t ws_bytes, void *stream);

/* An MLA + MoE decoder layer (K3LayerW with an MLA block): as K3GpuKdaLayerW with the MLA
 * weights in place of the KDA ones. */
typedef struct {
    const float *attn_res_fold, *mlp_res_fold, *in_norm, *post_norm;
    K3GpuMlaW mla;
    const float *gate_W, *gate_bias;
    const K3GpuExpertBank *bank;
    const K3GpuMoeW *moe;
} K3GpuMlaLayerW;

size_t k3gpu_decoder_layer_mla_workspace(const K3GpuLayerCfg *c, int B, int T, int max_ctx);

/* k3_decoder_layer_inc_log for an MLA + MoE layer: k3gpu_decoder_layer_kda_verify's steps
 * with k3gpu_mla_layer_verify as the attention (cache arguments as there). */
int k3gpu_decoder_layer_mla_verify(float *h, float *block_residual, int *n_blocks, int *moe_idx,
                                   float *moe_wt, const K3GpuMlaLayerW *w,
                                   const K3GpuLayerCfg *c, int layer_idx, uint16_t *lat,
                                   uint16_t *rope, int cap, const int *cached,
                                   const uint64_t *mask, int max_ctx, int B, int T,
                                   void *workspace, size_t ws_bytes, void *stream);

/* ------------------------------------------------------ model verify forward ---- */
/* The reference's forward() with arg_all (src/cli/k3_run.c:853-1138) for a whole model of
 * KDA + MoE and MLA + MoE decoder layers, over B sequences at once, and the commit behind
 * a speculative sweep (spec_commit :1270-1300 with `cached += keep` :2941-2943).
 * A sweep of T <= max_T positions per sequence: embed rows (bf16 -> fp32), every layer in
 * order (k3gpu_decoder_layer_kda_verify / _mla_verify: KDA tentative and logged, MLA
 * appending its rows at cached[b] + t), the model-level AttnRes over the block snapshots
 * (:1071-1087), the final RMSNorm, the lm_head over every position and the per-position
 * argmax (argmax_, :138-139). The commit replays the first keep[b] logged positions into
 * each KDA layer's state (k3_kda_advance) and advances cached[b]; the MLA rows past it
 * are overwritten by the next sweep, as in the reference. With a draft tree (parents
 * given) the KDA layers follow each node's ancestors (k3gpu_decoder_layer_kda_verify_tree),
 * the MLA layers the nodes' ancestor masks, and the commit first gathers the accepted
 * path's log rows and cache rows to the front.
 * Device memory: one caller-owned arena of k3gpu_model_arena_bytes (every KDA layer's
 * state, history and log, every MLA layer's bf16 latent and rope caches of kv_cap
 * positions, the sweep's activations, snapshots, logits [B*max_T][vocab] and the largest
 * layer workspace); the host object holds pointers, a small pinned staging ring and the
 * host copy of cached. Not for concurrent calls on one model. */
typedef struct {
    K3GpuLayerCfg layer;     /* every layer's configuration (max_blocks: the reference's
                                k3_attn_res_stride, n_layers / attn_res_block + 2)        */
    int n_layers, vocab;
    const int *is_mla;       /* host [n_layers]: 1 for an MLA layer (one-based
                                full_attn_layers of the config, src/core/k3_ops.c:119-127) */
} K3GpuModelCfg;

typedef struct {
    const uint16_t *embed;           /* bf16 [vocab][E]                                    */
    const uint16_t *lm_head;         /* bf16 [vocab][E]                                    */
    const float *norm;               /* [E], the final RMSNorm                             */
    const float *out_res_fold;       /* [E] or NULL: the model-level AttnRes fold           */
    const K3GpuKdaLayerW *kda;       /* host [n_layers]: the entries of the KDA layers      */
    const K3GpuMlaLayerW *mla;       /* host [n_layers]: the entries of the MLA layers      */
} K3GpuModelW;

typedef struct K3GpuModel K3GpuModel;

/* 0 for a configuration the layers refuse, B outside 1..4096, max_T outside 1..64 or
 * kv_cap < max_T. */
size_t k3gpu_model_arena_bytes(const K3GpuModelCfg *c, int B, int max_T, int kv_cap);
/* The weight structures are copied (their device pointers must stay valid); the arena
 * (256-byte aligned) is laid out and the states zeroed on `stream`. NULL on a bad
 * argument or a failed host allocation. */
K3GpuModel *k3gpu_model_create(const K3GpuModelCfg *c, const K3GpuModelW *w, int B, int max_T, int kv_cap,
                               void *arena, size_t arena_bytes, void *stream);
void k3gpu_model_free(K3GpuModel *m);
int k3gpu_model_set_stream(K3GpuModel *m, void *stream);
/* zero every KDA state and history, cached = 0 (the caches need no clearing) */
int k3gpu_model_reset(K3GpuModel *m);
/* ids: DEVICE [B][T]; parent: HOST [T] or NULL (a chain), one tree shape for every
 * sequence; arg: DEVICE [B][T] or NULL; *logits (optional) receives the model's logits
 * buffer [B][T][vocab], valid until the next sweep. K3GPU_ECAPACITY when a sequence's
 * cached + T passes kv_cap. */
int k3gpu_model_verify(K3GpuModel *m, const int *ids, int T, const int *parent, int *arg,
                       const float **logits);
/* The same sweep for greedy acceptance: the lm_head fused with the argmax
 * (k3gpu_lm_head_argmax), arg DEVICE [B][T] filled, no logits written. */
int k3gpu_model_verify_greedy(K3GpuModel *m, const int *ids, int T, const int *parent, int *arg);
/* keep: HOST [B], 0..T of the last verify; path: HOST [B][T] (a tree sweep only): the
 * accepted nodes root first along the parents. */
int k3gpu_model_commit(K3GpuModel *m, const int *keep, const int *path);
/* the chain commit with the counts already on the device (e.g. n_emit of an on-device
 * accept); keep_host [B] the same counts for the host copy of cached */
int k3gpu_model_commit_device(K3GpuModel *m, const int *keep_dev, const int *keep_host);
/* a prompt ids DEVICE [B][n] read in and committed in passes of max_T; next DEVICE [B]
 * the argmax after each sequence's last position */
int k3gpu_model_prefill(K3GpuModel *m, const int *ids, int n, int *next);
int k3gpu_model_cached(const K3GpuModel *m, int *cached);   /* host [B] */
/* Positions each sequence has consumed (host [B], 0..kv_cap), e.g. after the caller wrote
 * a resumed session's cache rows and KDA states through the views below. Discards a sweep
 * awaiting its commit. */
int k3gpu_model_set_cached(K3GpuModel *m, const int *cached);
/* device views of a layer's state: KDA [B][H][D][D] and [B][3][P][K-1]; MLA caches */
int k3gpu_model_kda_state(const K3GpuModel *m, int layer, float **state, float **conv_hist);
int k3gpu_model_mla_cache(const K3GpuModel *m, int layer, uint16_t **lat, uint16_t **rope);
/* the routing of the last layer of the last sweep: idx [B*T][topk] (device) */
int k3gpu_model_last_routing(const K3GpuModel *m, const int **idx);
/* The decode loop's callbacks (K3SpecVerifyFn / K3SpecCommitFn) for a model of B == 1,
 * ctx = the model: verify uploads the host ids, sweeps and returns every position's argmax
 * on the host (synchronising the model's stream); a read-in longer than max_T runs in
 * passes, all but the last committed at once. */
int k3gpu_model_loop_verify(void *ctx, const int *ids, const int *parent, int n, int base, int *arg);
int k3gpu_model_loop_commit(void *ctx, int base, const int *path, int keep);

/* ---------------------------------------------------- conversation state ------ */
/* Host C: the conversation state file, K3ST version 2 byte for byte as the reference's
 * k3_state_save / k3_state_peek / k3_state_load (src/cli/k3_run.c:162-407) write and read
 * it, so a session saved by either engine resumes on the other. The layout fields are the
 * header's (fp = k3_state_fp: hidden, n_layers, vocab, kda_heads, kda_head_dim, conv_k,
 * n_heads, qk_nope, qk_rope, v_head, n_experts, topk; kper = KDA floats per layer slot,
 * the matrices [H][D][D] then the ShortConv history [3][P][K-1]; kvpp / ropepp = cache and
 * rope floats per position per MLA layer) and the layer-loop record's (count 0: none). ks
 * [kper * slots] (slots = loop_nv with a loop, else n_bound), kvc [n_mla][kv_cap][kvpp] and
 * ropec [n_mla][kv_cap][ropepp] are host fp32 arrays (this library's bf16 MLA cache widens
 * exactly into them). A save holds the cached positions' ids and at most one pending id.
 * load refuses (K3GPU_EINVAL) another loop, fingerprint, layer count or cache width, a
 * malformed or truncated file; K3GPU_ECAPACITY when the file holds more positions than
 * kv_cap or more ids than seq_cap. */
typedef struct {
    int32_t fp[12];
    int32_t n_bound, n_mla;
    int64_t kper, kvpp, ropepp;
    int32_t loop_a, loop_b, loop_count, loop_nv;
    double loop_eps;
} K3StateLayout;
int k3_state_save(const char *path, const K3StateLayout *layout, const int *seq, int nseq,
                  int cached, const float *ks, const float *kvc, const float *ropec, int kv_cap,
                  const int *pcached, const int *passes);
int k3_state_peek(const char *path, K3StateLayout *layout, int *cached, int *nseq);
int k3_state_load(const char *path, const K3StateLayout *expect, int *seq, int seq_cap,
                  float *ks, float *kvc, float *ropec, int kv_cap, int *pcached, int *passes,
                  int *cached, int *nseq);

/* ------------------------------------------------------- expert parallel ------ */
/* The routed experts of a layer split over `world` ranks, one process per GPU, the token
 * rows exchanged through peer memory (NVLink / NVSwitch) instead of all-to-all calls:
 * each rank cudaMallocs an exchange arena (k3gpu_ep_arena_alloc) and shares it by CUDA IPC
 * (k3gpu_ep_ipc_handle on the owner, k3gpu_ep_ipc_open on every other rank). A step with
 * sequence number seq (1, 2, ... the same on every rank) is, on every rank:
 *   k3gpu_ep_dispatch  this rank's token rows to the ranks owning their experts
 *   k3gpu_ep_receive   wait for every source; the receive region (k3gpu_ep_recv_views,
 *                      world*cap rows, unused ones dropped) is then the input of
 *                      k3gpu_moe_experts over this rank's n_local experts
 *   k3gpu_ep_return    the experts' [world*cap][L] output rows back to their sources
 *   k3gpu_ep_combine   wait for every owner; out[t] += its rows' partial sums (owner order)
 * No host synchronisation; every wait is bounded (DEV_TIMEOUT in k3gpu_device_status, the
 * missing peer's rows counted as empty). */
#define K3GPU_EP_MAX_WORLD 8
#define K3GPU_EP_HANDLE_BYTES 64
typedef struct {
    void *arena[K3GPU_EP_MAX_WORLD];   /* every rank's arena as mapped here; own at [rank] */
    int world, rank;
    int cap;                           /* most token rows a rank sends in a step */
    int L, K, n_local;                 /* row width, top-k, experts per rank */
} K3GpuEpGroup;

size_t k3gpu_ep_arena_bytes(int world, int cap, int L, int K);
int k3gpu_ep_arena_alloc(void **arena, size_t bytes);   /* zeroed */
int k3gpu_ep_arena_free(void *arena);
int k3gpu_ep_ipc_handle(const void *arena, void *handle);   /* K3GPU_EP_HANDLE_BYTES out */
int k3gpu_ep_ipc_open(const void *handle, void **peer);
int k3gpu_ep_ipc_close(void *peer);
int k3gpu_ep_recv_views(const K3GpuEpGroup *g, float **x_recv, int **idx_recv, float **wt_recv);
/* x [T][L], idx/wt [T][K] (global expert ids, -1 dropped), T <= cap; pos [world][T]
 * (device workspace) receives each token's slot on each rank, for the combine. */
int k3gpu_ep_dispatch(const K3GpuEpGroup *g, const float *x, const int *idx, const float *wt,
                      int T, unsigned seq, int *pos, void *stream);
int k3gpu_ep_receive(const K3GpuEpGroup *g, unsigned seq, void *stream);
int k3gpu_ep_return(const K3GpuEpGroup *g, const float *part, unsigned seq, void *stream);
/* ok [world] (device) receives 1 per owner whose rows arrived. */
int k3gpu_ep_combine(const K3GpuEpGroup *g, float *out, const int *pos, int T, unsigned seq,
                     int *ok, void *stream);
/* The single-layer MoE (k3gpu_moe_layer) with its routed experts split over the ranks of g:
 * this rank's tokens are routed on the replicated gate (global expert ids), their rows
 * exchanged through peer memory (k3gpu_ep_dispatch / _receive / _return / _combine), this
 * rank's n_local experts (local, the experts rank * n_local .. + n_local - 1) run on what it
 * received, the replicated shared experts (shared, n_shared of them, may be NULL when 0) on
 * its own tokens, and out [T][L] = shared + the owners' partial sums in owner order. Every
 * rank calls it with the same seq, in the same order (seq 1, 2, ... per exchange step);
 * topk == g->K, n_routed == world * n_local, T <= g->cap. ok [world] (device) as
 * k3gpu_ep_combine. Equal to k3gpu_moe_layer over the whole bank to fp32 rounding (the
 * sum runs per owner, then across owners). */
size_t k3gpu_moe_layer_ep_workspace(const K3GpuEpGroup *g, int T, int n_shared, int I, int n_routed);
int k3gpu_moe_layer_ep(float *out, int *idx, float *wt, const float *x, const float *gate_W,
                       const float *bias, const K3GpuExpertBank *local, const K3GpuExpertBank *shared,
                       const K3GpuEpGroup *g, unsigned seq, int T, int topk, int n_routed, int n_shared,
                       int act, float b1, float b2, int renorm, float routed_scale, int *ok,
                       void *workspace, size_t ws_bytes, void *stream);

/* The whole model (k3gpu_model_*, above) with its MoE steps expert parallel. */
/* Expert parallel: every layer's MoE step splits its routed experts over the ranks of g
 * (k3gpu_moe_layer_ep), each rank running its own sequences. Set once after create; every
 * layer's bank then holds this rank's routed experts (g->n_local of them, the single-layer
 * MoE form) and shared [n_layers] (host array) the replicated shared experts of each layer.
 * Every rank must make the same sequence of sweeps (the layers' exchanges pair up by
 * step number). g->cap >= B * max_T. workspace (256-byte aligned, caller-owned) of
 * k3gpu_model_ep_workspace bytes. k3gpu_model_ep_status reads the last exchange's per-owner
 * flags (host [world]; synchronises the model's stream): a 0 is an owner whose bounded wait
 * ran out. */
size_t k3gpu_model_ep_workspace(const K3GpuModel *m, const K3GpuEpGroup *g);
int k3gpu_model_set_ep(K3GpuModel *m, const K3GpuEpGroup *g, const K3GpuExpertBank *const *shared,
                       void *workspace, size_t ws_bytes);
int k3gpu_model_ep_status(const K3GpuModel *m, int *ok_host);


/* The bound of every exchange wait, in flag polls about 100 ns apart (host, per process,
 * read at each launch; default 2^24, about 1.7 s; 1 .. 2^30). A wait that runs out records
 * DEV_TIMEOUT and treats the silent peer's rows as empty. */
int k3gpu_ep_set_wait_limit(long long polls);

/* ---------------------------------------------------------------- drafter ------ */
/* Host C (no GPU): the reference's n-gram drafter, spec_draft (src/cli/k3_run.c:450-491),
 * with the n range and cap as parameters (the reference fixes n = 4 then 3 and clamps
 * cap to K3_SPEC_MAX = 8). seq [T] host, out [cap] host; returns the draft count. */
int k3_spec_draft_ngram(const int *seq, int T, int cap, int nmax, int nmin, int *out);

/* Host C: the reference drafting study's P1 (tools/spec_replay.py:174-184): the most
 * recent earlier occurrence of the history's suffix 4-gram, else 3-gram, else 2-gram, and
 * the ids that followed it, up to cap (<= 8) and the end of the history; no agreement
 * gate. seq [T] host, out [cap]; returns the draft count. */
int k3_spec_draft_eager(const int *seq, int T, int cap, int *out);

/* Host C: the study's P2 (tools/spec_replay.py:256-336, 442-449) as an incremental
 * drafter: an online suffix automaton over the history. push appends ids; draft proposes,
 * after the history seq[0..T), the continuation of the longest suffix that also ends
 * earlier: with e its most recent earlier end, out[i] = seq[e + 1 + i % (T - 1 - e)] for
 * i < cap (<= 8), a copy that continues periodically past the end of the history. It
 * fires (returns cap) when that suffix has at least min_len ids, else returns 0;
 * match_len and period receive its length and T - 1 - e (0 when there is none). */
typedef struct K3SuffixDrafter K3SuffixDrafter;
K3SuffixDrafter *k3_suffix_drafter_create(int capacity);   /* most ids it will hold */
void k3_suffix_drafter_free(K3SuffixDrafter *d);
int k3_suffix_drafter_push(K3SuffixDrafter *d, const int *ids, int n);
int k3_suffix_drafter_length(const K3SuffixDrafter *d);
int k3_suffix_drafter_draft(const K3SuffixDrafter *d, int cap, int min_len, int *out,
                            int *match_len, int *period);
/* P3 of the drafting study (tools/spec_replay.py:340-397, 474-568): P2's draft with an
 * adaptive length read off an acceptance table q[K3_SPEC_P3_CODES] fitted offline (the
 * study's fit_acceptance_table). Feature code per draft position: (depth bucket x 13
 * match-length buckets) x 6 agreement buckets; 255 when the history has no earlier match. */
#define K3_SPEC_P3_CODES 234
/* The study's verify-step cost model in units of one plain decode step: a verify over nd
 * drafts costs a_T + a_E * u(nd + 1) + a_C * (nd + 1) + eps, u(n) = r * (1 - ((r-1)/r)^n)
 * with r = expert_ratio (routed experts / top-k; 56 for 896 top-16). */
typedef struct K3SpecCost {
    double a_T, a_E, a_C, eps, expert_ratio;
} K3SpecCost;
/* draft_features: codes[nd] (nd <= 8) for `draft` continuing the current history. */
int k3_suffix_drafter_features(const K3SuffixDrafter *d, const int *draft, int nd, unsigned char *codes);
/* adaptive_lengths: cumulative != 0 counts the positions whose cumulative estimate
 * (product of q over 1..j) exceeds delta; cumulative == 0 the leading positions whose own
 * estimate does. 0 when codes[0] is 255. */
int k3_spec_p3_length(const unsigned char *codes, int nd, const double *q, double delta, int cumulative);
/* cost_aware_lengths: draft j is kept while P_j > S(j+1) - S(j) (+ (P_{j-1} - P_j) R(j-1)
 * with replay != 0, R the replay pass after a partial acceptance). */
int k3_spec_p3_cost_length(const unsigned char *codes, int nd, const double *q, const K3SpecCost *cost,
                           int replay);
/* The P3 draft: P2's 8-id draft (any match length), its codes, then the delta rule (cost
 * NULL) or the cost rule; ids out[0..len), len <= cap returned. */
int k3_suffix_drafter_draft_p3(const K3SuffixDrafter *d, const double *q, double delta, const K3SpecCost *cost,
                               int replay, int cap, int *out);
/* ------------------------------------------------------- speculative decode loop -- */
/* The engine's incremental decode loop (src/cli/k3_run.c:2812-3047) as a step driver over
 * two callbacks, so the same bookkeeping drives the device forward:
 *   verify(ctx, ids, parent, n, base, arg): feed ids[0..n) tentatively from position base;
 *       parent NULL: a chain at positions base..base+n-1; else a draft tree (parent[0] = -1,
 *       parent[i] < i; node i sits at depth(i) past base and attends to its ancestors).
 *       arg[i] = the model's greedy next id after node i; 0 on success.
 *   commit(ctx, base, path, keep): keep `keep` positions of that verify -- the first keep
 *       (path NULL) or the tree nodes path[0..keep), root first -- so the model's state
 *       advances to base + keep; 0 on success.
 * Every verify is followed by exactly one commit before the next verify. The first step
 * reads every id not yet consumed (a prompt, or a resumed pending id plus a new prompt)
 * and emits the model's next id; later steps draft (policy below) when the context and the
 * cache have room for spec_n more ids (T + spec_n + 1 < tmax, cached + spec_n + 1 <= kv_cap),
 * verify the pending id plus the drafts, emit the accepted prefix plus the model's own next
 * id, and keep what emit_keep allows (gen, tmax, the first stop id; :1300-1317). */
enum {
    K3_DRAFT_NONE = 0,   /* serial decode                                       */
    K3_DRAFT_NGRAM = 1,  /* the engine's spec_draft (n = 4 then 3, agreement)   */
    K3_DRAFT_EAGER = 2,  /* P1                                                  */
    K3_DRAFT_SUFFIX = 3, /* P2 (min_len)                                        */
    K3_DRAFT_P3 = 4,     /* P3 (p3_q with p3_delta, or p3_cost and p3_replay)   */
    K3_DRAFT_TREE = 5,   /* a draft tree (k3_suffix_drafter_tree: tree_nodes,
                            tree_branch, depth spec_n, min_len), accepted as
                            k3gpu_accept_tree_greedy does                       */
    K3_DRAFT_MODEL = 6   /* a second model proposes spec_n ids (the engine's
                            --draft): k3_spec_loop_set_draft_model             */
};
enum { K3_SPEC_LOOP_GEN = 1, K3_SPEC_LOOP_STOP_ID = 2, K3_SPEC_LOOP_CONTEXT = 3, K3_SPEC_LOOP_PAUSED = 4 };
typedef struct K3SpecLoopCfg {
    int policy, spec_n, min_len;   /* spec_n <= 8                                          */
    int gen, tmax, kv_cap;         /* ids to generate; context limit; cache positions      */
    const int *stop_ids;           /* copied at create                                     */
    int n_stop;
    const double *p3_q;            /* [K3_SPEC_P3_CODES], read at every P3 draft           */
    double p3_delta;
    const K3SpecCost *p3_cost;     /* NULL: the delta rule                                 */
    int p3_replay;
    int tree_nodes, tree_branch;   /* the tree policy: nodes <= 64 per verify, children    */
    int prefill_chunk;             /* the first step reads the prompt in passes of at most
                                      this many positions (0: one pass; --prefill-chunk)    */
    int pause_after;               /* with a checkpoint callback: pause after this many
                                      checkpoints (0: never; --pause-after)                 */
} K3SpecLoopCfg;
/* The engine's spec counters (:2945-2955) and the histogram of accepted prefixes. */
typedef struct K3SpecLoopStats {
    long long steps, sweeps, drafted, accepted, dropped, full, partial, cut;
    long long hist[9];
    /* the draft model's (k3_run.c:2636): rounds, ids proposed, accepted, fed positions dropped */
    long long draft_rounds, draft_drafted, draft_accepted, draft_dropped;
} K3SpecLoopStats;
/* One step's (nd, m, keep) (the engine's spec_trace, :2946-2949) and the positions fed. */
typedef struct K3SpecStepTrace {
    int nd, m, keep, fed;
} K3SpecStepTrace;
typedef struct K3SpecLoop K3SpecLoop;
typedef int (*K3SpecVerifyFn)(void *ctx, const int *ids, const int *parent, int n, int base, int *arg);
typedef int (*K3SpecCommitFn)(void *ctx, int base, const int *path, int keep);
/* called after every read-in pass that leaves prompt positions to go, with the positions
 * read so far: the moment to save a checkpoint of the model's state (--checkpoint,
 * src/cli/k3_run.c:1225-1231); 0 on success. */
typedef int (*K3SpecCheckpointFn)(void *ctx, int cached);
/* ids[0..n_ids): the conversation so far; cached: positions the model has consumed
 * (0 on a fresh run). NULL on a bad configuration. */
K3SpecLoop *k3_spec_loop_create(const K3SpecLoopCfg *cfg, const int *ids, int n_ids, int cached,
                                K3SpecVerifyFn verify, K3SpecCommitFn commit, void *ctx);
void k3_spec_loop_free(K3SpecLoop *L);
/* One step: out[0..*n_out) the ids kept (<= 9), trace optional. Returns K3GPU_OK, or once
 * finished K3_SPEC_LOOP_GEN / _STOP_ID / _CONTEXT (this and every later call emit
 * nothing), or a negative status (K3GPU_ECALLBACK when a callback failed). */
int k3_spec_loop_step(K3SpecLoop *L, int *out, int *n_out, K3SpecStepTrace *trace);
/* The checkpoint callback for the prompt read-in, set before the first step. With it, the
 * read-in pauses after cfg.pause_after checkpoints or at the first checkpoint after
 * k3_spec_loop_request_pause (callable from any thread, the engine's SIGINT): the step then
 * returns K3_SPEC_LOOP_PAUSED having emitted nothing, k3_spec_loop_state's cached is the
 * positions read, and a new loop created with that `cached` continues the read-in. */
int k3_spec_loop_set_checkpoint(K3SpecLoop *L, K3SpecCheckpointFn fn, void *ctx);
void k3_spec_loop_request_pause(K3SpecLoop *L);
/* The draft model for K3_DRAFT_MODEL, set before the first step; its callbacks have the
 * target's signatures (parent always NULL). It reads the conversation once at the first
 * step (verify then commit of every id); each later drafting step calls dverify once with
 * the ids it has not seen plus the pending one and then once per further draft with its
 * own previous id, each call continuing where the previous tentative one ended, and then
 * dcommit(base, keep) keeps the first `keep` of those tentative positions. */
int k3_spec_loop_set_draft_model(K3SpecLoop *L, K3SpecVerifyFn dverify, K3SpecCommitFn dcommit, void *dctx);
/* T, cached, generated count and counters; returns the finished code (0 while running). */
int k3_spec_loop_state(const K3SpecLoop *L, int *T, int *cached, int *nout, K3SpecLoopStats *stats);
/* The conversation's ids (ids[0..T), cap >= T); returns T. */
int k3_spec_loop_ids(const K3SpecLoop *L, int *ids, int cap);

/* The layer loop's execution order (the engine's --loop / --loop-layers A-B /
 * --loop-count R, src/cli/k3_run.c:2140-2182): layers 0..B, then R - 1 repeats of A..B,
 * then B+1..n_layers-1. vmap[v] is the physical layer executed at position v; each
 * executed position owns its own KDA state and MLA cache slot (slot v), as a duplicated
 * layer would, so a K3ST file's loop record holds nv = the count returned. The span must
 * be whole AttnRes blocks (A a multiple of the block, B + 1 one too or B the last layer);
 * preset != 0 takes the block holding the middle layer (--loop) and ignores A, B.
 * span_out [2] (optional) receives A, B; attn_res_extra (optional) the block-residual
 * stride's growth, (R - 1) * ceil(span / block). Returns the executed layer count, or
 * K3GPU_EINVAL / K3GPU_ECAPACITY (vmap_cap short). Adaptive exit (--loop-exit) is not
 * planned here. */
int k3_layer_loop_plan(int n_layers, int attn_res_block, int preset, int loop_a, int loop_b, int loop_count,
                       int *vmap, int vmap_cap, int *span_out, int *attn_res_extra);

/* A draft TREE for tree verification (no counterpart in the reference, whose drafts are
 * chains): node 0 is the pending id; a node's children are the ids that followed its
 * context in the history, most frequent first (at most `branch`), the context backing off
 * to shorter suffixes of at least min_len ids when it has no continuation; nodes are
 * added best-first by the product of relative frequencies along their path, up to
 * max_nodes (<= 65536) and max_depth. tok/parent [max_nodes] in the order of
 * k3gpu_accept_tree_greedy (parents first, parent[0] = -1); returns the node count, 0 for
 * bad arguments. */
int k3_suffix_drafter_tree(const K3SuffixDrafter *d, int max_nodes, int branch, int max_depth,
                           int min_len, int *tok, int *parent);

#ifdef __cplusplus
}
#endif

#endif /* K3GPU_H */
