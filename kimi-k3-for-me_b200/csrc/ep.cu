// ep.cu -- expert-parallel dispatch and combine over peer memory (NVLink / NVSwitch).
//
// The routed experts of a layer are split over `world` ranks (one process per GPU). Each
// rank owns an exchange arena in its HBM that every other rank maps by CUDA IPC. A step:
//
//   dispatch  (source s) every token row goes once to each rank d that owns one of its
//             experts: P2P stores of the row into d's arena at x_recv[s][slot], the slot's
//             local expert ids and weights into idx_recv/wt_recv[s][slot], the row count
//             into recv_cnt[s]; then a release of recv_flag[s] = seq (system scope)
//   receive   (owner d) a bounded wait for every source's flag, then the slots past each
//             source's count are marked dropped (-1), so the experts run on the fixed
//             [world * cap] receive region with no host round trip
//   return    (owner d) the experts' weighted partial rows go back to each source's arena
//             at back[d][slot], then back_flag[d] = seq on the source
//   combine   (source s) a bounded wait for every owner's flag, then out[t] += the partial
//             rows of t from each owner, in owner order
//
// Single buffering is safe: a source writes step n+1 rows into an owner only after its
// combine of step n saw that owner's return, which the owner issues after its experts read
// step n's rows; likewise for the return rows. Waits are bounded: a wait that gives up
// records DEV_TIMEOUT and the slots of that peer are treated as empty. No TMA, no
// multicast: plain loads and stores through mapped peer pointers.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"

namespace k3 {
namespace ep {

constexpr int HDR_BYTES = 4096;                 // recv_cnt, recv_flag, back_flag, eff_cnt
constexpr long long SPIN_DEFAULT = 1LL << 24;   // flag polls (~100 ns apart) before giving up: ~1.7 s
static long long g_spin = SPIN_DEFAULT;          // k3gpu_ep_set_wait_limit

struct Layout {
    size_t x_recv, idx_recv, wt_recv, back, total;
};

static size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

static Layout layout(int world, int cap, int L, int K)
{
    Layout l;
    size_t o = HDR_BYTES;
    l.x_recv = o;
    o += a256((size_t)world * cap * L * 4);
    l.idx_recv = o;
    o += a256((size_t)world * cap * K * 4);
    l.wt_recv = o;
    o += a256((size_t)world * cap * K * 4);
    l.back = o;
    o += a256((size_t)world * cap * L * 4);
    l.total = o;
    return l;
}

struct Ptrs {   // kernel argument: every rank's arena as mapped in this process
    char *arena[K3GPU_EP_MAX_WORLD];
};

__device__ __forceinline__ int *recv_cnt(char *a) { return reinterpret_cast<int *>(a); }
__device__ __forceinline__ unsigned *recv_flag(char *a) { return reinterpret_cast<unsigned *>(a + 1024); }
__device__ __forceinline__ unsigned *back_flag(char *a) { return reinterpret_cast<unsigned *>(a + 2048); }
// the counts the owner accepted this step (0 for a source that never signalled)
__device__ __forceinline__ int *eff_cnt(char *a) { return reinterpret_cast<int *>(a + 3072); }

__device__ __forceinline__ void store_release_sys(unsigned *p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned load_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// bounded wait for *p == seq (flags only grow; a later value also means seq was passed)
__device__ __forceinline__ bool wait_flag(const unsigned *p, unsigned seq, long long spin)
{
    for (long long i = 0; i < spin; i++) {
        if ((int)(load_acquire_sys(p) - seq) >= 0) return true;
        __nanosleep(64);
    }
    return false;
}

// grid world, block 1024: CTA d finds the tokens with a slot on rank d (scan in token order),
// writes pos[d][t] (slot or -1) and each slot's local ids / weights into d's arena, and d's
// recv_cnt[me]
__global__ void __launch_bounds__(1024) dispatch_meta_kernel(Ptrs P, int *__restrict__ pos, const int *__restrict__ idx,
                                                              const float *__restrict__ wt, int T, int K, int n_local,
                                                              int cap, int me, int world, size_t off_idx,
                                                              size_t off_wt)
{
    __shared__ int warp_tot[32];
    __shared__ int carry;
    const int d = blockIdx.x;
    char *ad = P.arena[d];
    int *ri = reinterpret_cast<int *>(ad + off_idx) + (size_t)me * cap * K;
    float *rw = reinterpret_cast<float *>(ad + off_wt) + (size_t)me * cap * K;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += 1024) {
        const int t = t0 + threadIdx.x;
        int has = 0;
        if (t < T)
            for (int k = 0; k < K; k++) {
                const int e = idx[(size_t)t * K + k];
                if (e >= 0 && e / n_local == d) has = 1;
            }
        // block-wide exclusive scan of `has`, token order
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        const unsigned m = __ballot_sync(0xffffffffu, has);
        const int before = __popc(m & ((1u << lane) - 1u));
        if (lane == 0) warp_tot[w] = __popc(m);
        __syncthreads();
        int wbase = 0;
        for (int i = 0; i < w; i++) wbase += warp_tot[i];
        int total = 0;
        for (int i = 0; i < 32; i++) total += warp_tot[i];
        const int slot = carry + wbase + before;
        if (t < T) {
            const bool ok = has && slot < cap;
            if (has && slot >= cap) flag(DEV_BAD_COUNT);
            pos[(size_t)d * T + t] = ok ? slot : -1;
            if (ok)
                for (int k = 0; k < K; k++) {
                    const int e = idx[(size_t)t * K + k];
                    const bool mine = e >= 0 && e / n_local == d;
                    ri[(size_t)slot * K + k] = mine ? e - d * n_local : -1;
                    rw[(size_t)slot * K + k] = mine ? wt[(size_t)t * K + k] : 0.0f;
                }
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) recv_cnt(ad)[me] = min(carry, cap);
}

// grid (T, world), block 256: row t to rank d's x_recv[me][pos[d][t]] when it goes there
// (vec: 16-byte rows on both sides, chosen per call from L and the caller's pointer)
__global__ void __launch_bounds__(256) dispatch_rows_kernel(Ptrs P, const int *__restrict__ pos,
                                                             const float *__restrict__ x, int T, int L, int cap,
                                                             int me, size_t off_x, int vec)
{
    const int t = blockIdx.x, d = blockIdx.y;
    const int slot = pos[(size_t)d * T + t];
    if (slot < 0) return;
    float *dst = reinterpret_cast<float *>(P.arena[d] + off_x) + ((size_t)me * cap + slot) * L;
    const float *src = x + (size_t)t * L;
    if (vec) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = threadIdx.x; i < L / 4; i += 256) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < L; i += 256) dst[i] = src[i];
    }
}

// block world: thread d publishes seq to rank d (recv_flag[me] for dispatch, back_flag[me]
// for return) after every store of the preceding kernels
__global__ void signal_kernel(Ptrs P, int world, int me, unsigned seq, int which)
{
    const int d = threadIdx.x;
    if (d >= world) return;
    __threadfence_system();
    store_release_sys(which ? back_flag(P.arena[d]) + me : recv_flag(P.arena[d]) + me, seq);
}

// grid world, block 256 (owner): wait for source s's rows, then mark its unused slots
// dropped; a source that never signalled counts as empty
__global__ void __launch_bounds__(256) receive_kernel(char *own, int cap, int K, unsigned seq, size_t off_idx,
                                                      long long spin)
{
    __shared__ int n;
    const int s = blockIdx.x;
    if (threadIdx.x == 0) {
        const bool ok = wait_flag(recv_flag(own) + s, seq, spin);
        if (!ok) flag(DEV_TIMEOUT);
        n = ok ? min(max(recv_cnt(own)[s], 0), cap) : 0;
        eff_cnt(own)[s] = n;
    }
    __syncthreads();
    int *ri = reinterpret_cast<int *>(own + off_idx) + (size_t)s * cap * K;
    for (long long i = (long long)n * K + threadIdx.x; i < (long long)cap * K; i += 256) ri[i] = -1;
}

// grid (cap, world), block 256 (owner): partial row of (source s, slot) back to s
__global__ void __launch_bounds__(256) return_rows_kernel(Ptrs P, const float *__restrict__ part, int L, int cap,
                                                           int me, size_t off_back, int vec)
{
    const int slot = blockIdx.x, s = blockIdx.y;
    char *own = P.arena[me];
    if (slot >= eff_cnt(own)[s]) return;
    float *dst = reinterpret_cast<float *>(P.arena[s] + off_back) + ((size_t)me * cap + slot) * L;
    const float *src = part + ((size_t)s * cap + slot) * L;
    if (vec) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = threadIdx.x; i < L / 4; i += 256) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < L; i += 256) dst[i] = src[i];
    }
}

// block world (source): wait for every owner's return; ok[o] = 1 when it arrived
__global__ void wait_back_kernel(char *own, int world, unsigned seq, int *__restrict__ ok, long long spin)
{
    const int o = threadIdx.x;
    if (o >= world) return;
    const bool got = wait_flag(back_flag(own) + o, seq, spin);
    if (!got) flag(DEV_TIMEOUT);
    ok[o] = got ? 1 : 0;
}

// grid (T, ceil(L / 1024)), block 256 (source): out[t] += back[o][pos[o][t]] for o ascending
__global__ void __launch_bounds__(256) combine_kernel(float *__restrict__ out, const char *__restrict__ own,
                                                      const int *__restrict__ pos, const int *__restrict__ ok,
                                                      int T, int L, int cap, int world, size_t off_back)
{
    const int t = blockIdx.x;
    const int i = (blockIdx.y * 256 + threadIdx.x) * 4;
    if (i >= L) return;
    const float *back = reinterpret_cast<const float *>(own + off_back);
    float *o_row = out + (size_t)t * L;
    for (int j = i; j < i + 4 && j < L; j++) {
        float v = o_row[j];
        for (int o = 0; o < world; o++) {
            const int slot = pos[(size_t)o * T + t];
            if (slot >= 0 && ok[o]) v += back[((size_t)o * cap + slot) * L + j];
        }
        o_row[j] = v;
    }
}

static bool group_ok(const K3GpuEpGroup *g)
{
    if (!g || g->world < 1 || g->world > K3GPU_EP_MAX_WORLD || g->rank < 0 || g->rank >= g->world) return false;
    if (g->cap <= 0 || g->L <= 0 || g->K <= 0 || g->n_local <= 0) return false;
    for (int r = 0; r < g->world; r++)
        if (!g->arena[r]) return false;
    return true;
}

static Ptrs ptrs(const K3GpuEpGroup *g)
{
    Ptrs p = {};
    for (int r = 0; r < g->world; r++) p.arena[r] = static_cast<char *>(g->arena[r]);
    return p;
}

}  // namespace ep
}  // namespace k3

extern "C" size_t k3gpu_ep_arena_bytes(int world, int cap, int L, int K)
{
    if (world < 1 || world > K3GPU_EP_MAX_WORLD || cap <= 0 || L <= 0 || K <= 0) return 0;
    return k3::ep::layout(world, cap, L, K).total;
}

extern "C" int k3gpu_ep_arena_alloc(void **arena, size_t bytes)
{
    if (!arena || bytes == 0) return K3GPU_EINVAL;
    void *p = nullptr;
    int st = k3::cuda_status(cudaMalloc(&p, bytes));
    if (st) return st;
    if ((st = k3::cuda_status(cudaMemset(p, 0, bytes)))) {
        cudaFree(p);
        return st;
    }
    *arena = p;
    return K3GPU_OK;
}

extern "C" int k3gpu_ep_arena_free(void *arena)
{
    if (!arena) return K3GPU_EINVAL;
    return k3::cuda_status(cudaFree(arena));
}

extern "C" int k3gpu_ep_ipc_handle(const void *arena, void *handle)
{
    if (!arena || !handle) return K3GPU_EINVAL;
    cudaIpcMemHandle_t h;
    const int st = k3::cuda_status(cudaIpcGetMemHandle(&h, const_cast<void *>(arena)));
    if (st) return st;
    memcpy(handle, &h, sizeof(h) < K3GPU_EP_HANDLE_BYTES ? sizeof(h) : K3GPU_EP_HANDLE_BYTES);
    return K3GPU_OK;
}

extern "C" int k3gpu_ep_ipc_open(const void *handle, void **peer)
{
    if (!handle || !peer) return K3GPU_EINVAL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return k3::cuda_status(cudaIpcOpenMemHandle(peer, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int k3gpu_ep_ipc_close(void *peer)
{
    if (!peer) return K3GPU_EINVAL;
    return k3::cuda_status(cudaIpcCloseMemHandle(peer));
}

extern "C" int k3gpu_ep_recv_views(const K3GpuEpGroup *g, float **x_recv, int **idx_recv, float **wt_recv)
{
    using namespace k3::ep;
    if (!group_ok(g) || !x_recv || !idx_recv || !wt_recv) return K3GPU_EINVAL;
    const Layout l = layout(g->world, g->cap, g->L, g->K);
    char *own = static_cast<char *>(g->arena[g->rank]);
    *x_recv = reinterpret_cast<float *>(own + l.x_recv);
    *idx_recv = reinterpret_cast<int *>(own + l.idx_recv);
    *wt_recv = reinterpret_cast<float *>(own + l.wt_recv);
    return K3GPU_OK;
}

extern "C" int k3gpu_ep_dispatch(const K3GpuEpGroup *g, const float *x, const int *idx, const float *wt, int T,
                                 unsigned seq, int *pos, void *stream)
{
    using namespace k3::ep;
    if (!group_ok(g) || !x || !idx || !wt || !pos || T <= 0 || T > g->cap || seq == 0) return K3GPU_EINVAL;
    const Layout l = layout(g->world, g->cap, g->L, g->K);
    cudaStream_t s = k3::as_stream(stream);
    const Ptrs P = ptrs(g);
    dispatch_meta_kernel<<<g->world, 1024, 0, s>>>(P, pos, idx, wt, T, g->K, g->n_local, g->cap, g->rank, g->world,
                                                  l.idx_recv, l.wt_recv);
    int st = k3::launch_status();
    if (st) return st;
    // the arena rows start on 16-byte boundaries when L % 4 == 0 (regions are 256-aligned)
    const int vec = (g->L & 3) == 0 && k3::aligned(x, 16);
    dispatch_rows_kernel<<<dim3(T, g->world), 256, 0, s>>>(P, pos, x, T, g->L, g->cap, g->rank, l.x_recv, vec);
    if ((st = k3::launch_status())) return st;
    signal_kernel<<<1, 32, 0, s>>>(P, g->world, g->rank, seq, 0);
    return k3::launch_status();
}

extern "C" int k3gpu_ep_receive(const K3GpuEpGroup *g, unsigned seq, void *stream)
{
    using namespace k3::ep;
    if (!group_ok(g) || seq == 0) return K3GPU_EINVAL;
    const Layout l = layout(g->world, g->cap, g->L, g->K);
    receive_kernel<<<g->world, 256, 0, k3::as_stream(stream)>>>(static_cast<char *>(g->arena[g->rank]), g->cap, g->K,
                                                                seq, l.idx_recv, g_spin);
    return k3::launch_status();
}

extern "C" int k3gpu_ep_return(const K3GpuEpGroup *g, const float *part, unsigned seq, void *stream)
{
    using namespace k3::ep;
    if (!group_ok(g) || !part || seq == 0) return K3GPU_EINVAL;
    const Layout l = layout(g->world, g->cap, g->L, g->K);
    cudaStream_t s = k3::as_stream(stream);
    const Ptrs P = ptrs(g);
    const int vec = (g->L & 3) == 0 && k3::aligned(part, 16);
    return_rows_kernel<<<dim3(g->cap, g->world), 256, 0, s>>>(P, part, g->L, g->cap, g->rank, l.back, vec);
    int st = k3::launch_status();
    if (st) return st;
    signal_kernel<<<1, 32, 0, s>>>(P, g->world, g->rank, seq, 1);
    return k3::launch_status();
}

extern "C" int k3gpu_ep_combine(const K3GpuEpGroup *g, float *out, const int *pos, int T, unsigned seq, int *ok,
                                void *stream)
{
    using namespace k3::ep;
    if (!group_ok(g) || !out || !pos || !ok || T <= 0 || T > g->cap || seq == 0) return K3GPU_EINVAL;
    const Layout l = layout(g->world, g->cap, g->L, g->K);
    cudaStream_t s = k3::as_stream(stream);
    char *own = static_cast<char *>(g->arena[g->rank]);
    wait_back_kernel<<<1, 32, 0, s>>>(own, g->world, seq, ok, g_spin);
    int st = k3::launch_status();
    if (st) return st;
    combine_kernel<<<dim3(T, (g->L + 1023) / 1024), 256, 0, s>>>(out, own, pos, ok, T, g->L, g->cap, g->world, l.back);
    return k3::launch_status();
}

extern "C" int k3gpu_ep_set_wait_limit(long long polls)
{
    if (polls < 1 || polls > (1LL << 30)) return K3GPU_EINVAL;
    k3::ep::g_spin = polls;
    return K3GPU_OK;
}

// ---- the expert-parallel MoE layer: route, exchange, local and shared experts, combine ----
namespace k3 {
namespace ep {

// sidx[t][j] = j, swt[t][j] = 1 for the shared experts of every token
__global__ void shared_slots_kernel(int *__restrict__ sidx, float *__restrict__ swt, int n, int n_shared)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        sidx[i] = i % n_shared;
        swt[i] = 1.0f;
    }
}

struct MoeEpWs {
    char *router, *local, *shared;
    int *pos, *sidx;
    float *part, *swt;
    size_t router_bytes, local_bytes, shared_bytes, total;
};

static MoeEpWs moe_ep_layout(const K3GpuEpGroup *g, int T, int n_shared, int I, int n_routed, char *base)
{
    MoeEpWs w{};
    size_t o = 0;
    auto take = [&](size_t b) {
        char *r = base ? base + o : nullptr;
        o += a256(b);
        return r;
    };
    const int R = g->world * g->cap;
    w.router_bytes = k3gpu_router_workspace(T, n_routed);
    w.router = take(w.router_bytes);
    w.local_bytes = k3gpu_moe_workspace(R, g->K, 0, g->L, I, g->n_local);
    w.local = take(w.local_bytes);
    w.shared_bytes = n_shared > 0 ? k3gpu_moe_workspace(T, n_shared, 0, g->L, I, n_shared) : 0;
    w.shared = take(w.shared_bytes);
    w.pos = (int *)take((size_t)g->world * T * 4);
    w.part = (float *)take((size_t)R * g->L * 4);
    w.sidx = (int *)take((size_t)T * (n_shared > 0 ? n_shared : 1) * 4);
    w.swt = (float *)take((size_t)T * (n_shared > 0 ? n_shared : 1) * 4);
    w.total = o;
    return w;
}

}  // namespace ep
}  // namespace k3

extern "C" size_t k3gpu_moe_layer_ep_workspace(const K3GpuEpGroup *g, int T, int n_shared, int I, int n_routed)
{
    if (!k3::ep::group_ok(g) || T <= 0 || T > g->cap || n_shared < 0 || I <= 0 || n_routed <= 0) return 0;
    return k3::ep::moe_ep_layout(g, T, n_shared, I, n_routed, nullptr).total;
}

extern "C" int k3gpu_moe_layer_ep(float *out, int *idx, float *wt, const float *x, const float *gate_W,
                                  const float *bias, const K3GpuExpertBank *local, const K3GpuExpertBank *shared,
                                  const K3GpuEpGroup *g, unsigned seq, int T, int topk, int n_routed, int n_shared,
                                  int act, float b1, float b2, int renorm, float routed_scale, int *ok,
                                  void *workspace, size_t ws_bytes, void *stream)
{
    using namespace k3::ep;
    if (!out || !idx || !wt || !x || !gate_W || !local || !ok || !workspace || !group_ok(g) || seq == 0)
        return K3GPU_EINVAL;
    if (T <= 0 || T > g->cap || topk != g->K || n_routed != g->world * g->n_local || local->n_experts != g->n_local ||
        local->L != g->L || n_shared < 0 || (n_shared > 0 && (!shared || shared->n_experts != n_shared ||
                                                              shared->L != g->L || shared->I != local->I)))
        return K3GPU_EINVAL;
    const size_t need = k3gpu_moe_layer_ep_workspace(g, T, n_shared, local->I, n_routed);
    if (!need) return K3GPU_EINVAL;
    if (ws_bytes < need) return K3GPU_ECAPACITY;
    const MoeEpWs w = moe_ep_layout(g, T, n_shared, local->I, n_routed, static_cast<char *>(workspace));
    cudaStream_t s = k3::as_stream(stream);
    int st;
    // 1. the replicated gate on this rank's tokens (global expert ids)
    if ((st = k3gpu_router(idx, wt, x, gate_W, bias, T, g->L, n_routed, topk, renorm, routed_scale, w.router,
                           w.router_bytes, stream)))
        return st;
    // 2. every token row once to each owner of one of its experts
    if ((st = k3gpu_ep_dispatch(g, x, idx, wt, T, seq, w.pos, stream))) return st;
    // 3. the shared experts on this rank's own tokens while the rows travel (out = shared)
    if (n_shared > 0) {
        shared_slots_kernel<<<k3::ceil_div((long long)T * n_shared, 256), 256, 0, s>>>(w.sidx, w.swt, T * n_shared,
                                                                                       n_shared);
        if ((st = k3::launch_status())) return st;
        if ((st = k3gpu_moe_experts(out, x, w.sidx, w.swt, shared, T, n_shared, n_shared, 0, act, b1, b2, nullptr,
                                    0.0f, w.shared, w.shared_bytes, stream)))
            return st;
    } else if ((st = k3::cuda_status(cudaMemsetAsync(out, 0, (size_t)T * g->L * 4, s)))) {
        return st;
    }
    // 4. this rank's experts over the fixed receive region (dropped slots skipped)
    if ((st = k3gpu_ep_receive(g, seq, stream))) return st;
    float *xr;
    int *ir;
    float *wr;
    if ((st = k3gpu_ep_recv_views(g, &xr, &ir, &wr))) return st;
    if ((st = k3gpu_moe_experts(w.part, xr, ir, wr, local, g->world * g->cap, topk, g->n_local, 0, act, b1, b2,
                                nullptr, 0.0f, w.local, w.local_bytes, stream)))
        return st;
    // 5. the partial rows home, added per token in owner order
    if ((st = k3gpu_ep_return(g, w.part, seq, stream))) return st;
    return k3gpu_ep_combine(g, out, w.pos, T, seq, ok, stream);
}
