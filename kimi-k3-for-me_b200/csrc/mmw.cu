// mmw.cu -- the bf16 trunk matmul of a verify sweep on tcgen05:
//   Y[t][o] = sum_i W[o][i] * X[t][i],  W bf16 [out][in], X fp32 [T][in], Y fp32 [T][out]
// (k3_matmul_bf16_batch_ld, src/core/k3_ops.c:953, tiles :700-937; the reference takes each
// product in double and its sums in a fixed 16-accumulator order).
//
// The activations are split exactly enough into two bf16 pieces, hi = bf16(x) and
// lo = bf16(x - hi) (x = hi + lo to 2^-17 relative; only hi when x is already bf16), and
// the products W * piece are exact in the tensor core's fp32 accumulator. The sums run in
// that accumulator over the K range of a unit, so results agree with the reference's
// double sums to about 1e-5 relative (the sweep's logits tolerance is 1e-3 rel-L2).
//
// A chain sweep has T <= 128 positions: every output row block is a weight stream; a tree
// sweep over a batch (T ~ 1024) is a real GEMM. One persistent CTA per SM walks units (128
// output rows x one tile of at most 128 positions x one K split; one tile when T <= 128,
// else T split into equal tiles), 7 warps:
//   warp 0     TMA: a 64-K stage = one 128-byte-swizzled box of 128 weight rows (16 KB)
//              and one box per activation piece (Np rows, Np = the tile rounded up to 16)
//   warps 1-2  MMA issuers: issuer i owns K16 steps 2i, 2i+1 of every stage and its own
//              fp32 accumulator in TMEM (two issuers: one thread issues an MMA about every
//              55-75 clocks); tcgen05.mma kind::f16 with bf16 A and B from shared memory
//   warps 3-6  epilogue: tcgen05.ld of both accumulators at the end of a unit, summed,
//              written to Y (one split) or to a split partial that a second kernel sums in
//              split order.
// Every wait is bounded; TMEM is freed on every exit path. No TMA multicast.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"

namespace k3 {
namespace mmw {

constexpr int THREADS = 7 * 32;
constexpr int KB = 64;                    // K per stage: one 128-byte swizzled box row
constexpr int W_BYTES = 128 * 128;        // 128 weight rows x 128 bytes
constexpr int MAX_NS = 8;
constexpr int TILE_T = 128;               // positions per tile when T is larger
constexpr int PASS_T = 2048;              // positions per launch (bounds the workspace)
constexpr int MAX_SPLIT = 8;
constexpr long long SPIN = 1LL << 22;
constexpr int SUSPEND_NS = 1000;

__device__ __forceinline__ uint32_t s_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint32_t b, uint32_t n)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect(uint32_t b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
// bounded: each try may suspend the warp until the phase completes or SUSPEND_NS pass
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t parity)
{
    for (long long i = 0; i < SPIN; i++) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                     " selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(ok)
                     : "r"(b), "r"(parity), "n"(SUSPEND_NS)
                     : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap *m, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// K-major, 128-byte swizzle shared-memory descriptor: start, LBO 16 B (unused), SBO 1024 B
// between 8-row groups, version 1, layout SWIZZLE_128B
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: D f32, A bf16, B bf16, both K-major, N, M = 128
__host__ __device__ constexpr uint32_t bf16_idesc(int N)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
}
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

struct Args {
    float *Y;            // [T][ldy] (one split) or nullptr
    float *part;         // [nsplit][T][out] split partials, or nullptr
    const int *lo_flag;  // 1 when some activation needs its lo piece
    int T, Np, in, out, ldy;
    int nsplit, kst;     // K splits; 64-K stages per split
    int ttiles, Tpad;    // position tiles of Np rows; rows of each activation piece
    int n_units, NS, stage_bytes;
    int dbuf;            // Np <= 128: two accumulator sets, so a unit's epilogue overlaps the next unit
    // the fused greedy argmax (one split only): instead of Y, each unit writes its 128-row
    // block's best (value, row) per position to best_v/best_i [T][nrb] and, for row block 0,
    // whether row 0 is NaN to nan0 [T]
    float *best_v;
    int *best_i, *nan0;
    int nrb;
};

// (v, i) beats (bv, bi): a candidate (i >= 0) over none, a larger value, or an equal value
// at a smaller index -- the sequential scan's first maximum
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi)
{
    if (i < 0) return false;
    if (bi < 0) return true;
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(THREADS, 1) mmw_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                                                            const __grid_constant__ CUtensorMap xmap, Args a)
{
    extern __shared__ __align__(1024) unsigned char smem[];
    if ((s_addr(smem) & 1023u) != 0u) {   // never expected: refuse rather than mis-swizzle
        if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)a.NS * a.stage_bytes);
    uint64_t *b_full = bars, *b_empty = bars + MAX_NS, *b_dfull = bars + 2 * MAX_NS, *b_dfree = b_dfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * MAX_NS + 4);
    float *red_v = reinterpret_cast<float *>(tmem_slot + 4);   // fused argmax: [4 warps][16 positions]
    int *red_i = reinterpret_cast<int *>(red_v + 64);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < a.NS; s++) {
            bar_init(s_addr(&b_full[s]), 1);
            bar_init(s_addr(&b_empty[s]), 2);      // both issuers' commits
        }
        for (int d = 0; d < 2; d++) {
            bar_init(s_addr(&b_dfull[d]), 2);      // both issuers, end of a unit
            bar_init(s_addr(&b_dfree[d]), 4);      // the four epilogue warps
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // 512 columns: issuer i's accumulators at column 256 i (+ 128 for the second set)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s_addr(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int P = *a.lo_flag ? 2 : 1;            // activation pieces in use
    const int nkb = (a.in + KB - 1) / KB;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            int item = 0;
            for (int u = blockIdx.x; u < a.n_units && !failed; u += gridDim.x) {
                const int rb = u / (a.nsplit * a.ttiles), tt = (u / a.nsplit) % a.ttiles, ks = u % a.nsplit;
                const int kb1 = min(nkb, (ks + 1) * a.kst);
                for (int kb = ks * a.kst; kb < kb1; kb++, item++) {
                    const int st = item % a.NS;
                    const uint32_t par = (uint32_t)((item / a.NS) & 1);
                    if (!bar_wait(s_addr(&b_empty[st]), par ^ 1u)) { failed = true; break; }
                    unsigned char *sw = smem + (size_t)st * a.stage_bytes;
                    const uint32_t full = s_addr(&b_full[st]);
                    bar_expect(full, (uint32_t)(W_BYTES + P * a.Np * 128));
                    tma2d(s_addr(sw), &wmap, kb * KB, rb * 128, full);
                    for (int p = 0; p < P; p++)
                        tma2d(s_addr(sw + W_BYTES + p * a.Np * 128), &xmap, kb * KB, p * a.Tpad + tt * a.Np, full);
                }
            }
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (warp <= 2) {
        if (lane == 0) {
            const int i = warp - 1;
            const uint32_t idesc = bf16_idesc(a.Np);
            int item = 0, unit_i = 0;
            for (int u = blockIdx.x; u < a.n_units && !failed; u += gridDim.x, unit_i++) {
                const int ks = u % a.nsplit;
                const int kb1 = min(nkb, (ks + 1) * a.kst);
                const int db = a.dbuf ? (unit_i & 1) : 0, use = a.dbuf ? (unit_i >> 1) : unit_i;
                const uint32_t dt = tmem + (uint32_t)(i * 256 + db * 128);
                // the epilogue has drained this accumulator set's previous unit
                if (!bar_wait(s_addr(&b_dfree[db]), (uint32_t)((use & 1) ^ 1))) { failed = true; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                uint32_t acc = 0;
                for (int kb = ks * a.kst; kb < kb1; kb++, item++) {
                    const int st = item % a.NS;
                    const uint32_t par = (uint32_t)((item / a.NS) & 1);
                    if (!bar_wait(s_addr(&b_full[st]), par)) { failed = true; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // one descriptor per stage, advanced by 16-byte offsets (the 14-bit start
                    // field does not carry: shared addresses stay below 256 KB)
                    const uint64_t d0 = sw128_desc(s_addr(smem + (size_t)st * a.stage_bytes));
                    const uint32_t b0 = W_BYTES >> 4, bp = (uint32_t)(a.Np * 128) >> 4;
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const uint32_t tk = (uint32_t)((2 * i + u) * 32) >> 4;
                        mma_ss(dt, d0 + tk, d0 + b0 + tk, idesc, acc);
                        acc = 1;
                        if (P == 2) mma_ss(dt, d0 + tk, d0 + b0 + bp + tk, idesc, 1u);
                    }
                    mma_commit(s_addr(&b_empty[st]));
                }
                if (failed) break;
                mma_commit(s_addr(&b_dfull[db]));
            }
            if (failed) flag(DEV_TIMEOUT);
        }
    } else {
        const int q = warp & 3;                   // TMEM lane quarter of this warp
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int unit_i = 0;
        for (int u = blockIdx.x; u < a.n_units && !failed; u += gridDim.x, unit_i++) {
            const int rb = u / (a.nsplit * a.ttiles), tt = (u / a.nsplit) % a.ttiles, ks = u % a.nsplit;
            const int row = rb * 128 + r;
            const int db = a.dbuf ? (unit_i & 1) : 0, use = a.dbuf ? (unit_i >> 1) : unit_i;
            if (!bar_wait(s_addr(&b_dfull[db]), (uint32_t)(use & 1))) { failed = true; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t dcol = (uint32_t)(db * 128);
            for (int c0 = 0; c0 < a.Np; c0 += 16) {
                uint32_t v0[16], v1[16];
                tmem_ld16(tmem + lane_addr + dcol + (uint32_t)c0, v0);
                tmem_ld16(tmem + lane_addr + 256u + dcol + (uint32_t)c0, v1);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (a.best_v) {
                    // the block's best row per position: each warp over its 32 rows by
                    // shuffles, then warp 0 over the four warps in row order
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float y = __fadd_rn(__uint_as_float(v0[j]), __uint_as_float(v1[j]));
                        float bv = y;
                        int bi = (row < a.out && y == y) ? row : -1;   // NaN is never a candidate
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                        }
                        if (lane == 0) { red_v[q * 16 + j] = bv; red_i[q * 16 + j] = bi; }
                        const int t = tt * a.Np + c0 + j;
                        if (row == 0 && t < a.T) a.nan0[t] = y != y;
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (q == 0 && lane < 16) {
                        float bv = red_v[lane];
                        int bi = red_i[lane];
#pragma unroll
                        for (int w = 1; w < 4; w++)
                            if (am_better(red_v[w * 16 + lane], red_i[w * 16 + lane], bv, bi)) {
                                bv = red_v[w * 16 + lane];
                                bi = red_i[w * 16 + lane];
                            }
                        const int t = tt * a.Np + c0 + lane;
                        if (t < a.T) {
                            a.best_v[(size_t)t * a.nrb + rb] = bv;
                            a.best_i[(size_t)t * a.nrb + rb] = bi;
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    continue;
                }
                if (row < a.out) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int t = tt * a.Np + c0 + j;
                        if (t < a.T) {
                            const float y = __fadd_rn(__uint_as_float(v0[j]), __uint_as_float(v1[j]));
                            if (a.part) a.part[((size_t)ks * a.T + t) * a.out + row] = y;
                            else a.Y[(size_t)t * a.ldy + row] = y;
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(s_addr(&b_dfree[db]));
        }
        if (failed && lane == 0) flag(DEV_TIMEOUT);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// hi/lo bf16 pieces of X, [2][Tpad][in_pad], zero past T and past in; lo_flag = 1 when any
// lo != 0 (one plain store per block that saw one: every writer writes the same value)
__global__ void __launch_bounds__(256) split_kernel(__nv_bfloat16 *__restrict__ xp, int *__restrict__ lo_flag,
                                                   const float *__restrict__ X, int ldx, int T, int Tpad,
                                                   int in, int in_pad, int vec)
{
    // eight columns a thread: two 16-byte loads (vec: X rows 16-byte aligned) and one
    // 16-byte store per piece (in_pad is a multiple of 64, xp 16-byte aligned)
    const int t = blockIdx.y;
    const int k0 = (blockIdx.x * 256 + threadIdx.x) * 8;
    int nz = 0;
    if (k0 < in_pad) {
        float x[8];
        const float *xr = X + (size_t)t * ldx + k0;
        if (vec && t < T && k0 + 8 <= in) {
            const float4 a = *reinterpret_cast<const float4 *>(xr), b = *reinterpret_cast<const float4 *>(xr + 4);
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = (t < T && k0 + i < in) ? xr[i] : 0.0f;
        }
        __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            hi[i] = __float2bfloat16_rn(x[i]);
            lo[i] = __float2bfloat16_rn(__fsub_rn(x[i], __bfloat162float(hi[i])));
            nz |= __bfloat16_as_ushort(lo[i]) & 0x7FFF;
        }
        *reinterpret_cast<uint4 *>(xp + (size_t)t * in_pad + k0) = *reinterpret_cast<const uint4 *>(hi);
        *reinterpret_cast<uint4 *>(xp + ((size_t)Tpad + t) * in_pad + k0) = *reinterpret_cast<const uint4 *>(lo);
    }
    if (__syncthreads_or(nz) && threadIdx.x == 0) *lo_flag = 1;
}

// The fused argmax's second half: one warp per position merges the row blocks' bests
// (blocks in ascending order hold ascending rows, so the first maximum wins on ties) and
// applies the sequential scan's rule for a NaN at row 0: arg = 0 (no value compares greater
// than NaN), as when every value is NaN.
__global__ void __launch_bounds__(256) argmax_merge_kernel(int *__restrict__ arg, const float *__restrict__ best_v,
                                                           const int *__restrict__ best_i,
                                                           const int *__restrict__ nan0, int T, int nrb)
{
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    float bv = 0.0f;
    int bi = -1;
    for (int b = lane; b < nrb; b += 32) {
        const float v = best_v[(size_t)t * nrb + b];
        const int i = best_i[(size_t)t * nrb + b];
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) arg[t] = (nan0[t] || bi < 0) ? 0 : bi;
}

// Y[t][o] = sum over splits in order; block (x, t) covers 4 * 256 outputs of row t
__global__ void __launch_bounds__(256) reduce_kernel(float *__restrict__ Y, const float *__restrict__ part,
                                                    int T, int out, int ldy, int nsplit)
{
    const int t = blockIdx.y;
    const int o = (blockIdx.x * 256 + threadIdx.x) * 4;
    if (o >= out) return;
    const size_t plane = (size_t)T * out;
    const float *src = part + (size_t)t * out + o;
    float *dst = Y + (size_t)t * ldy + o;
    if (o + 4 <= out && (out & 3) == 0 && (ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(Y) & 15u) == 0) {
        float4 y = *reinterpret_cast<const float4 *>(src);
        for (int s = 1; s < nsplit; s++) {
            const float4 v = *reinterpret_cast<const float4 *>(src + s * plane);
            y.x = __fadd_rn(y.x, v.x); y.y = __fadd_rn(y.y, v.y);
            y.z = __fadd_rn(y.z, v.z); y.w = __fadd_rn(y.w, v.w);
        }
        *reinterpret_cast<float4 *>(dst) = y;
    } else {
        for (int j = 0; j < 4 && o + j < out; j++) {
            float y = src[j];
            for (int s = 1; s < nsplit; s++) y = __fadd_rn(y, src[s * plane + j]);
            dst[j] = y;
        }
    }
}

// ---- host ----------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(q);
    });
    return fn;
}

static int bf16_map(CUtensorMap *m, const void *base, long long cols, long long rows, int box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return K3GPU_ECUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {(cuuint32_t)KB, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        g_last_cuda_error = (int)r;
        return K3GPU_ECUDA;
    }
    return K3GPU_OK;
}

struct Plan {
    int Np, ttiles, Tpad, in_pad, nkb, nsplit, kst, rowblocks, n_units;
    size_t xp_bytes, part_bytes;
};

// One launch over Tc <= PASS_T positions; at most max_split K splits.
static Plan plan(int Tc, int in, int out, int sms, int max_split)
{
    Plan p;
    p.ttiles = Tc <= TILE_T ? 1 : (Tc + TILE_T - 1) / TILE_T;
    p.Np = ((Tc + p.ttiles - 1) / p.ttiles + 15) / 16 * 16;
    p.Tpad = p.ttiles * p.Np;
    p.in_pad = (in + KB - 1) / KB * KB;
    p.nkb = p.in_pad / KB;
    p.rowblocks = (out + 127) / 128;
    // K splits: minimise the busiest CTA's stages (units are handed out round-robin), with
    // a cost per unit (accumulator drain) and, when split, the partial-sum pass
    const int max_ns = std::max(1, std::min(max_split, p.nkb / 4));
    double best = 1e300;
    p.kst = p.nkb;
    for (int ns = 1; ns <= max_ns; ns++) {
        const int kst = (p.nkb + ns - 1) / ns;
        const int nsr = (p.nkb + kst - 1) / kst;
        const long long per_cta = ((long long)p.rowblocks * p.ttiles * nsr + sms - 1) / sms;
        double cost = (double)per_cta * (kst + 2.0);
        if (nsr > 1) cost += 3.0 + (double)nsr * Tc * out * 4.0 / 2.5e6;   // stage ~ 0.45 us
        if (cost < best - 1e-9) { best = cost; p.kst = kst; }
    }
    p.nsplit = (p.nkb + p.kst - 1) / p.kst;                    // every split non-empty
    p.n_units = p.rowblocks * p.ttiles * p.nsplit;
    p.xp_bytes = (size_t)2 * p.Tpad * p.in_pad * 2;
    p.part_bytes = p.nsplit > 1 ? (size_t)p.nsplit * Tc * out * 4 : 0;
    return p;
}

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

static int g_attr_dev = -1;
static std::mutex g_attr_mu;

}  // namespace mmw
}  // namespace k3

extern "C" size_t k3gpu_matmul_bf16_workspace(int T, int in, int out)
{
    using namespace k3::mmw;
    if (T <= 0 || in <= 0 || out <= 0) return 0;
    // the largest pass and, when T is not a multiple of it, the last one
    size_t xp = 0, part = 0;
    for (int Tc : {std::min(T, PASS_T), T % PASS_T}) {
        if (Tc <= 0) continue;
        const Plan p = plan(Tc, in, out, 148, MAX_SPLIT);
        xp = std::max(xp, p.xp_bytes);
        part = std::max(part, p.part_bytes);
    }
    return align256(xp) + align256(part) + 256;
}

// The bf16 trunk matmul over T positions in launches of PASS_T; with arg set, the lm_head
// fused with the greedy argmax (one K split, no Y): arg [T] receives each position's first
// maximum, the row blocks' bests staged in the workspace after the activation pieces.
static int matmul_run(float *Y, int ldy, const float *X, int ldx, const uint16_t *W, int in, int out, int T,
                      void *workspace, size_t ws_bytes, cudaStream_t s, int *arg)
{
    using namespace k3::mmw;
    int dev = 0, st = k3::cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    {
        std::lock_guard<std::mutex> lock(g_attr_mu);
        if (g_attr_dev != dev) {
            st = k3::cuda_status(cudaFuncSetAttribute(mmw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      220 * 1024));
            if (st) return st;
            g_attr_dev = dev;
        }
    }
    char *ws = static_cast<char *>(workspace);
    CUtensorMap wm;
    if ((st = bf16_map(&wm, W, in, out, 128))) return st;
    const int nrb = (out + 127) / 128;
    for (int t0 = 0; t0 < T; t0 += PASS_T) {           // launches of up to PASS_T positions
        const int Tc = std::min(PASS_T, T - t0);
        // the K splits this workspace holds partials for (the SM count may differ from the
        // one the workspace query assumed); one split when the argmax is fused
        const size_t xp_b = align256(plan(Tc, in, out, sms, 1).xp_bytes);
        const size_t room = ws_bytes - 256 - xp_b;
        const int max_split = arg ? 1 : (int)std::max<size_t>(1, std::min<size_t>(MAX_SPLIT, room / ((size_t)Tc * out * 4)));
        const Plan p = plan(Tc, in, out, sms, max_split);
        __nv_bfloat16 *xp = reinterpret_cast<__nv_bfloat16 *>(ws);
        float *part = reinterpret_cast<float *>(ws + xp_b);
        // the flag sits in the last 256 bytes, past any partials this launch writes
        int *lo_flag = reinterpret_cast<int *>((reinterpret_cast<uintptr_t>(ws + ws_bytes - 256) + 15) & ~(uintptr_t)15);
        if ((st = k3::cuda_status(cudaMemsetAsync(lo_flag, 0, sizeof(int), s)))) return st;
        const float *Xt = X + (size_t)t0 * ldx;
        const int vec = (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(Xt) & 15u) == 0;
        split_kernel<<<dim3((p.in_pad + 2047) / 2048, p.Tpad), 256, 0, s>>>(xp, lo_flag, Xt, ldx, Tc, p.Tpad, in,
                                                                           p.in_pad, vec);
        if ((st = k3::launch_status())) return st;
        CUtensorMap xm;
        if ((st = bf16_map(&xm, xp, p.in_pad, 2LL * p.Tpad, p.Np))) return st;
        Args a;
        a.Y = (!arg && p.nsplit == 1) ? Y + (size_t)t0 * ldy : nullptr;
        a.part = (!arg && p.nsplit > 1) ? part : nullptr;
        a.best_v = arg ? reinterpret_cast<float *>(ws + xp_b) : nullptr;
        a.best_i = arg ? reinterpret_cast<int *>(ws + xp_b + align256((size_t)Tc * nrb * 4)) : nullptr;
        a.nan0 = arg ? reinterpret_cast<int *>(ws + xp_b + 2 * align256((size_t)Tc * nrb * 4)) : nullptr;
        a.nrb = nrb;
        a.lo_flag = lo_flag;
        a.T = Tc; a.Np = p.Np; a.in = in; a.out = out; a.ldy = ldy;
        a.nsplit = p.nsplit; a.kst = p.kst; a.n_units = p.n_units;
        a.ttiles = p.ttiles; a.Tpad = p.Tpad;
        a.dbuf = p.Np <= 128 ? 1 : 0;
        a.stage_bytes = W_BYTES + 2 * p.Np * 128;
        a.NS = std::min(MAX_NS, (200 * 1024) / a.stage_bytes);
        // at least 120 KB, so one CTA per SM: each allocates all 512 TMEM columns
        const int smem = std::max(120 * 1024, a.NS * a.stage_bytes + (2 * MAX_NS + 4) * 8 + 16 + 512);
        mmw_tc_kernel<<<std::min(p.n_units, sms), THREADS, smem, s>>>(wm, xm, a);
        if ((st = k3::launch_status())) return st;
        if (arg) {
            argmax_merge_kernel<<<(unsigned)((Tc + 7) / 8), 256, 0, s>>>(arg + t0, a.best_v, a.best_i, a.nan0, Tc, nrb);
            if ((st = k3::launch_status())) return st;
        } else if (p.nsplit > 1) {
            reduce_kernel<<<dim3((unsigned)((out + 1023) / 1024), (unsigned)Tc), 256, 0, s>>>(
                Y + (size_t)t0 * ldy, part, Tc, out, ldy, p.nsplit);
            if ((st = k3::launch_status())) return st;
        }
    }
    return K3GPU_OK;
}

extern "C" int k3gpu_matmul_bf16_batch(float *Y, int ldy, const float *X, int ldx, const uint16_t *W, int in,
                                       int out, int T, void *workspace, size_t ws_bytes, void *stream)
{
    if (!Y || !X || !W || !workspace || T <= 0 || in <= 0 || out <= 0) return K3GPU_EINVAL;
    if (in % 8 || ldy < out || ldx < in || (reinterpret_cast<uintptr_t>(W) & 15u)) return K3GPU_EINVAL;
    if (reinterpret_cast<uintptr_t>(workspace) & 15u) return K3GPU_EINVAL;   // the pieces are stored 16 bytes at a time
    if (ws_bytes < k3gpu_matmul_bf16_workspace(T, in, out)) return K3GPU_ECAPACITY;
    return matmul_run(Y, ldy, X, ldx, W, in, out, T, workspace, ws_bytes, k3::as_stream(stream), nullptr);
}

extern "C" size_t k3gpu_lm_head_argmax_workspace(int T, int in, int vocab)
{
    using namespace k3::mmw;
    if (T <= 0 || in <= 0 || vocab <= 0) return 0;
    const int Tc = std::min(T, PASS_T), nrb = (vocab + 127) / 128;
    return align256(plan(Tc, in, vocab, 148, 1).xp_bytes) + 2 * align256((size_t)Tc * nrb * 4) +
           align256((size_t)Tc * 4) + 256;
}

extern "C" int k3gpu_lm_head_argmax(int *arg, const float *X, int ldx, const uint16_t *W, int in, int vocab, int T,
                                    void *workspace, size_t ws_bytes, void *stream)
{
    if (!arg || !X || !W || !workspace || T <= 0 || in <= 0 || vocab <= 0) return K3GPU_EINVAL;
    if (in % 8 || ldx < in || (reinterpret_cast<uintptr_t>(W) & 15u)) return K3GPU_EINVAL;
    if (reinterpret_cast<uintptr_t>(workspace) & 15u) return K3GPU_EINVAL;
    if (ws_bytes < k3gpu_lm_head_argmax_workspace(T, in, vocab)) return K3GPU_ECAPACITY;
    return matmul_run(nullptr, vocab, X, ldx, W, in, vocab, T, workspace, ws_bytes, k3::as_stream(stream), arg);
}
