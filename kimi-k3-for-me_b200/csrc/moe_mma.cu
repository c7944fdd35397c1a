// moe_mma.cu -- the tensor-core expert FFN for verify batches (the routed half of
// k3_moe_prefill, src/core/k3_ops.c:2058-2132 of the reference, plus shared experts).
//
// Why this shape. A verify step routes B*(1+k) tokens to top-8 of 384 experts, so most
// active experts see one or two tokens and every weight byte is read once: the kernel is
// HBM-bound, and the work per byte is the decode of two E2M1 nibbles. Doing the multiply
// on the tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate) leaves the CUDA cores
// with one hardware conversion per byte (cvt.rn.f16x2.e2m1x2, exact) and a per-group
// scale, which is what lets the stream run at HBM speed.
//
// Tiles. A CTA unit is 128 weight rows of one expert: for gate/up 64 rows of w1 and the
// same 64 rows of w3, for down 128 rows of w2. Each of the eight consumer warps owns one
// m16 tile of the unit (gate/up: 8 w1 rows stacked on the matching 8 w3 rows, so the
// activation runs in-thread) over the whole K, so no cross-warp reduction is needed.
// Token chunks of 8 ride in the MMA N dimension, two chunks per pass over the weights.
//
// Data movement. One producer warp feeds a ring of shared-memory stages, each a K-chunk
// of 256 elements: the weight rows arrive by one 2D TMA load per matrix (a tensor map
// over the whole bank, 128-byte rows of the box swizzled so the consumers' fragment
// loads hit distinct banks), the token rows of the activations by 1D bulk copies into
// padded rows, and the producer's lanes turn the E8M0 scale bytes into floats in the
// stage. mbarriers count the bytes in (full) and the consumer warps out (empty). Every
// wait is bounded. No TMA multicast anywhere.
//
// Exactness. E2M1 values are exact in f16. Activations enter as an exact f16 hi/lo pair
// with one power-of-two exponent per row (x = (hi + lo) * 2^e, 22 significant bits; the
// lo MMAs and copies are skipped when every lo half of the pass is zero, e.g. for bf16
// inputs). A group's MMAs accumulate from zero and join the running fp32 sum scaled by
// the group's E8M0 power of two; the row exponent is applied in the epilogue.
#include <cuda.h>
#include <cuda_fp16.h>
#include <string.h>

#include <mutex>

#include "moe.cuh"

namespace k3 {

constexpr int MM_CWARPS = 8;
constexpr int MM_THREADS = (MM_CWARPS + 1) * 32;
constexpr int MM_ROWS = 128;                 // weight rows per unit
constexpr int MM_KC = 512;                   // K elements per stage (256 packed bytes)
constexpr int MM_GS = MM_KC / 32;            // groups per stage (16 scale bytes per row)
constexpr int MM_MAXCH = 2;                  // 8-token chunks per pass
constexpr int MM_BROW = 1088;                // padded bytes of one activation row (1024 + 64)
constexpr int MM_W_BYTES = MM_ROWS * 256;    // 32 KB: four (or two) swizzled 128-byte-wide boxes
constexpr int MM_S_BYTES = MM_ROWS * 16;     // 2 KB of E8M0 bytes
constexpr int MM_B_BYTES = MM_MAXCH * 8 * MM_BROW;   // one of hi / lo
constexpr int MM_STAGE = ((MM_W_BYTES + MM_S_BYTES + 2 * MM_B_BYTES) + 1023) & ~1023;
constexpr int MM_NS = 3;
constexpr int MM_SMEM = MM_NS * MM_STAGE + 1024 /*align slack*/ + 2 * MM_NS * 8;
constexpr long long MM_SPIN = 1LL << 24;     // bounded mbarrier waits (~seconds)

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase: false after MM_SPIN polls (the caller records a
// timeout in the device status word and leaves).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
    for (long long i = 0; i < MM_SPIN; i++) {
        if (mbar_try(bar, parity)) return true;
        if (i > 32) __nanosleep(64);
    }
    return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// four packed bytes (8 E2M1 values) -> four f16x2 words, low nibble in the low half
__device__ __forceinline__ void cvt4(uint32_t w, uint32_t (&h)[4])
{
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(w));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1, float c0, float c1,
                                         float c2, float c3)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

struct MmaArgs {
    int K;          // reduction width of the phase (L for gate/up, I for down)
    int UE;         // units per expert
    // Row coordinates in the tensor maps of expert 0's first row of each matrix; expert e
    // adds e * (its run's rows). Weights map: rows of K/2 packed bytes; scales map: rows
    // of K/32 bytes.
    long long wy1, wy3, wys;   // weights: w1 (or w2), w3, rows per run
    long long sy1, sy3, sys;   // scales:  s1 (or s2), s3, rows per run
    const uint8_t *skip;       // per expert: 1 = run by the tcgen05 kernels instead (or NULL)
};

// Stage layout (1024-aligned):
//   [0, 32K)    weights: four 8 KB boxes (gate/up: w1 lo-K, w1 hi-K, w3 lo-K, w3 hi-K, 64
//               rows x 128 B each) or two 16 KB boxes (down: w2 lo-K, hi-K, 128 rows),
//               128-byte swizzled
//   [32K, 34K)  E8M0 bytes, 16 per row (gate/up: 64 w1 rows then 64 w3 rows)
//   then B hi [MAXCH*8 rows][MM_BROW] and B lo, the activation rows of the pass
template <int PHASE>   // 0 = gate/up (activation fused), 1 = down
__global__ void __launch_bounds__(MM_THREADS, 1) moe_mma_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                const __grid_constant__ CUtensorMap smap,
                                                                MoePlan p, K3GpuExpertBank bank,
                                                                MmaArgs ma, int act, float b1, float b2)
{
    // declared 1024-aligned (the 128-byte TMA swizzle repeats every 1024 bytes) and used
    // as is, so every access below stays a shared-memory access
    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_addr(smem) & 1023u) != 0u) {   // never expected: refuse rather than mis-swizzle
        if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
        return;
    }
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)MM_NS * MM_STAGE);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < MM_NS; s++) {
            mbar_init(smem_addr(&bars[s]), 1);                  // full: the expect_tx arrive
            mbar_init(smem_addr(&bars[MM_NS + s]), MM_CWARPS);  // empty: consumer warps
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int K = ma.K, NK = K / MM_KC;
    const int n_units = *p.n_active * ma.UE;
    const __half *Xh = PHASE == 0 ? p.zh : p.hh;
    const __half *Xl = PHASE == 0 ? p.zl : p.hl;
    const int *Xe = PHASE == 0 ? p.ze : p.he;
    const int *Xf = PHASE == 0 ? p.zf : p.hf;

    if (warp == MM_CWARPS) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&smap) : "memory");
        }
        int item = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
            const int e = p.act[u / ma.UE], ub = u % ma.UE;
            if (ma.skip && ma.skip[e]) continue;
            const int nt = p.cnt[e], q0 = p.off[e];
            for (int tb = 0; tb < nt; tb += 8 * MM_MAXCH) {
                const int npt = min(8 * MM_MAXCH, nt - tb);          // tokens this pass
                int row = -1;                                        // lane's token row
                if (lane < npt) row = q0 + tb + lane;
                const bool lo_any = __any_sync(0xffffffffu, row >= 0 && Xf[row] != 0);
                const uint32_t bbytes = (uint32_t)npt * 1024u * (lo_any ? 2u : 1u);
                for (int kc = 0; kc < NK; kc++, item++) {
                    const int st = item % MM_NS;
                    const uint32_t par = (uint32_t)((item / MM_NS) & 1);
                    const uint32_t full = smem_addr(&bars[st]), empty = smem_addr(&bars[MM_NS + st]);
                    if (!mbar_wait(empty, par ^ 1u)) {
                        if (lane == 0) flag(DEV_TIMEOUT);
                        for (int back = 1; back < MM_NS && back <= item; back++) {   // drain
                            const int it = item - back;
                            mbar_wait(smem_addr(&bars[it % MM_NS]), (uint32_t)((it / MM_NS) & 1));
                        }
                        return;
                    }
                    unsigned char *sw = smem + (size_t)st * MM_STAGE;
                    unsigned char *ssb = sw + MM_W_BYTES;
                    unsigned char *sbh = ssb + MM_S_BYTES;
                    unsigned char *sbl = sbh + MM_B_BYTES;
                    if (lane == 0) {
                        mbar_expect_tx(full, (uint32_t)(MM_W_BYTES + MM_S_BYTES) + bbytes);
                        const int x0 = kc * 256, xs = kc * 16;
                        if (PHASE == 0) {
                            const int y1 = (int)(e * ma.wys + ma.wy1 + ub * 64);
                            const int y3 = (int)(e * ma.wys + ma.wy3 + ub * 64);
                            tma_2d(smem_addr(sw), &wmap, x0, y1, full);
                            tma_2d(smem_addr(sw + 8192), &wmap, x0 + 128, y1, full);
                            tma_2d(smem_addr(sw + 16384), &wmap, x0, y3, full);
                            tma_2d(smem_addr(sw + 24576), &wmap, x0 + 128, y3, full);
                            tma_2d(smem_addr(ssb), &smap, xs, (int)(e * ma.sys + ma.sy1 + ub * 64), full);
                            tma_2d(smem_addr(ssb + 1024), &smap, xs, (int)(e * ma.sys + ma.sy3 + ub * 64), full);
                        } else {
                            const int y1 = (int)(e * ma.wys + ma.wy1 + ub * 128);
                            tma_2d(smem_addr(sw), &wmap, x0, y1, full);
                            tma_2d(smem_addr(sw + 16384), &wmap, x0 + 128, y1, full);
                            tma_2d(smem_addr(ssb), &smap, xs, (int)(e * ma.sys + ma.sy1 + ub * 128), full);
                        }
                    }
                    __syncwarp();
                    if (row >= 0) {
                        const size_t src = (size_t)row * K + (size_t)kc * MM_KC;   // elements
                        const uint32_t dsto = (uint32_t)lane * MM_BROW;
                        bulk_g2s(smem_addr(sbh + dsto), Xh + src, 1024u, full);
                        if (lo_any) bulk_g2s(smem_addr(sbl + dsto), Xl + src, 1024u, full);
                    }
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumer warps
    const int g = lane >> 2, t = lane & 3;
    // this warp's tile: A row g and A row g+8, as (box base in the stage, row in the box)
    int aboxa, aboxb, rowa, rowb, sra, srb;
    if (PHASE == 0) {
        rowa = rowb = 8 * warp + g;            // w1 row and the matching w3 row
        aboxa = 0; aboxb = 16384;              // + 8192 for the hi-K box
        sra = rowa; srb = 64 + rowb;           // scale rows
    } else {
        rowa = 16 * warp + g; rowb = 16 * warp + 8 + g;
        aboxa = aboxb = 0;                     // + 16384 for the hi-K box
        sra = rowa; srb = rowb;
    }
    const int hoff = PHASE == 0 ? 8192 : 16384;
    const int offa = aboxa + rowa * 128 + 4 * t, offb = aboxb + rowb * 128 + 4 * t;
    const int swa = rowa & 7, swb = rowb & 7;
    int item = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const int e = p.act[u / ma.UE], ub = u % ma.UE;
        if (ma.skip && ma.skip[e]) continue;
        const int nt = p.cnt[e], q0 = p.off[e];
        for (int tb = 0; tb < nt; tb += 8 * MM_MAXCH) {
            const int npt = min(8 * MM_MAXCH, nt - tb);
            const int nch = (npt + 7) / 8;
            bool mylo = false;
            if (lane < npt) {
                mylo = Xf[q0 + tb + lane] != 0;
            }
            const bool lo_any = __any_sync(0xffffffffu, mylo);
            const bool v0 = g < npt, v1 = 8 + g < npt;   // column g of chunk 0 / 1 is a token
            float D[MM_MAXCH][4];
#pragma unroll
            for (int c = 0; c < MM_MAXCH; c++)
#pragma unroll
                for (int j = 0; j < 4; j++) D[c][j] = 0.0f;

            for (int kc = 0; kc < NK; kc++, item++) {
                const int st = item % MM_NS;
                const uint32_t par = (uint32_t)((item / MM_NS) & 1);
                if (!mbar_wait(smem_addr(&bars[st]), par)) {
                    if (lane == 0) flag(DEV_TIMEOUT);
                    return;
                }
                const unsigned char *sw = smem + (size_t)st * MM_STAGE;
                const unsigned char *ssb = sw + MM_W_BYTES;
                const unsigned char *sbh = ssb + MM_S_BYTES;
                const unsigned char *sbl = sbh + MM_B_BYTES;
                // the 16 E8M0 bytes of rows a and b for this stage
                const uint4 sca = *reinterpret_cast<const uint4 *>(ssb + sra * 16);
                const uint4 scb = *reinterpret_cast<const uint4 *>(ssb + srb * 16);
                const uint32_t swds_a[4] = {sca.x, sca.y, sca.z, sca.w};
                const uint32_t swds_b[4] = {scb.x, scb.y, scb.z, scb.w};
#pragma unroll
                for (int gs = 0; gs < MM_GS; gs++) {
                    const int half = gs >> 3, c8 = gs & 7;
                    const uint32_t wa = *reinterpret_cast<const uint32_t *>(sw + offa + half * hoff + ((c8 ^ swa) << 4));
                    const uint32_t wc = *reinterpret_cast<const uint32_t *>(sw + offb + half * hoff + ((c8 ^ swb) << 4));
                    uint32_t A0[4], A1[4];
                    cvt4(wa, A0);
                    cvt4(wc, A1);
                    // E8M0 -> float: 2^(S-127); 255 (NaN) -> 0. (S = 0 gives 0 here where
                    // the exact value is 2^-127: the products are below 6 * 2^-127 * |x|.)
                    const uint32_t Sa = (swds_a[gs >> 2] >> (8 * (gs & 3))) & 0xFFu;
                    const uint32_t Sb = (swds_b[gs >> 2] >> (8 * (gs & 3))) & 0xFFu;
                    const float s0 = Sa == 255u ? 0.0f : __uint_as_float(Sa << 23);
                    const float s1 = Sb == 255u ? 0.0f : __uint_as_float(Sb << 23);
#pragma unroll
                    for (int c = 0; c < MM_MAXCH; c++) {
                        if (c >= nch) break;
                        const bool valid = c == 0 ? v0 : v1;
                        uint4 bh = make_uint4(0, 0, 0, 0), bl = make_uint4(0, 0, 0, 0);
                        const int boff = (c * 8 + g) * MM_BROW + gs * 64 + 16 * t;
                        if (valid) {
                            bh = *reinterpret_cast<const uint4 *>(sbh + boff);
                            if (lo_any) bl = *reinterpret_cast<const uint4 *>(sbl + boff);
                        }
                        float Cg[4];
                        mma16816(Cg, A0[0], A1[0], A0[1], A1[1], bh.x, bh.y, 0.f, 0.f, 0.f, 0.f);
                        mma16816(Cg, A0[2], A1[2], A0[3], A1[3], bh.z, bh.w, Cg[0], Cg[1], Cg[2], Cg[3]);
                        if (lo_any) {
                            mma16816(Cg, A0[0], A1[0], A0[1], A1[1], bl.x, bl.y, Cg[0], Cg[1], Cg[2], Cg[3]);
                            mma16816(Cg, A0[2], A1[2], A0[3], A1[3], bl.z, bl.w, Cg[0], Cg[1], Cg[2], Cg[3]);
                        }
                        D[c][0] = fmaf(s0, Cg[0], D[c][0]);
                        D[c][1] = fmaf(s0, Cg[1], D[c][1]);
                        D[c][2] = fmaf(s1, Cg[2], D[c][2]);
                        D[c][3] = fmaf(s1, Cg[3], D[c][3]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_addr(&bars[MM_NS + st]));
            }

            // ---- epilogue: thread holds rows g (D[.][0..1]) and g+8 (D[.][2..3]) for the
            // token columns 2t and 2t+1 of each chunk
#pragma unroll
            for (int c = 0; c < MM_MAXCH; c++) {
                if (c >= nch) break;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int tok = tb + 8 * c + 2 * t + j;
                    if (tok >= nt) continue;
                    const int q = q0 + tok;
                    if (PHASE == 0) {
                        const int ex = Xe[q];
                        const float gv = __fmul_rn(D[c][j], pow2f(ex)), uv = __fmul_rn(D[c][2 + j], pow2f(ex));
                        const float hv = act == K3GPU_ACT_SITU ? act_situ(gv, uv, b1, b2) : act_swiglu(gv, uv);
                        p.H[(size_t)q * bank.I + ub * 64 + 8 * warp + g] = hv;
                    } else {
                        const int ex = Xe[q];
                        const size_t o = (size_t)p.pair_dst[q] * bank.L + ub * 128 + 16 * warp + g;
                        p.contrib[o] = __fmul_rn(D[c][j], pow2f(ex));
                        p.contrib[o + 8] = __fmul_rn(D[c][2 + j], pow2f(ex));
                    }
                }
            }
        }
    }
}

// One CTA per row: fp32 [rows][K] -> f16 hi/lo with the row's power-of-two exponent
// (max |x| * 2^-e in [2^14, 2^15)) and a flag for a nonzero lo half. Rows at or past
// *nrows (when given) are skipped.
__global__ void __launch_bounds__(256) act_pack_kernel(__half *__restrict__ hi, __half *__restrict__ lo,
                                                       int *__restrict__ ex, int *__restrict__ lf,
                                                       const float *__restrict__ x, int K,
                                                       const int *__restrict__ nrows,
                                                       const int *__restrict__ pair_exp,
                                                       int *__restrict__ elo)
{
    __shared__ float redm[8];
    __shared__ int redf[8];
    const int row = blockIdx.x;
    if (nrows && row >= *nrows) return;
    const float *xr = x + (size_t)row * K;
    float m = 0.f;
    for (int i = threadIdx.x; i < K; i += 256) m = fmaxf(m, fabsf(xr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) redm[threadIdx.x >> 5] = m;
    __syncthreads();
    m = redm[0];
    for (int w = 1; w < 8; w++) m = fmaxf(m, redm[w]);
    int e = 0;
    if (m > 0.f && m <= 3.4e38f) e = max(-126, min(127, ilogbf(m) - 14));
    int any = 0;
    for (int i = threadIdx.x; i < K; i += 256) {
        const float y = __fmul_rn(xr[i], pow2f(-e));
        const __half h = __float2half_rn(y);
        const __half l = __float2half_rn(y - __half2float(h));
        hi[(size_t)row * K + i] = h;
        lo[(size_t)row * K + i] = l;
        any |= __half_as_ushort(l) != 0;
    }
    any = __any_sync(0xffffffffu, any);
    if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = any;
    __syncthreads();
    if (threadIdx.x == 0) {
        int f = 0;
        for (int w = 0; w < 8; w++) f |= redf[w];
        ex[row] = e;
        lf[row] = f;
        if (f && elo) atomicOr(&elo[pair_exp[row]], 1);
    }
}

// ---- host side --------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// A 2D u8 tensor map over the whole bank with rows of `pitch` bytes and a box of
// box_w bytes x box_rows rows (128-byte swizzle when box_w is 128).
static int make_map(CUtensorMap *m, const K3GpuExpertBank &b, int pitch, int box_w, int box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return K3GPU_ECUDA;
    const unsigned long long bytes = (unsigned long long)b.n_experts * (unsigned long long)b.stride;
    cuuint64_t dims[2] = {(cuuint64_t)pitch, (cuuint64_t)(bytes / (unsigned long long)pitch)};
    cuuint64_t strides[1] = {(cuuint64_t)pitch};
    cuuint32_t box[2] = {(cuuint32_t)box_w, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(b.base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          box_w == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        g_last_cuda_error = (int)r;
        return K3GPU_ECUDA;
    }
    return K3GPU_OK;
}

bool mma_bank_ok(const K3GpuExpertBank &b)
{
    const int L = b.L, I = b.I;
    if (L % 512 || I % 512 || L < 512 || I < 512 || L > 65536 || I > 65536) return false;
    const long long pl = L / 2, pi = I / 2, ql = L / 32, qi = I / 32;
    if (b.stride % pl || b.stride % pi || b.p1 % pl || b.p3 % pl || b.p2 % pi) return false;
    if (b.s1 % ql || b.s3 % ql || b.s2 % qi) return false;
    const unsigned long long rows = (unsigned long long)b.n_experts * (unsigned long long)b.stride / (unsigned long long)qi;
    return rows < (1ull << 31) && ((unsigned long long)b.n_experts * b.stride) / (unsigned long long)ql < (1ull << 31);
}

struct MapCache {
    const uint8_t *base = nullptr;
    int64_t stride = 0;
    int n = 0, L = 0, I = 0, dev = -1;
    CUtensorMap m[4];     // w1/w3 weights, w1/w3 scales, w2 weights, w2 scales
};
static std::mutex g_map_mu;
static MapCache g_map_cache[8];
static int g_map_next = 0;

static int maps_for(const K3GpuExpertBank &b, CUtensorMap (&out)[4])
{
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(g_map_mu);
    for (auto &c : g_map_cache) {
        if (c.base == b.base && c.stride == b.stride && c.n == b.n_experts && c.L == b.L &&
            c.I == b.I && c.dev == dev) {
            for (int i = 0; i < 4; i++) out[i] = c.m[i];
            return K3GPU_OK;
        }
    }
    MapCache &c = g_map_cache[g_map_next++ % 8];
    c.base = nullptr;
    int st = make_map(&c.m[0], b, b.L / 2, 128, 64);
    if (!st) st = make_map(&c.m[1], b, b.L / 32, 16, 64);
    if (!st) st = make_map(&c.m[2], b, b.I / 2, 128, 128);
    if (!st) st = make_map(&c.m[3], b, b.I / 32, 16, 128);
    if (st) return st;
    c.base = b.base; c.stride = b.stride; c.n = b.n_experts; c.L = b.L; c.I = b.I; c.dev = dev;
    for (int i = 0; i < 4; i++) out[i] = c.m[i];
    return K3GPU_OK;
}

static std::mutex g_mma_mu;
static int g_mma_sms[64] = {};   // per device: its SM count once set up, 0 before

void act_pack_rows_launch(const MoePlan &p, int I, int P, int E, cudaStream_t s)
{
    // the pair rows that exist are 0 .. off[E]-1 (<= P); the grid covers every possible
    // pair and the rows past off[E] return at once
    act_pack_kernel<<<P, 256, 0, s>>>(p.hh, p.hl, p.he, p.hf, p.H, I, p.off + E, p.pair_exp, p.elo + E);
}

int mma_phase_launch(int phase, const MoePlan &p, const K3GpuExpertBank &bank, int act, float b1,
                     float b2, cudaStream_t s)
{
    const int L = bank.L, I = bank.I;
    CUtensorMap m[4];
    int st = maps_for(bank, m);
    if (st) return st;
    // once per device: the shared-memory opt-in (a function's attributes belong to each
    // device's context) and the SM count the persistent grid is sized by
    int dev = 0;
    if ((st = cuda_status(cudaGetDevice(&dev)))) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    int sms = 0;
    {
        std::lock_guard<std::mutex> lock(g_mma_mu);
        if (g_mma_sms[dev] == 0) {
            int n = 0;
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
            if (n <= 0) n = 148;
            st = cuda_status(cudaFuncSetAttribute(moe_mma_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, MM_SMEM));
            if (!st) st = cuda_status(cudaFuncSetAttribute(moe_mma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, MM_SMEM));
            if (st) return st;
            g_mma_sms[dev] = n;
        }
        sms = g_mma_sms[dev];
    }
    const long long pl = L / 2, pi = I / 2, ql = L / 32, qi = I / 32;
    MmaArgs a;
    a.skip = bank.f16_safe;
    if (phase == 0) {
        a.K = L; a.UE = I / 64;
        a.wys = bank.stride / pl; a.wy1 = bank.p1 / pl; a.wy3 = bank.p3 / pl;
        a.sys = bank.stride / ql; a.sy1 = bank.s1 / ql; a.sy3 = bank.s3 / ql;
        moe_mma_kernel<0><<<sms, MM_THREADS, MM_SMEM, s>>>(m[0], m[1], p, bank, a, act, b1, b2);
    } else {
        a.K = I; a.UE = L / 128;
        a.wys = bank.stride / pi; a.wy1 = bank.p2 / pi; a.wy3 = 0;
        a.sys = bank.stride / qi; a.sy1 = bank.s2 / qi; a.sy3 = 0;
        moe_mma_kernel<1><<<sms, MM_THREADS, MM_SMEM, s>>>(m[2], m[3], p, bank, a, act, b1, b2);
    }
    return launch_status();
}

}  // namespace k3
