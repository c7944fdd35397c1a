// moe_tc.cu -- the tcgen05 expert FFN: MXFP4 weights decoded straight into tensor memory.
//
// The verify batch's expert GEMM is a weight stream (most experts see one or two of the
// step's tokens), so the work per weight byte must be small. This kernel makes it one
// hardware nibble-pair conversion plus one f16 multiply per two weights:
//
//   TMA       packed E2M1 rows (128-byte swizzled boxes), their E8M0 bytes, and the
//             activation tiles (f16 hi/lo, K-major, 128-byte swizzle) -> shared memory
//   decode    eight warps, one thread per weight row: cvt.rn.f16x2.e2m1x2 (exact), times
//             the group's power of two 2^(S-127) as an f16 (exact for 104 <= S <= 140, which
//             bank_scan certifies per expert), tcgen05.st into a TMEM A buffer
//   MMA       four issuer warps, one K quarter of the stage each: tcgen05.mma kind::f16,
//             A from TMEM (128 rows x 16 K), B from shared memory (K x the pass's 8 token
//             rows, then their 8 lo halves: one N = 16 MMA gives both), fp32 accumulator in
//             TMEM, one per issuer
//   epilogue  four warps: tcgen05.ld of the four stage partials, fp32 sum, row exponent,
//             activation (gate/up) or the contribution store (down)
//
// Shared memory carries only packed bytes and activation tiles; the f16 weights live in
// tensor memory, so the shared-memory bandwidth is not a ceiling. Every wait is bounded;
// TMEM is freed on every exit path. No TMA multicast anywhere.
//
// Units: gate/up = 64 rows of w1 (TMEM lanes 0..63) and the same 64 rows of w3 (lanes
// 64..127) of one expert; down = 128 rows of w2. Up to 8 tokens per pass: a verify step
// gives most experts one to three, and the half-height activation tile leaves room for a
// fourth stage of weights in flight.
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "moe.cuh"

namespace k3 {

constexpr int TC_DEQ_WARPS = 8;          // warps 0..7: decode (two per TMEM lane quarter)
constexpr int TC_EPI_WARP0 = 8;          // warps 8..11: epilogue
constexpr int TC_TMA_WARP = 12;
constexpr int TC_MMA_WARP0 = 13;         // warps 13..: MMA issuers
constexpr int TC_KC = 512;               // K elements per shared-memory stage
constexpr int TC_W_BYTES = 128 * 256;    // packed weights of a stage (32 KB)
constexpr int TC_S_BYTES = 128 * 16;     // E8M0 bytes of a stage

// The pass shape. Sparse (a verify step: most experts see one to three tokens): up to 8
// tokens a pass, four issuers (two per K half of a stage, each its own accumulator and its
// own 128-K A sub-buffer) and four stages -- the weight bytes in flight per SM, not any unit's rate,
// set the stream's pace (at the loaded latency of ~3.4 us, 3 x 32 KB allow ~30 GB/s per
// SM), and the half-height activation tile is what leaves room for the fourth stage.
// Dense (many tokens an expert, e.g. a 64-node tree over 16 sequences: ~21 tokens per
// expert): up to 32 tokens a pass so each weight is decoded once for all of its expert's
// tokens -- the decode, not the tensor pipe, bounds the sparse shape once an expert needs
// several passes -- at the cost of one issuer per K half (an N = 64 MMA keeps the pipe busy
// from one thread, two A sub-buffers per half), and split rings: at 32 tokens a stage's activation tile
// (64 KB of hi and lo rows) is twice its weights, and in one ring a stage's weights stay
// resident until its MMAs finish. Split, the weights and scales (NS stages) return to the
// TMA as soon as the decode warps have read them, and the activation tiles come in K halves
// (NBH slots, their own producer warp) that each half's issuer frees: 96 KB of weights in
// flight per SM instead of 64 KB, over a shorter lifetime.
template <int NP_, int NMMA_, int NA_, int NS_, int TAB_, int NBH_, int SUBS_> struct TcShape {
    static constexpr int NP = NP_;                      // tokens per pass
    static constexpr int N = 2 * NP;                    // MMA N: the pass's hi rows, then their lo rows
    static constexpr int NMMA = NMMA_;                  // issuers: NMMA / 2 per K half
    static constexpr int MPI = 32 / NMMA;               // K16 MMAs per issuer per stage
    static constexpr int NA = NA_;                      // TMEM A buffers (ACOLS columns each)
    static constexpr int NS = NS_;                      // shared-memory stages (split: weight stages)
    static constexpr int NBH = NBH_;                    // split rings: activation half-stage slots
    static constexpr bool SPLIT = NBH_ > 0;
    // a K half's A rows in SUBS sub-buffers (two: 64 columns = 128 K each), so an issuer runs
    // one sub-buffer's MMAs while the decode warps fill the other, and the next stage's decode
    // starts as soon as the first is free: decode and MMA issue overlap instead of taking
    // turns on one buffer per half. Each half owns its sub-buffers (NA = 2 SUBS): buffers
    // that the halves took turns in let one half's decode warps run a rotation ahead of its
    // own issuers and pass a parity wait meant for an earlier phase.
    static constexpr int SUBS = SUBS_;                  // A buffers per K half of a stage
    static constexpr int SUB_STEPS = 16 / SUBS;         // K16 steps per sub-buffer
    static constexpr int ACOLS = 128 / SUBS;
    static constexpr int TAB = TAB_;                    // active-expert entries kept in shared memory
    static constexpr int B_BYTES = (TC_KC / 64) * NP * 128;   // one activation piece of a stage
    static constexpr int STAGE = TC_W_BYTES + TC_S_BYTES + 2 * B_BYTES + 1024 - TC_S_BYTES % 1024;
    // a B atom: 64 K x NP hi rows, then the same rows' lo halves (SBO = 1024 between 8-row
    // groups), so one N = 2 NP MMA yields the hi products in D columns 0..NP-1 and the lo
    // products in NP..2NP-1; without lo halves the upper columns are unused
    static constexpr int ATOM = 2 * NP * 128;
    static constexpr int WSTAGE = TC_W_BYTES + 1024 * ((TC_S_BYTES + 1023) / 1024);   // split: weights + scales
    static constexpr int BHALF = (256 / 64) * ATOM;     // split: the activation atoms of one K half
    static constexpr int RINGS = SPLIT ? NS * WSTAGE + NBH * BHALF : NS * STAGE;
    static constexpr int PW = N;                        // D columns per issuer
    static constexpr int PCOLS = NMMA * PW;             // one stage-partial set
    static constexpr int ACOL0 = 2 * PCOLS;             // first A column
    static constexpr int XCH_BYTES = 64 * NP * 4;       // gate/up exchange in the epilogue
    // barriers: full[NS] empty[NS] (split: bfull[NBH][2] bempty[NBH]) aready[NA][2] afree[NA]
    // pfree[2] (split: pfull[2], the issuers' stage partials final). Every parity wait has
    // one waiter role that sees every phase of its barrier in order: each half owns its A
    // sub-buffers, and the activation slots, which the halves take turns in (3 slots, 2
    // fills an item), have one full barrier PER HALF. On a barrier both halves' fills
    // completed, a waiter running an item ahead could test a parity whose phase still
    // belonged to the other half's earlier fill and pass at once.
    static constexpr int NBAR_RAW = 2 * NS + 3 * NBH + 3 * NA + 2 + (SPLIT ? 2 : 0);
    static constexpr int NBAR = (NBAR_RAW + 1) & ~1;   // keeps the int4 table 16-byte aligned
    // items between two uses of one A buffer (one activation slot) by the same half: its
    // k-th use waits for phase parity (k / PERIOD) & 1 of that half's barrier
    static constexpr int A_PERIOD = 1;                  // a half fills each of its buffers every stage
    static constexpr int B_PERIOD = NBH > 0 ? NBH : 1;
    // after the expert table: the E8M0 byte -> f16x2 scale pair table (256 entries), then
    // the work items' prefix over the active experts (TAB + 1 ints)
    static constexpr int SMEM = RINGS + XCH_BYTES + NBAR * 8 + 16 + TAB * 16 + 256 * 4 + (TAB + 1) * 4;
    // split: one more warp, the activation producer
    static constexpr int THREADS = (TC_MMA_WARP0 + NMMA + (SPLIT ? 1 : 0)) * 32;
    static_assert(ACOL0 + NA * ACOLS <= 512, "TMEM columns");
    static_assert(STAGE % 1024 == 0 && WSTAGE % 1024 == 0 && BHALF % 1024 == 0, "stage alignment");
    static_assert((RINGS + XCH_BYTES + (NBAR + 2) * 8) % 16 == 0, "int4 expert table alignment");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(NMMA == 2 || NMMA == 4, "issuers per K half");
    static_assert(NP == 8 || NP % 16 == 0, "pass width");
    static_assert(NA == 2 * SUBS, "A buffers: each K half owns SUBS of them");
    static_assert(MPI % SUB_STEPS == 0 || SUB_STEPS % MPI == 0, "issuer steps against sub-buffers");
    // issuers of one half that read each sub-buffer (its afree count)
    static constexpr int SUB_READERS = MPI >= SUB_STEPS ? 1 : SUB_STEPS / MPI;
    static_assert(NBH == 0 || NBH % 2 == 1, "activation slots: an odd rotation");
};
using TcSparse = TcShape<8, 4, 4, 4, 512, 0, 2>;
using TcDense = TcShape<32, 2, 4, 3, 512, 3, 2>;
constexpr long long TC_SPIN = 1LL << 22;
constexpr int TC_SUSPEND_NS = 1000;


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
// A bounded wait on an mbarrier phase. Each try lets the hardware suspend the warp until
// the phase completes or TC_SUSPEND_NS pass, so waiting warps (most of the epilogue's time,
// a good part of everyone else's) do not take issue slots from the decode warps beside
// them; TC_SPIN tries bound the whole wait (about 4 s).
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t parity)
{
    for (long long i = 0; i < TC_SPIN; i++) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                     " selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(ok)
                     : "r"(b), "r"(parity), "n"(TC_SUSPEND_NS)
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

__device__ __forceinline__ void cvt4h(uint32_t w, uint32_t (&h)[4])
{
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(w));
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// E8M0 byte -> the f16x2 pair (2^(S-127), 2^(S-127)); exact for 104 <= S <= 140 (the
// range bank_scan certifies); 255 (NaN by the MX spec) -> 0, as the reference.
__device__ __forceinline__ uint32_t scale_h2(uint32_t S)
{
    uint32_t h;
    if (S == 255u) h = 0u;
    else if (S >= 113u) h = (S - 112u) << 10;          // normal f16
    else h = 1u << (S - 103u);                         // subnormal f16, S in 104..112
    return h | (h << 16);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
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

// K-major, 128-byte swizzle shared-memory matrix descriptor (tcgen05 version 1): start
// address, leading offset 16 B (unused for this layout), stride 1024 B between 8-row
// groups, layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A f16, B f16, both K-major, N, M = 128.
__host__ __device__ constexpr uint32_t f16_idesc(int N)
{
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

struct TcArgs {
    int K;              // reduction width (L for gate/up, I for down)
    int UE;             // units per expert
    long long wy1, wy3, wys;   // weights map: first w1 (w2) row, first w3 row, rows per run
    long long sy1, sy3, sys;   // scales map: same for the E8M0 rows
    const uint8_t *safe;       // per-expert: 1 when every scale byte is in 104..140 or 255
};

template <int PHASE, class CF>   // PHASE 0 = gate/up (activation fused), 1 = down; CF the pass shape
__global__ void __launch_bounds__(CF::THREADS, 1) moe_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                                                               const __grid_constant__ CUtensorMap smap,
                                                               const __grid_constant__ CUtensorMap bhmap,
                                                               const __grid_constant__ CUtensorMap blmap,
                                                               MoePlan p, K3GpuExpertBank bank, TcArgs ta,
                                                               int act, float b1, float b2)
{
    // declared 1024-aligned (the 128-byte TMA swizzle repeats every 1024 bytes) and used
    // as is, so every access below stays a shared-memory access
    extern __shared__ __align__(1024) unsigned char smem[];
    if ((s_addr(smem) & 1023u) != 0u) {   // never expected: refuse rather than mis-swizzle
        if (threadIdx.x == 0) flag(DEV_BAD_INDEX);
        return;
    }
    float *xch = reinterpret_cast<float *>(smem + (size_t)CF::RINGS);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)CF::RINGS + CF::XCH_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + CF::NBAR);
    int4 *tab = reinterpret_cast<int4 *>(bars + CF::NBAR + 2);   // [CF::TAB] {e, cnt, off, flags}
    uint32_t *stab = reinterpret_cast<uint32_t *>(tab + CF::TAB);   // [256] scale_h2 of each byte
    uint64_t *b_full = bars, *b_empty = bars + CF::NS;   // split: the weight ring
    uint64_t *b_bfull = bars + 2 * CF::NS;                // split: the activation ring, [slot][half]
    uint64_t *b_bempty = b_bfull + 2 * CF::NBH;           // [slot]
    uint64_t *b_aready = b_bempty + CF::NBH;              // [A buffer][half]
    uint64_t *b_afree = b_aready + 2 * CF::NA;            // [A buffer]
    uint64_t *b_pfree = b_afree + CF::NA;                 // partial buffers: epilogue -> MMA
    uint64_t *b_pfull = b_pfree + 2;                      // split: partial buffers: MMA -> epilogue
    // a stage's weights (and, in one ring, its activation tile) and a split activation slot
    auto wstage = [&](int st) { return smem + (size_t)st * (CF::SPLIT ? CF::WSTAGE : CF::STAGE); };
    auto bslot = [&](int b) { return smem + (size_t)CF::NS * CF::WSTAGE + (size_t)b * CF::BHALF; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < CF::NS; s++) {
            bar_init(s_addr(&b_full[s]), 1);
            // decode warps (+ the MMA commits when the stage also holds the activations)
            bar_init(s_addr(&b_empty[s]), TC_DEQ_WARPS + (CF::SPLIT ? 0 : CF::NMMA));
        }
        for (int b = 0; b < CF::NBH; b++) {
            bar_init(s_addr(&b_bfull[2 * b]), 1);
            bar_init(s_addr(&b_bfull[2 * b + 1]), 1);
            bar_init(s_addr(&b_bempty[b]), CF::NMMA / 2);       // commits of the filling half's issuers
        }
        for (int a = 0; a < CF::NA; a++) {
            bar_init(s_addr(&b_aready[2 * a]), 4);              // the four decode warps of K half 0
            bar_init(s_addr(&b_aready[2 * a + 1]), 4);          // ... of K half 1
            bar_init(s_addr(&b_afree[a]), CF::SUB_READERS);     // commits of the issuers that read it
        }
        for (int d = 0; d < 2; d++) {
            bar_init(s_addr(&b_pfree[d]), 4);                   // epilogue warps
            if (CF::SPLIT) bar_init(s_addr(&b_pfull[d]), CF::NMMA);   // every issuer's commit
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the active experts of this call, once per CTA: {expert, tokens, first pair, flags}
    // with flags bit 0 = some input row has a lo half, bit 1 = left to the mma.sync path
    const int na = *p.n_active;
    for (int a = tid; a < na && a < CF::TAB; a += CF::THREADS) {
        const int e = p.act[a];
        const int lo = p.elo[(PHASE == 0 ? 0 : bank.n_experts) + e];
        const int skip = (ta.safe && !ta.safe[e]) ? 2 : 0;
        tab[a] = make_int4(e, p.cnt[e], p.off[e], (lo ? 1 : 0) | skip);
    }
    for (int b = tid; b < 256; b += CF::THREADS)   // only certified bytes are ever looked up
        stab[b] = (b == 255 || (b >= 104 && b <= 140)) ? scale_h2((uint32_t)b) : 0u;
    // Work items: one per (expert, unit, pass of NP tokens), expert-major, so an expert with
    // many tokens (the shared expert sees every token of the call) spreads its passes over
    // as many CTAs as other experts' units instead of lengthening the CTAs that drew its
    // units; a unit's passes are consecutive items, run side by side on neighbouring CTAs,
    // so its weights come from HBM once and from L2 for the others. wpre[a] = the first item
    // of active expert a (experts left to the mma.sync kernel have none). Past TAB active
    // experts the items fall back to one per (expert, unit) with all its passes.
    int *wpre = reinterpret_cast<int *>(stab + 256);
    const bool by_pass = na <= CF::TAB;
    if (by_pass && warp == 0) {
        __syncwarp();
        const int per = (na + 31) / 32, a0 = min(na, lane * per), a1 = min(na, a0 + per);
        int sum = 0;
        for (int a = a0; a < a1; a++) {
            const int e = p.act[a];
            const bool skip = ta.safe && !ta.safe[e];
            sum += skip ? 0 : ta.UE * ((p.cnt[e] + CF::NP - 1) / CF::NP);
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int run = incl - sum;   // items before this lane's first expert
        for (int a = a0; a < a1; a++) {
            wpre[a] = run;
            const int e = p.act[a];
            const bool skip = ta.safe && !ta.safe[e];
            run += skip ? 0 : ta.UE * ((p.cnt[e] + CF::NP - 1) / CF::NP);
        }
        if (lane == 31) wpre[na] = incl;
        __syncwarp();   // warp 0 converged again before its tcgen05.alloc (a .sync.aligned op)
    }
    if (warp == 0) {   // 512 TMEM columns: partial sets at 0 and 64, A buffers from 128
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s_addr(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    const int K = ta.K, NK = K / TC_KC;
    const int n_work = by_pass ? wpre[na] : na * ta.UE;
    const int *Xe = PHASE == 0 ? p.ze : p.he;
    bool failed = false;
    // work item w -> active expert a, unit ub, passes [p0, p1)
    auto work_of = [&](int w, int &a, int &ub, int &p0, int &p1) {
        if (!by_pass) {
            a = w / ta.UE;
            ub = w % ta.UE;
            p0 = 0;
            p1 = 1 << 30;
            return;
        }
        int lo = 0, hi = na - 1;   // the last a with wpre[a] <= w
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (wpre[mid] <= w) lo = mid;
            else hi = mid - 1;
        }
        a = lo;
        const int local = w - wpre[a], np = (wpre[a + 1] - wpre[a]) / ta.UE;
        ub = local / np;
        p0 = local % np;
        p1 = p0 + 1;
    };

// the work item/pass/stage sequence every role walks identically
#define TC_FOR_UNITS(...)                                                                   \
    {                                                                                        \
        int item = 0;                                                                        \
        for (int w = blockIdx.x; w < n_work && !failed; w += gridDim.x) {                   \
            int a_, ub, p0_, p1_;                                                            \
            work_of(w, a_, ub, p0_, p1_);                                                    \
            const int4 ent = unit_entry(a_);                                                 \
            if (ent.w & 2) continue;                                                         \
            const int e = ent.x, nt = ent.y, q0 = ent.z;                                     \
            const bool lo_any = (ent.w & 1) != 0;                                            \
            (void)e; (void)q0; (void)lo_any;   /* not every role reads them */                \
            const int tb_end = (int)min((long long)nt, (long long)p1_ * CF::NP);             \
            for (int tb = p0_ * CF::NP; tb < tb_end && !failed; tb += CF::NP) {              \
                const int npt = min(CF::NP, nt - tb);                                         \
                __VA_ARGS__                                                                  \
            }                                                                                \
        }                                                                                    \
    }
    auto unit_entry = [&](int a) -> int4 {
        if (a < CF::TAB) return tab[a];
        const int e = p.act[a];
        const int lo = p.elo[(PHASE == 0 ? 0 : bank.n_experts) + e];
        return make_int4(e, p.cnt[e], p.off[e], (lo ? 1 : 0) | ((ta.safe && !ta.safe[e]) ? 2 : 0));
    };

    if (warp == TC_TMA_WARP) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&smap) : "memory");
            TC_FOR_UNITS({
                for (int kc = 0; kc < NK && !failed; kc++, item++) {
                    const int st = item % CF::NS;
                    const uint32_t par = (uint32_t)((item / CF::NS) & 1);
                    if (!bar_wait(s_addr(&b_empty[st]), par ^ 1u)) { failed = true; break; }
                    unsigned char *sw = wstage(st);
                    unsigned char *ssb = sw + TC_W_BYTES;
                    unsigned char *sbh = sw + TC_W_BYTES + 1024 * ((TC_S_BYTES + 1023) / 1024);
                    const uint32_t full = s_addr(&b_full[st]);
                    bar_expect(full, (uint32_t)(TC_W_BYTES + TC_S_BYTES + (CF::SPLIT ? 0 : CF::B_BYTES * (lo_any ? 2 : 1))));
                    const int x0 = kc * 256, xs = kc * 16;
                    if (PHASE == 0) {
                        const int y1 = (int)(e * ta.wys + ta.wy1 + ub * 64), y3 = (int)(e * ta.wys + ta.wy3 + ub * 64);
                        tma2d(s_addr(sw), &wmap, x0, y1, full);
                        tma2d(s_addr(sw + 8192), &wmap, x0 + 128, y1, full);
                        tma2d(s_addr(sw + 16384), &wmap, x0, y3, full);
                        tma2d(s_addr(sw + 24576), &wmap, x0 + 128, y3, full);
                        tma2d(s_addr(ssb), &smap, xs, (int)(e * ta.sys + ta.sy1 + ub * 64), full);
                        tma2d(s_addr(ssb + 1024), &smap, xs, (int)(e * ta.sys + ta.sy3 + ub * 64), full);
                    } else {
                        const int y1 = (int)(e * ta.wys + ta.wy1 + ub * 128);
                        tma2d(s_addr(sw), &wmap, x0, y1, full);
                        tma2d(s_addr(sw + 16384), &wmap, x0 + 128, y1, full);
                        tma2d(s_addr(ssb), &smap, xs, (int)(e * ta.sys + ta.sy1 + ub * 128), full);
                    }
                    // activation tiles: 8 atoms of 64 K x 16 pair rows (rows past the expert
                    // belong to the next one or lie past the tensor: those columns are
                    // never read back; out-of-range rows are filled with zeros)
                    for (int a = 0; a < (CF::SPLIT ? 0 : TC_KC / 64); a++) {
                        tma2d(s_addr(sbh + a * CF::ATOM), &bhmap, kc * TC_KC + a * 64, q0 + tb, full);
                        if (lo_any) tma2d(s_addr(sbh + a * CF::ATOM + CF::NP * 128), &blmap, kc * TC_KC + a * 64, q0 + tb, full);
                    }
                }
            });
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (CF::SPLIT && warp == TC_MMA_WARP0 + CF::NMMA) {
        // split rings: the activation producer, one K half (4 atoms) per slot
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&bhmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&blmap) : "memory");
            TC_FOR_UNITS({
                for (int kc = 0; kc < NK && !failed; kc++, item++) {
                    for (int h = 0; h < 2 && !failed; h++) {
                        const int fill = 2 * item + h;
                        const int slot = fill % (CF::SPLIT ? CF::NBH : 1);
                        const uint32_t par = (uint32_t)((fill / (CF::SPLIT ? CF::NBH : 1)) & 1);
                        if (!bar_wait(s_addr(&b_bempty[slot]), par ^ 1u)) { failed = true; break; }
                        unsigned char *sb = bslot(slot);
                        const uint32_t full = s_addr(&b_bfull[2 * slot + h]);
                        bar_expect(full, (uint32_t)(4 * CF::NP * 128 * (lo_any ? 2 : 1)));
                        for (int a = 0; a < 4; a++) {
                            const int x = kc * TC_KC + h * 256 + a * 64;
                            tma2d(s_addr(sb + a * CF::ATOM), &bhmap, x, q0 + tb, full);
                            if (lo_any) tma2d(s_addr(sb + a * CF::ATOM + CF::NP * 128), &blmap, x, q0 + tb, full);
                        }
                    }
                }
            });
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (warp >= TC_MMA_WARP0 && warp < TC_MMA_WARP0 + CF::NMMA) {
        // One thread issues an MMA about every 55 clocks however small N is, while the
        // tensor pipe finishes an M128 x N16 x K16 step in about 9: four issuer warps, each
        // with its own accumulator, keep the pipe fed. Issuer i takes K steps 8j..8j+7 of
        // stage half h (i = 2h + j); every stage starts fresh partials (double-buffered)
        // that the epilogue warps sum in fp32.
        if (lane == 0) {
            constexpr int PER_HALF = CF::NMMA / 2;
            const int mi = warp - TC_MMA_WARP0, h = mi / PER_HALF, j = mi % PER_HALF;
            const uint32_t idesc = f16_idesc(CF::N);
            using TM = CF;
            // the B offsets of the half's 16 K16 steps, in 16-byte descriptor units: the
            // descriptor of a stage's tile is built once and advanced by these (the 14-bit
            // start field does not carry: shared addresses stay below 256 KB)
            uint32_t boffh[16];
_Pragma("unroll")
            for (int sx = 0; sx < 16; sx++) {
                const int kk = (CF::SPLIT ? 0 : h * 256) + sx * 16;   // split: K inside the half
                boffh[sx] = (uint32_t)(((kk >> 6) * CF::ATOM + (kk & 63) * 2) >> 4);
            }
            TC_FOR_UNITS({
                for (int kc = 0; kc < NK && !failed; kc++, item++) {
                    const int st = item % CF::NS;
                    const uint32_t par = (uint32_t)((item / CF::NS) & 1);
                    const int pb = item & 1;
                    const int hfill = 2 * item + h;   // this half's place in the activation ring
                    // split: this half's activation slot
                    const int bslot_i = hfill % (CF::SPLIT ? CF::NBH : 1);
                    const uint32_t bpar = (uint32_t)((item / CF::B_PERIOD) & 1);   // this half's uses of the slot
                    if (!bar_wait(s_addr(&b_pfree[pb]), (uint32_t)(((item >> 1) & 1) ^ 1))) { failed = true; break; }
                    if (CF::SPLIT) {
                        if (!bar_wait(s_addr(&b_bfull[2 * bslot_i + h]), bpar)) { failed = true; break; }
                    } else {
                        if (!bar_wait(s_addr(&b_full[st]), par)) { failed = true; break; }
                    }
                    const uint32_t dtm = tmem + (uint32_t)(pb * TM::PCOLS + mi * TM::PW);
                    const uint32_t bh = CF::SPLIT ? s_addr(bslot(bslot_i))
                                                  : s_addr(wstage(st) + TC_W_BYTES + 1024 * ((TC_S_BYTES + 1023) / 1024));
                    const uint64_t dh = sw128_desc(bh);
                    // this issuer's K16 steps j*MPI .. (j+1)*MPI-1 of the half, sub-buffer by
                    // sub-buffer (dense: one issuer reads both of its half's sub-buffers;
                    // sparse: issuer j reads sub-buffer j)
                    constexpr int SS = CF::SUB_STEPS;
                    const int s_lo = j * CF::MPI, s_hi = s_lo + CF::MPI;
_Pragma("unroll")
                    for (int sb = 0; sb < CF::SUBS; sb++) {
                        if ((sb + 1) * SS <= s_lo || sb * SS >= s_hi) continue;   // not this issuer's
                        const int fill = hfill * CF::SUBS + sb;   // the A buffer the decode warps filled
                        const int ab = fill % TM::NA;
                        const uint32_t apar = (uint32_t)((item / TM::A_PERIOD) & 1);   // this half's uses of ab
                        if (!bar_wait(s_addr(&b_aready[2 * ab + h]), apar)) { failed = true; break; }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t atm = tmem + (uint32_t)(TM::ACOL0 + ab * TM::ACOLS);
                        // the atom's hi and lo rows as one N = 2 NP operand
_Pragma("unroll")
                        for (int st16 = 0; st16 < SS; st16++) {   // K16 steps of this sub-buffer
                            const int sx = sb * SS + st16;
                            if (sx < s_lo || sx >= s_hi) continue;
                            mma_ts(dtm, atm + (uint32_t)(st16 * 8), dh + boffh[sx], idesc, sx != s_lo ? 1u : 0u);
                        }
                        mma_commit(s_addr(&b_afree[ab]));
                    }
                    if (failed) break;
                    if (CF::SPLIT) {
                        mma_commit(s_addr(&b_bempty[bslot_i]));
                        mma_commit(s_addr(&b_pfull[pb]));   // the epilogue's signal
                    } else {
                        mma_commit(s_addr(&b_empty[st]));   // also tells the epilogue (no pfull commit)
                    }
                }
            });
            if (failed) flag(DEV_TIMEOUT);
        }
    } else if (warp < TC_DEQ_WARPS) {
        // ------------------------------------------------------------------ decode
        const int quarter = warp & 3, h = warp >> 2;     // TMEM lanes 32*quarter.., K half h
        const int r = quarter * 32 + lane;                // weight row of the unit = TMEM lane
        // shared-memory rows of this thread: box row and box base inside the stage
        int boxrow, boxbase;
        if (PHASE == 0) { boxrow = r & 63; boxbase = r < 64 ? 0 : 16384; }
        else { boxrow = r; boxbase = 0; }
        const int hbox = PHASE == 0 ? 8192 : 16384;       // the second (hi-K) box
        const int swz = boxrow & 7;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        TC_FOR_UNITS({
            for (int kc = 0; kc < NK && !failed; kc++, item++) {
                const int st = item % CF::NS;
                const uint32_t par = (uint32_t)((item / CF::NS) & 1);
                if (!bar_wait(s_addr(&b_full[st]), par)) { failed = true; break; }
                const unsigned char *sw = wstage(st);
                const unsigned char *row = sw + boxbase + h * hbox + boxrow * 128;
                const uint2 sc = *reinterpret_cast<const uint2 *>(sw + TC_W_BYTES + r * 16 + h * 8);
                constexpr int GS = 8 / CF::SUBS;                  // groups of 32 K per sub-buffer
_Pragma("unroll")
                for (int sb = 0; sb < CF::SUBS; sb++) {
                    // the A buffer this warp fills: sub-buffer sb of half h of this stage
                    const int fill = (2 * item + h) * CF::SUBS + sb;
                    const int ab = fill % CF::NA;
                    const uint32_t apar = (uint32_t)((fill / CF::NA) & 1);
                    if (!bar_wait(s_addr(&b_afree[ab]), apar ^ 1u)) { failed = true; break; }
                    const uint32_t atm = tmem + lane_addr + (uint32_t)(CF::ACOL0 + ab * CF::ACOLS);
                    // the groups of 32 in this sub-buffer, four at a time: the four loads go
                    // first (a load placed after a tcgen05.st would wait for it)
_Pragma("unroll")
                    for (int g4 = sb * GS; g4 < (sb + 1) * GS; g4 += 4) {
                        uint4 pks[4];
_Pragma("unroll")
                        for (int i = 0; i < 4; i++) pks[i] = *reinterpret_cast<const uint4 *>(row + (((g4 + i) ^ swz) << 4));
_Pragma("unroll")
                        for (int i = 0; i < 4; i++) {
                            const int g8 = g4 + i;
                            const uint4 pk = pks[i];
                            const uint32_t S = ((g8 < 4 ? sc.x : sc.y) >> (8 * (g8 & 3))) & 0xFFu;
                            const uint32_t s2 = stab[S];          // one shared load instead of ~8 ALU ops
                            uint32_t v[16];
                            uint32_t t4[4];
                            cvt4h(pk.x, t4);
                            v[0] = hmul2u(t4[0], s2); v[1] = hmul2u(t4[1], s2); v[2] = hmul2u(t4[2], s2); v[3] = hmul2u(t4[3], s2);
                            cvt4h(pk.y, t4);
                            v[4] = hmul2u(t4[0], s2); v[5] = hmul2u(t4[1], s2); v[6] = hmul2u(t4[2], s2); v[7] = hmul2u(t4[3], s2);
                            cvt4h(pk.z, t4);
                            v[8] = hmul2u(t4[0], s2); v[9] = hmul2u(t4[1], s2); v[10] = hmul2u(t4[2], s2); v[11] = hmul2u(t4[3], s2);
                            cvt4h(pk.w, t4);
                            v[12] = hmul2u(t4[0], s2); v[13] = hmul2u(t4[1], s2); v[14] = hmul2u(t4[2], s2); v[15] = hmul2u(t4[3], s2);
                            tmem_st16(atm + (uint32_t)((g8 - sb * GS) * 16), v);
                        }
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) bar_arrive(s_addr(&b_aready[2 * ab + h]));
                }
                if (failed) break;
                if (lane == 0) bar_arrive(s_addr(&b_empty[st]));
            }
        });
        if (failed && lane == 0) flag(DEV_TIMEOUT);
    } else if (warp >= TC_EPI_WARP0 && warp < TC_EPI_WARP0 + 4) {
        // ---------------------------------------------------------------- epilogue
        const int quarter = warp - TC_EPI_WARP0;
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        TC_FOR_UNITS({
            // the pass's per-token metadata, one token per lane, fetched before the stages
            const int nl = lane & (CF::NP - 1);
            const bool vl = nl < npt;
            const int ex_l = vl ? Xe[q0 + tb + nl] : 0;
            const int dst_l = (PHASE == 1 && vl) ? p.pair_dst[q0 + tb + nl] : 0;
            float acc[CF::NP];
_Pragma("unroll")
            for (int n = 0; n < CF::NP; n++) acc[n] = 0.0f;
            for (int kc = 0; kc < NK && !failed; kc++, item++) {
                const int pb = item & 1;
                // empty[st] completes once all four issuers' MMAs of the stage are done: the
                // partials are final. (The MMAs run at most two stages ahead of this wait --
                // they need pfree -- so the phase cannot be lapped.)
                if (CF::SPLIT) {   // both issuers' commits of this item
                    if (!bar_wait(s_addr(&b_pfull[pb]), (uint32_t)((item >> 1) & 1))) { failed = true; break; }
                } else {
                    if (!bar_wait(s_addr(&b_empty[item % CF::NS]), (uint32_t)((item / CF::NS) & 1))) { failed = true; break; }
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                using TM = CF;
                const uint32_t pt = tmem + lane_addr + (uint32_t)(pb * TM::PCOLS);
                if constexpr (CF::NMMA == 4) {
                    // four issuers x (hi products in columns 0..7, lo products in 8..15)
                    uint32_t d0[16], d1[16], d2[16], d3[16];
                    tmem_ld16(pt, d0);
                    tmem_ld16(pt + TM::PW, d1);
                    tmem_ld16(pt + 2 * TM::PW, d2);
                    tmem_ld16(pt + 3 * TM::PW, d3);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
_Pragma("unroll")
                    for (int n = 0; n < CF::NP; n++) {
                        float v = (__uint_as_float(d0[n]) + __uint_as_float(d1[n])) +
                                  (__uint_as_float(d2[n]) + __uint_as_float(d3[n]));
                        if (lo_any)
                            v += (__uint_as_float(d0[n + CF::NP]) + __uint_as_float(d1[n + CF::NP])) +
                                 (__uint_as_float(d2[n + CF::NP]) + __uint_as_float(d3[n + CF::NP]));
                        acc[n] += v;
                    }
                } else {
                    // two issuers (one per K half), 16 tokens at a time: hi products in
                    // columns c..c+15, their lo products NP columns further
_Pragma("unroll")
                    for (int c = 0; c < CF::NP; c += 16) {
                        uint32_t h0[16], h1[16], l0[16], l1[16];
                        tmem_ld16(pt + c, h0);
                        tmem_ld16(pt + TM::PW + c, h1);
                        if (lo_any) {
                            tmem_ld16(pt + CF::NP + c, l0);
                            tmem_ld16(pt + TM::PW + CF::NP + c, l1);
                        }
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
_Pragma("unroll")
                        for (int n = 0; n < 16; n++) {
                            float v = __uint_as_float(h0[n]) + __uint_as_float(h1[n]);
                            if (lo_any) v += __uint_as_float(l0[n]) + __uint_as_float(l1[n]);
                            acc[c + n] += v;
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(s_addr(&b_pfree[pb]));
            }
            if (failed) break;
            if (PHASE == 0) {
                // lanes 0..63 hold the gate rows, 64..127 the up rows of the same 64 rows:
                // each side hands the other half of its tokens over (gate values of odd
                // tokens, up values of even ones; [side][token / 2][row], conflict-free), so
                // all 128 threads apply the activation, to half the tokens each. The unit's
                // next MMAs wait on this tail, so it must be short.
                const int rr = r & 63, side = r >> 6;   // side is warp-uniform
_Pragma("unroll")
                for (int n = 0; n < CF::NP; n++)
                    if ((n & 1) != side) xch[(side * (CF::NP / 2) + n / 2) * 64 + rr] = acc[n];
                asm volatile("bar.sync 2, 128;" ::: "memory");
                // this side's tokens n = 2k + side: every activation first, unguarded (the
                // NP/2 chains are independent and interleave), the guarded stores after;
                // acc is indexed by compile-time k only, so it stays in registers
                float gv[CF::NP / 2], uv[CF::NP / 2], hv[CF::NP / 2];
_Pragma("unroll")
                for (int k = 0; k < CF::NP / 2; k++) {
                    const float mine = side ? acc[2 * k + 1] : acc[2 * k];
                    const float other = xch[((1 - side) * (CF::NP / 2) + k) * 64 + rr];
                    const float p2 = pow2f(__shfl_sync(0xffffffffu, ex_l, 2 * k + side));
                    gv[k] = __fmul_rn(side ? other : mine, p2);
                    uv[k] = __fmul_rn(side ? mine : other, p2);
                }
                if (act == K3GPU_ACT_SITU) {
_Pragma("unroll")
                    for (int k = 0; k < CF::NP / 2; k++) hv[k] = act_situ(gv[k], uv[k], b1, b2);
                } else {
_Pragma("unroll")
                    for (int k = 0; k < CF::NP / 2; k++) hv[k] = act_swiglu(gv[k], uv[k]);
                }
_Pragma("unroll")
                for (int k = 0; k < CF::NP / 2; k++)
                    if (2 * k + side < npt) p.H[(size_t)(q0 + tb + 2 * k + side) * bank.I + ub * 64 + rr] = hv[k];
                asm volatile("bar.sync 2, 128;" ::: "memory");
            } else {
_Pragma("unroll")
                for (int n = 0; n < CF::NP; n++) {
                    if (n < npt) {
                        const int ex = __shfl_sync(0xffffffffu, ex_l, n);
                        const int dst = __shfl_sync(0xffffffffu, dst_l, n);
                        p.contrib[(size_t)dst * bank.L + ub * 128 + r] = __fmul_rn(acc[n], pow2f(ex));
                    }
                }
            }
        });
        if (failed && lane == 0) flag(DEV_TIMEOUT);
    }
#undef TC_FOR_UNITS
    // every role reaches here (waits are bounded); free TMEM before leaving
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Gather the expert inputs into pair order as exact f16 hi/lo rows with the row's
// power-of-two exponent (the gate/up B operand): row q = z[pair_tok[q]].
__global__ void __launch_bounds__(256) tc_pack_pairs_kernel(__half *__restrict__ hi, __half *__restrict__ lo,
                                                            int *__restrict__ ex, int *__restrict__ lf,
                                                            const float *__restrict__ z,
                                                            const int *__restrict__ pair_tok,
                                                            const int *__restrict__ pair_exp,
                                                            int *__restrict__ elo,
                                                            const int *__restrict__ nrows, int K)
{
    __shared__ float redm[8];
    __shared__ int redf[8];
    const int q = blockIdx.x;
    if (q >= *nrows) return;
    const float *xr = z + (size_t)pair_tok[q] * K;
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
        hi[(size_t)q * K + i] = h;
        lo[(size_t)q * K + i] = l;
        any |= __half_as_ushort(l) != 0;
    }
    any = __any_sync(0xffffffffu, any);
    if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = any;
    __syncthreads();
    if (threadIdx.x == 0) {
        int f = 0;
        for (int w = 0; w < 8; w++) f |= redf[w];
        ex[q] = e;
        lf[q] = f;
        if (f) atomicOr(&elo[pair_exp[q]], 1);
    }
}

// One CTA per expert: 1 when every E8M0 byte of its three matrices lies in 104..140 or is
// 255, i.e. when scale * E2M1 is exact in f16 for every weight.
__global__ void __launch_bounds__(256) tc_bank_scan_kernel(uint8_t *__restrict__ safe, K3GpuExpertBank b)
{
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    const uint8_t *run = b.base + (size_t)blockIdx.x * b.stride;
    const long long n1 = (long long)b.I * (b.L / 32), n2 = (long long)b.L * (b.I / 32);
    int mybad = 0;
    for (long long i = threadIdx.x; i < n1; i += 256) {
        const unsigned s1 = run[b.s1 + i], s3 = run[b.s3 + i];
        mybad |= (s1 != 255u && (s1 < 104u || s1 > 140u)) | (s3 != 255u && (s3 < 104u || s3 > 140u));
    }
    for (long long i = threadIdx.x; i < n2; i += 256) {
        const unsigned s2 = run[b.s2 + i];
        mybad |= s2 != 255u && (s2 < 104u || s2 > 140u);
    }
    if (mybad) atomicOr(&bad, 1);
    __syncthreads();
    if (threadIdx.x == 0) safe[blockIdx.x] = bad ? 0 : 1;
}

// ---- host side ---------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn2)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 tc_encode()
{
    static EncodeTiledFn2 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn2>(q);
    });
    return fn;
}

static int tc_map(CUtensorMap *m, CUtensorMapDataType dt, int esize, const void *base, long long cols,
                  long long rows, int box_w, int box_rows, CUtensorMapSwizzle swz)
{
    EncodeTiledFn2 fn = tc_encode();
    if (!fn) return K3GPU_ECUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
    cuuint32_t box[2] = {(cuuint32_t)box_w, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        g_last_cuda_error = (int)r;
        return K3GPU_ECUDA;
    }
    return K3GPU_OK;
}

bool tc_bank_ok(const K3GpuExpertBank &b)
{
    return b.f16_safe != nullptr && mma_bank_ok(b);
}

static std::mutex g_tc_mu;
static bool g_tc_ready[64][2] = {};   // per device and shape: the shared-memory opt-in is done
int g_tc_shape = 0;                   // 0: by tokens per expert, 1: sparse always, 2: dense always

int tc_pack_pairs_launch(const MoePlan &p, const float *z, int L, int P, int E, cudaStream_t s)
{
    tc_pack_pairs_kernel<<<P, 256, 0, s>>>(p.zh, p.zl, p.ze, p.zf, z, p.pair_tok, p.pair_exp, p.elo,
                                           p.off + E, L);
    return launch_status();
}

template <class CF>
static int tc_shape_launch(int phase, const MoePlan &p, const K3GpuExpertBank &bank, int P, int act, float b1,
                           float b2, cudaStream_t s, int shape_id)
{
    const int L = bank.L, I = bank.I;
    const unsigned long long bytes = (unsigned long long)bank.n_experts * (unsigned long long)bank.stride;
    CUtensorMap wm, sm, bh, bl;
    int st;
    if (phase == 0) {
        st = tc_map(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, bank.base, L / 2, (long long)(bytes / (L / 2)), 128, 64,
                    CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st) st = tc_map(&sm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, bank.base, L / 32, (long long)(bytes / (L / 32)), 16, 64,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
        if (!st) st = tc_map(&bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.zh, L, P, 64, CF::NP, CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st) st = tc_map(&bl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.zl, L, P, 64, CF::NP, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        st = tc_map(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, bank.base, I / 2, (long long)(bytes / (I / 2)), 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st) st = tc_map(&sm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, bank.base, I / 32, (long long)(bytes / (I / 32)), 16, 128,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
        if (!st) st = tc_map(&bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.hh, I, P, 64, CF::NP, CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st) st = tc_map(&bl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.hl, I, P, 64, CF::NP, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (st) return st;
    // the shared-memory opt-in, once per device and shape (a function's attributes belong to
    // each device's context)
    int dev = 0;
    if ((st = cuda_status(cudaGetDevice(&dev)))) return st;
    if (dev < 0 || dev >= 64) return K3GPU_EINVAL;
    {
        std::lock_guard<std::mutex> lock(g_tc_mu);
        if (!g_tc_ready[dev][shape_id]) {
            st = cuda_status(cudaFuncSetAttribute(moe_tc_kernel<0, CF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  CF::SMEM));
            if (!st)
                st = cuda_status(cudaFuncSetAttribute(moe_tc_kernel<1, CF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      CF::SMEM));
            if (st) return st;
            g_tc_ready[dev][shape_id] = true;
        }
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long pl = L / 2, pi = I / 2, ql = L / 32, qi = I / 32;
    TcArgs a;
    a.safe = bank.f16_safe;
    if (phase == 0) {
        a.K = L; a.UE = I / 64;
        a.wys = bank.stride / pl; a.wy1 = bank.p1 / pl; a.wy3 = bank.p3 / pl;
        a.sys = bank.stride / ql; a.sy1 = bank.s1 / ql; a.sy3 = bank.s3 / ql;
        moe_tc_kernel<0, CF><<<sms, CF::THREADS, CF::SMEM, s>>>(wm, sm, bh, bl, p, bank, a, act, b1, b2);
    } else {
        a.K = I; a.UE = L / 128;
        a.wys = bank.stride / pi; a.wy1 = bank.p2 / pi; a.wy3 = 0;
        a.sys = bank.stride / qi; a.sy1 = bank.s2 / qi; a.sy3 = 0;
        moe_tc_kernel<1, CF><<<sms, CF::THREADS, CF::SMEM, s>>>(wm, sm, bh, bl, p, bank, a, act, b1, b2);
    }
    return launch_status();
}

// The pass shape by the call's tokens per routed expert: the sparse shape while most experts
// need one pass of 8, the dense one once they need several (TC_DENSE_MIN and up on average).
constexpr double TC_DENSE_MIN = 12.0;

bool tc_dense_for(double tokens_per_expert)
{
    return g_tc_shape == 2 || (g_tc_shape == 0 && tokens_per_expert >= TC_DENSE_MIN);
}

int tc_phase_launch(int phase, const MoePlan &p, const K3GpuExpertBank &bank, int P, int act, float b1,
                    float b2, cudaStream_t s, double tokens_per_expert)
{
    if (tc_dense_for(tokens_per_expert))
        return tc_shape_launch<TcDense>(phase, p, bank, P, act, b1, b2, s, 1);
    return tc_shape_launch<TcSparse>(phase, p, bank, P, act, b1, b2, s, 0);
}

int tc_bank_scan(const K3GpuExpertBank &b, uint8_t *safe, cudaStream_t s)
{
    tc_bank_scan_kernel<<<b.n_experts, 256, 0, s>>>(safe, b);
    return launch_status();
}

}  // namespace k3
