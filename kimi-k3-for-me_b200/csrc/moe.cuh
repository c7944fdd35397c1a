// moe.cuh -- the MoE plan shared by the expert kernels (moe.cu, moe_mma.cu).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace k3 {

// Workspace regions of one MoE call. P = T * (topk + n_shared) (token, slot) pairs; the
// pairs are grouped by expert (off/cnt) in the "sorted" order the expert kernels walk.
struct MoePlan {
    int *cnt;        // [E]
    int *fill;       // [E]
    int *off;        // [E+1]
    int *act;        // [E] active expert ids, ascending
    int *n_active;   // [1]
    int *pair_tok;   // [P] token of sorted pair p
    int *pair_dst;   // [P] contribution row (t*S + s) of sorted pair p
    float *H;        // [P][I] activations after act(), fp32
    float *contrib;  // [T*S][L]
    // exact f16 split of the expert inputs in pair order for the tensor-core paths:
    // row q = z[pair_tok[q]] = (hi + lo) * 2^e
    __half *zh, *zl; // [P][L]
    int *ze;         // [P] per-row power-of-two exponent
    int *zf;         // [P] 1 if the row's lo half is not all zero
    __half *hh, *hl; // [P][I]
    int *he, *hf;    // [P]
    int *pair_exp;   // [P] expert of sorted pair p
    int *elo;        // [2][E] per expert: some input row has a nonzero lo half (z, then H)
};

inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

inline size_t plan_bytes(int T, int S, int E, int L, int I, MoePlan *p, char *base)
{
    const size_t P = (size_t)T * S;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += align256(bytes);
        return r;
    };
    char *cnt = take(sizeof(int) * E), *fill = take(sizeof(int) * E);
    char *off = take(sizeof(int) * (E + 1)), *act = take(sizeof(int) * E);
    char *na = take(sizeof(int)), *pt = take(sizeof(int) * P), *pd = take(sizeof(int) * P);
    char *H = take(sizeof(float) * P * I), *C = take(sizeof(float) * P * L);
    char *zh = take(2 * P * L), *zl = take(2 * P * L);
    char *ze = take(sizeof(int) * P), *zf = take(sizeof(int) * P);
    char *hh = take(2 * P * I), *hl = take(2 * P * I);
    char *he = take(sizeof(int) * P), *hf = take(sizeof(int) * P);
    char *pe = take(sizeof(int) * P), *el = take(sizeof(int) * 2 * E);
    if (p) {
        p->cnt = (int *)cnt; p->fill = (int *)fill; p->off = (int *)off; p->act = (int *)act;
        p->n_active = (int *)na; p->pair_tok = (int *)pt; p->pair_dst = (int *)pd;
        p->H = (float *)H; p->contrib = (float *)C;
        p->zh = (__half *)zh; p->zl = (__half *)zl; p->ze = (int *)ze; p->zf = (int *)zf;
        p->hh = (__half *)hh; p->hl = (__half *)hl; p->he = (int *)he; p->hf = (int *)hf;
        p->pair_exp = (int *)pe; p->elo = (int *)el;
    }
    return o;
}

// 2^e exactly, for the row exponents of the expert paths (e in -127..127: the packers clamp
// e to -126..127 and scale by 2^-e). x * pow2f(e) rounds once, so it equals ldexpf(x, e)
// bit for bit, at a fraction of its cost (the epilogues scale every output this way).
__device__ __forceinline__ float pow2f(int e)
{
    return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(0x00400000);   // 2^-127
}

__device__ __forceinline__ float act_situ(float g, float u, float b1, float b2)
{
    const float a = b1 * tanhf(g / b1) * (1.0f / (1.0f + expf(-g)));
    return a * (b2 * tanhf(u / b2));
}

__device__ __forceinline__ float act_swiglu(float g, float u)
{
    return (g * (1.0f / (1.0f + expf(-g)))) * u;
}

// E8M0 byte -> its power of two; 255 (NaN by the OCP MX spec) -> 0, as the reference.
__device__ __forceinline__ float e8m0_scale(unsigned b)
{
    if (b == 255u) return 0.0f;
    if (b == 0u) return __int_as_float(0x00400000);   // 2^-127, subnormal
    return __int_as_float((int)(b << 23));
}

// Whether the tensor-core expert kernels take this bank: L and I multiples of 256, and
// every expert run and matrix starting on a whole row of its tensor map (the layout
// k3gpu_bank_layout produces); otherwise the CUDA-core kernels run.
bool mma_bank_ok(const K3GpuExpertBank &b);

// The two tensor-core expert paths share the pair-ordered activation rows: gate/up reads
// row q = z[pair_tok[q]] (tc_pack_pairs), down reads row q of H (act_pack_rows).
bool tc_bank_ok(const K3GpuExpertBank &b);
int tc_bank_scan(const K3GpuExpertBank &b, uint8_t *safe, cudaStream_t s);
int tc_pack_pairs_launch(const MoePlan &p, const float *z, int L, int P, int E, cudaStream_t s);
void act_pack_rows_launch(const MoePlan &p, int I, int P, int E, cudaStream_t s);
// tcgen05 kernels on the certified experts (phase 0 = gate/up, 1 = down), in the pass shape
// the call's routed tokens per expert select (tc_dense_for; k3gpu_moe_select_kernels 2 / 3
// force the dense / sparse shape)
extern int g_tc_shape;
bool tc_dense_for(double tokens_per_expert);
int tc_phase_launch(int phase, const MoePlan &p, const K3GpuExpertBank &bank, int P, int act,
                    float b1, float b2, cudaStream_t s, double tokens_per_expert);
// mma.sync kernels on the experts the tcgen05 kernels do not take
int mma_phase_launch(int phase, const MoePlan &p, const K3GpuExpertBank &bank, int act,
                     float b1, float b2, cudaStream_t s);

}  // namespace k3
