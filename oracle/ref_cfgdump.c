/* ref_cfgdump.c -- test infrastructure: runs the REFERENCE's own config loader
 * (k3_cfg_load_file, include/k3/k3_cfg.h:253 of the reference, header-only with its
 * third_party/json.h) on one config file and prints what it parsed as one line
 *   CFG {"hidden": ..., ..., "full_attn": [...], "stride": ...}
 * or the line REFUSED. The loader's own diagnostics go to stderr/stdout beside it.
 * Built into _ref/ by the Makefile when the reference tree is present; used only by
 * tests/golden/make_cfg_golden.py to record the reference's answers. */
#include <stdio.h>

#include "k3_cfg.h"

int main(int argc, char **argv)
{
    if (argc != 2) return 2;
    K3Cfg c;
    int fa[256];
    if (!k3_cfg_load_file(&c, fa, 256, argv[1])) {
        printf("\nREFUSED\n");
        return 0;
    }
    printf("\nCFG {\"hidden\": %d, \"n_layers\": %d, \"vocab\": %d, \"rms_eps\": %.9g, \"kda_heads\": %d, "
           "\"kda_head_dim\": %d, \"conv_k\": %d, \"gate_lb\": %.9g, \"n_heads\": %d, \"q_lora\": %d, "
           "\"kv_lora\": %d, \"qk_nope\": %d, \"qk_rope\": %d, \"v_head\": %d, \"mla_out_gate\": %d, "
           "\"n_experts\": %d, \"topk\": %d, \"n_shared\": %d, \"latent\": %d, \"moe_inter\": %d, "
           "\"routed_scale\": %.9g, \"moe_renorm\": %d, \"latent_norm\": %d, \"first_dense\": %d, "
           "\"dense_inter\": %d, \"attn_res_block\": %d, \"situ_b1\": %.9g, \"situ_b2\": %.9g, \"stride\": %d, "
           "\"full_attn\": [",
           c.hidden, c.n_layers, c.vocab, (double)c.rms_eps, c.kda_heads, c.kda_head_dim, c.conv_k,
           (double)c.gate_lb, c.n_heads, c.q_lora, c.kv_lora, c.qk_nope, c.qk_rope, c.v_head, c.mla_out_gate,
           c.n_experts, c.topk, c.n_shared, c.latent, c.moe_inter, (double)c.routed_scale, c.moe_renorm,
           c.latent_norm, c.first_dense, c.dense_inter, c.attn_res_block, (double)c.situ_b1, (double)c.situ_b2,
           k3_attn_res_stride(&c));
    for (int i = 0; i < c.n_full_attn; i++) printf("%s%d", i ? ", " : "", c.full_attn[i]);
    printf("]}\n");
    return 0;
}
