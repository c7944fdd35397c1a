// layer.cuh -- the decoder layers with an optional expert-parallel MoE step, for the model
// driver (model.cu). The extern "C" k3gpu_decoder_layer_* entry points are these with no
// exchange.
#pragma once

#include "k3gpu.h"

namespace k3 {

// The MoE step of a layer split over the ranks of g (k3gpu_moe_layer_ep): the layer's bank
// holds this rank's routed experts, `shared` the replicated shared experts; seq is this
// step's exchange number, the same on every rank.
struct LayerEp {
    const K3GpuEpGroup *g;
    const K3GpuExpertBank *shared;
    unsigned seq;
    int *ok;
    void *ws;
    size_t ws_bytes;
};

int decoder_layer_kda(float *h, float *block_residual, int *n_blocks, int *moe_idx, float *moe_wt,
                      const K3GpuKdaLayerW *w, const K3GpuLayerCfg *c, int layer_idx, const float *state,
                      const float *conv_hist, const K3GpuKdaLog *log, const int *parent, int B, int T,
                      void *workspace, size_t ws_bytes, void *stream, const LayerEp *ep);

int decoder_layer_mla(float *h, float *block_residual, int *n_blocks, int *moe_idx, float *moe_wt,
                      const K3GpuMlaLayerW *w, const K3GpuLayerCfg *c, int layer_idx, uint16_t *lat,
                      uint16_t *rope, int cap, const int *cached, const uint64_t *mask, int max_ctx, int B,
                      int T, void *workspace, size_t ws_bytes, void *stream, const LayerEp *ep);

}  // namespace k3
