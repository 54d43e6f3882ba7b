/* LLaMA-2 block builders (reference: src/models/vkllm_llama2_layers.h:19-49, src/models/vkllm_llama2_layers.c).
 *
 * They append the reference's node sequence to a graph (so node names, ops, shapes and fp16 rounding
 * points are those of the reference) and, like the reference, return no tensor: the block's output
 * is the last node appended. */
#ifndef VKLLM_LLAMA2_LAYERS_H
#define VKLLM_LLAMA2_LAYERS_H

#include "vkllm_errors.h"
#include "vkllm_op_rope.h"
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct vkllm_context;
struct vkllm_graph;
struct vkllm_tensor;
struct vkllm_kvcache;

struct vkllm_llama2_self_attn_layer_params
{
    struct vkllm_tensor *WK, *WQ, *WV, *WO;
    struct vkllm_tensor *norm_weight;
    float norm_power;
    float norm_eps;
    float freq_base;
    uint32_t offsets;
    uint32_t num_head;
};

struct vkllm_llama2_ffn_layer_params
{
    struct vkllm_tensor *WU, *WG, *WD;
    struct vkllm_tensor *norm_weight;
    float norm_power;
    float norm_eps;
};

struct vkllm_llama2_transformer_block_params
{
    struct vkllm_llama2_ffn_layer_params ffn;
    struct vkllm_llama2_self_attn_layer_params attn;
};

extern vkllm_err_t vkllm_llama2_build_self_attn_layer(struct vkllm_context *context, struct vkllm_graph *graph,
                                                      struct vkllm_kvcache *kvcache, struct vkllm_tensor *input,
                                                      struct vkllm_llama2_self_attn_layer_params params,
                                                      uint32_t block_idx);
extern vkllm_err_t vkllm_llama2_build_ffn_layer(struct vkllm_context *context, struct vkllm_graph *graph,
                                                struct vkllm_tensor *input, struct vkllm_llama2_ffn_layer_params params,
                                                uint32_t block_idx);
extern vkllm_err_t vkllm_llama2_build_transformer_block(struct vkllm_context *context, struct vkllm_graph *graph,
                                                        struct vkllm_kvcache *kvcache, struct vkllm_tensor *input,
                                                        struct vkllm_llama2_transformer_block_params params,
                                                        uint32_t block_idx);

#ifdef __cplusplus
}
#endif
#endif
