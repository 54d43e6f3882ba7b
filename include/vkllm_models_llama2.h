/* LLaMA-2 model: GGUF load, graph build, tokenizer (reference: src/models/vkllm_models_llama2.h:6-146).
 *
 * The struct keeps the reference's fields. `b200` is appended: it holds the fused decode engine
 * bound to this model (created on first use) and the tensor-parallel shard description.
 */
#ifndef VKLLM_MODELS_LLAMA2_H
#define VKLLM_MODELS_LLAMA2_H

#include "vkllm_array.h"
#include "vkllm_llama2_layers.h"

#ifdef __cplusplus
extern "C" {
#endif

struct block_weights
{
    struct vkllm_tensor *attn_norm_weight;
    struct vkllm_tensor *ffn_norm_weight;
    struct vkllm_tensor *WQ;
    struct vkllm_tensor *WK;
    struct vkllm_tensor *WV;
    struct vkllm_tensor *WO;
    struct vkllm_tensor *WU;
    struct vkllm_tensor *WG;
    struct vkllm_tensor *WD;
};

VKLLM_DEF_ARRAY(block_weights, struct block_weights *)

struct vkllm_graph;
struct vkllm_kvcache;

struct vkllm_token
{
    char *text;
    float score;
    int32_t type;
};

VKLLM_DEF_ARRAY(token, struct vkllm_token)
VKLLM_DEF_ARRAY(token_id, uint32_t)

struct vkllm_models_llama2
{
    struct
    {
        uint32_t block_count;
        uint32_t context_length;
        uint32_t embedding_length;
        float rope_freq_base;
        float layer_norm_rms_epsilon;
        uint32_t key_length;
        uint32_t value_length;
        uint32_t vocab_size;
        uint32_t head_count;
        uint32_t head_count_kv;
        uint32_t bos_token_id;
        uint32_t eos_token_id;
        uint32_t padding_token_id;
        bool add_bos_token;
        bool add_eos_token;
        struct vkllm_array_token *tokens;
    } meta;

    struct
    {
        struct vkllm_tensor *tok_embed_weights;
        struct vkllm_array_block_weights *blocks;
        struct vkllm_tensor *output_norm_weight;
        struct vkllm_tensor *output_weight;
        struct vkllm_kvcache *kvcache;
    } weights;

    struct
    {
        void *engine;      /* fused decode engine (opaque), created on first fused run */
        uint32_t tp_rank;  /* tensor-parallel shard of this replica (0 when not sharded) */
        uint32_t tp_size;  /* 1 when not sharded */
        void *tp_comm;     /* peer-memory exchange of the tensor-parallel ranks (opaque) when tp_size > 1 */
    } b200;
};

/* GGUF v2/v3 file -> weights on the context's device + KV cache sized by llama.context_length
 * (reference: src/models/vkllm_models_llama2.c:255-412). Only F32 and F16 tensors are meaningful;
 * any other type is loaded as F16 bytes, as in the reference. */
extern vkllm_err_t vkllm_models_llama2_load(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                            const char *file);
extern vkllm_err_t vkllm_models_llama2_free(struct vkllm_context *context, struct vkllm_models_llama2 *model);
/* Appends the reference LLaMA-2 DAG for one step of S = input_toks->shapes[3] tokens at position
 * `offsets`, ending in a mapped u32 ARG_MAX node [1,1,S,1] set as the graph output
 * (reference: src/models/vkllm_models_llama2.c:488-602). */
extern vkllm_err_t vkllm_models_llama2_build_graph(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                   struct vkllm_tensor *input_toks, struct vkllm_graph *graph,
                                                   uint32_t offsets);
/* Greedy longest-match SentencePiece-style tokenizer over the GGUF vocabulary
 * (reference: src/models/vkllm_models_llama2.c:604-816). */
extern vkllm_err_t vkllm_models_llama2_tokenize(struct vkllm_models_llama2 *model, const char *sentence,
                                                struct vkllm_array_token_id **token_ids);

#ifdef __cplusplus
}
#endif
#endif
