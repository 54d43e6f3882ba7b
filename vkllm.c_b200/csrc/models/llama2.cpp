// LLaMA-2 model: GGUF load, free, graph build, tokenizer, and random initialisation on the device
// (reference: src/models/vkllm_models_llama2.c).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../engine/plan.h"
#include "../runtime/internal.h"
#include "gguf.h"
#include "vkllm_b200.h"
#include "vkllm_kvcache.h"
#include "vkllm_models_llama2.h"
#include "vkllm_op_matmul.h"
#include "vkllm_op_rmsnorm.h"

namespace vkb
{
void engine_destroy(vkllm_context *ctx, vkllm_models_llama2 *model);
void tp_comm_free(vkllm_models_llama2 *model);
vkllm_err_t fill_random_f16_shard(vkllm_context *ctx, void *dst, uint64_t rows, uint64_t cols, uint64_t full_cols,
                                  uint64_t row0, uint64_t col0, uint64_t seed, uint64_t tensor_id, float std_dev);
vkllm_err_t fill_random_f16(vkllm_context *ctx, void *dst, uint64_t n, uint64_t seed, uint64_t tensor_id,
                            float std_dev);
vkllm_err_t fill_const_f32(vkllm_context *ctx, void *dst, uint64_t n, float v);
void plan_free(vkllm_context *ctx, vkllm_graph *graph);
// Structural graph cache (graph_cache.cpp).
bool graph_cache_take(vkllm_context *ctx, vkllm_models_llama2 *model, vkllm_tensor *input_toks, vkllm_graph *graph,
                      uint32_t offsets, Plan *plan);
void graph_cache_register(vkllm_context *ctx, vkllm_models_llama2 *model, vkllm_graph *graph, Plan *plan);
void graph_cache_purge(vkllm_context *ctx, const vkllm_models_llama2 *model);
} // namespace vkb

namespace
{

// Defaults for metadata keys a file may omit (src/models/vkllm_models_llama2.c:224-241).
void set_defaults(vkllm_models_llama2 *m)
{
    m->meta.block_count = 32;
    m->meta.context_length = 2048;
    m->meta.embedding_length = 4096;
    m->meta.rope_freq_base = 10000.0f;
    m->meta.layer_norm_rms_epsilon = 1e-6f;
    m->meta.key_length = 128;
    m->meta.value_length = 128;
    m->meta.vocab_size = 32000;
    m->meta.head_count = 32;
    m->meta.head_count_kv = 32;
    m->meta.bos_token_id = 1;
    m->meta.eos_token_id = 2;
    m->meta.padding_token_id = 0;
    m->meta.add_bos_token = true;
    m->meta.add_eos_token = true;
}

// Metadata keys and their typed targets (src/models/vkllm_models_llama2.c:67-187). A key only
// takes effect with the expected GGUF type, as in the reference.
void apply_kv(vkllm_models_llama2 *m, const vkb::GgufKV &kv)
{
    struct U32Key
    {
        const char *name;
        uint32_t *dst;
    };
    const U32Key u32keys[] = {
        {"llama.block_count", &m->meta.block_count},
        {"llama.context_length", &m->meta.context_length},
        {"llama.embedding_length", &m->meta.embedding_length},
        {"llama.attention.key_length", &m->meta.key_length},
        {"llama.attention.value_length", &m->meta.value_length},
        {"llama.vocab_size", &m->meta.vocab_size},
        {"llama.attention.head_count", &m->meta.head_count},
        {"llama.attention.head_count_kv", &m->meta.head_count_kv},
        {"tokenizer.ggml.bos_token_id", &m->meta.bos_token_id},
        {"tokenizer.ggml.eos_token_id", &m->meta.eos_token_id},
        {"tokenizer.ggml.padding_token_id", &m->meta.padding_token_id},
    };
    for (const auto &k : u32keys)
        if (kv.key == k.name && kv.type == vkb::GGUF_U32)
            *k.dst = (uint32_t)kv.u;
    if (kv.key == "llama.rope.freq_base" && kv.type == vkb::GGUF_F32)
        m->meta.rope_freq_base = (float)kv.f;
    if (kv.key == "llama.attention.layer_norm_rms_epsilon" && kv.type == vkb::GGUF_F32)
        m->meta.layer_norm_rms_epsilon = (float)kv.f;
    if (kv.key == "tokenizer.ggml.add_bos_token" && kv.type == vkb::GGUF_BOOL)
        m->meta.add_bos_token = kv.u != 0;
    if (kv.key == "tokenizer.ggml.add_eos_token" && kv.type == vkb::GGUF_BOOL)
        m->meta.add_eos_token = kv.u != 0;
}

vkllm_tensor **block_slot(block_weights *bw, const std::string &leaf)
{
    if (leaf == "attn_norm.weight")
        return &bw->attn_norm_weight;
    if (leaf == "ffn_norm.weight")
        return &bw->ffn_norm_weight;
    if (leaf == "attn_q.weight")
        return &bw->WQ;
    if (leaf == "attn_k.weight")
        return &bw->WK;
    if (leaf == "attn_v.weight")
        return &bw->WV;
    if (leaf == "attn_output.weight")
        return &bw->WO;
    if (leaf == "ffn_gate.weight")
        return &bw->WG;
    if (leaf == "ffn_up.weight")
        return &bw->WU;
    if (leaf == "ffn_down.weight")
        return &bw->WD;
    return nullptr;
}

vkllm_err_t ensure_blocks(vkllm_models_llama2 *m, size_t n)
{
    while (m->weights.blocks->used_n < n)
    {
        block_weights *bw = (block_weights *)calloc(1, sizeof(block_weights));
        if (!bw)
            return VKLLM_ERR_ALLOC;
        _CHECK(vkllm_array_block_weights_append(m->weights.blocks, bw));
    }
    return VKLLM_ERR_OK;
}

// GGUF dims are innermost-first; the tensor shape is their reverse (src/models/vkllm_models_llama2.c:198-202).
vkllm_err_t tensor_from_gguf(vkllm_context *ctx, const vkb::GgufTensor &gt, vkllm_tensor **out)
{
    if (gt.type != vkb::GGML_F32 && gt.type != vkb::GGML_F16)
    {
        log_error("tensor %s has GGML type %u; only F32 and F16 are supported", gt.name.c_str(), gt.type);
        return VKLLM_ERR_ARGS;
    }
    vkllm_dtype_t dt = gt.type == vkb::GGML_F32 ? vkllm_dtype_float32 : vkllm_dtype_float16;
    uint32_t shapes[4] = {1, 1, 1, 1};
    for (uint32_t i = 0; i < gt.n_dims && i < 4; ++i)
        shapes[3 - i] = (uint32_t)gt.dims[i];
    _CHECK(vkllm_tensor_new(ctx, gt.name.c_str(), shapes, dt, VKLLM_OP_NONE, NULL, 0, NULL, 0, false, out));
    void *d = vkb::dev_ptr(ctx, *out);
    if (!d)
        return VKLLM_ERR_ALLOC;
    VKB_CUDA(cudaMemcpyAsync(d, gt.data, gt.bytes, cudaMemcpyHostToDevice, ctx->runtime->stream));
    return VKLLM_ERR_OK;
}

// Tensor-parallel split of a llama2 GGUF tensor, by name (the layout init_random_tp writes): 1 = rows
// (Wq, Wk, Wv, Wgate, Wup, output), 2 = columns (Wo, Wdown), 0 = whole (embedding, norm gains).
int tp_split_of(const std::string &name)
{
    if (name == "output.weight")
        return 1;
    const size_t dot = name.rfind(".weight");
    if (name.compare(0, 4, "blk.") != 0 || dot == std::string::npos)
        return 0;
    const size_t leaf = name.find('.', 4);
    if (leaf == std::string::npos)
        return 0;
    const std::string l = name.substr(leaf + 1, dot - leaf - 1);
    if (l == "attn_q" || l == "attn_k" || l == "attn_v" || l == "ffn_gate" || l == "ffn_up")
        return 1;
    if (l == "attn_output" || l == "ffn_down")
        return 2;
    return 0;
}

// The shard of GGUF tensor t held by rank r of n: sp = {row0, rows, col0, cols} (vkllm_b200_tp_shard)
// of its [rows = ne1][cols = ne0] matrix; 1-D and whole tensors are one row block of all elements.
// Returns VKLLM_ERR_ARGS for a non-F16/F32 tensor or dimensions the split does not divide.
vkllm_err_t tp_shard_of(const vkb::GgufTensor &t, uint32_t rank, uint32_t n, uint32_t sp[4], uint32_t *esz)
{
    if (t.type != vkb::GGML_F32 && t.type != vkb::GGML_F16)
        return VKLLM_ERR_ARGS;
    *esz = t.type == vkb::GGML_F32 ? 4 : 2;
    const int split = t.n_dims == 2 ? tp_split_of(t.name) : 0;
    const uint64_t cols = t.dims[0], rows = t.n_dims >= 2 ? t.bytes / (*esz * cols) : 1;
    if (cols == 0 || rows * cols * *esz != t.bytes || rows > 0xffffffffull || cols > 0xffffffffull)
        return VKLLM_ERR_ARGS;
    return vkllm_b200_tp_shard((uint32_t)rows, (uint32_t)cols, split, rank, n, sp);
}

// Copies shard sp of t (row-major) to dst as a dense [sp[1]][sp[3]] block.
void copy_tp_shard(const vkb::GgufTensor &t, const uint32_t sp[4], uint32_t esz, uint8_t *dst)
{
    const uint64_t cols = t.dims[0], row_b = (uint64_t)sp[3] * esz;
    if (sp[2] == 0 && sp[3] == cols)
    {
        memcpy(dst, t.data + (uint64_t)sp[0] * cols * esz, (uint64_t)sp[1] * row_b);
        return;
    }
    for (uint32_t i = 0; i < sp[1]; ++i)
        memcpy(dst + i * row_b, t.data + (((uint64_t)sp[0] + i) * cols + sp[2]) * esz, row_b);
}

// tensor_from_gguf for rank r of n: the tensor holds only its shard ([1, 1, rows, cols] for a 2-D
// matrix; whole tensors keep their shape), staged on the host and uploaded.
vkllm_err_t tensor_from_gguf_shard(vkllm_context *ctx, const vkb::GgufTensor &gt, uint32_t rank, uint32_t n,
                                   vkllm_tensor **out)
{
    uint32_t sp[4], esz = 0;
    if (tp_shard_of(gt, rank, n, sp, &esz) != VKLLM_ERR_OK)
    {
        log_error("tensor %s cannot be split %u ways (GGML type %u)", gt.name.c_str(), n, gt.type);
        return VKLLM_ERR_ARGS;
    }
    if (gt.n_dims != 2 || tp_split_of(gt.name) == 0)
        return tensor_from_gguf(ctx, gt, out);
    uint32_t shapes[4] = {1, 1, sp[1], sp[3]};
    _CHECK(vkllm_tensor_new(ctx, gt.name.c_str(), shapes, gt.type == vkb::GGML_F32 ? vkllm_dtype_float32
                                                                                   : vkllm_dtype_float16,
                            VKLLM_OP_NONE, NULL, 0, NULL, 0, false, out));
    void *d = vkb::dev_ptr(ctx, *out);
    if (!d)
        return VKLLM_ERR_ALLOC;
    std::vector<uint8_t> host((size_t)sp[1] * sp[3] * esz);
    copy_tp_shard(gt, sp, esz, host.data());
    VKB_CUDA(cudaMemcpyAsync(d, host.data(), host.size(), cudaMemcpyHostToDevice, ctx->runtime->stream));
    VKB_CUDA(cudaStreamSynchronize(ctx->runtime->stream)); // the staging buffer ends with this call
    return VKLLM_ERR_OK;
}

vkllm_err_t create_kvcache(vkllm_context *ctx, vkllm_models_llama2 *m)
{
    _CHECK_ARGS(m->weights.blocks->used_n > 0 && m->weights.blocks->data[0]->WK && m->weights.blocks->data[0]->WV);
    // a tensor-parallel shard holds head_count / tp_size heads (its rows of Wk / Wv)
    uint32_t H = m->meta.head_count / (m->b200.tp_size > 0 ? m->b200.tp_size : 1);
    // head size = rows of Wk / Wv (heads x head_dim of this shard)
    uint32_t kd = m->weights.blocks->data[0]->WK->shapes[2] / H;
    uint32_t vd = m->weights.blocks->data[0]->WV->shapes[2] / H;
    uint32_t kshape[4] = {1, H, m->meta.context_length, kd};
    uint32_t vshape[4] = {1, H, m->meta.context_length, vd};
    return vkllm_kvcache_new(ctx, kshape, vshape, m->meta.block_count, &m->weights.kvcache);
}

} // namespace

extern "C" vkllm_err_t vkllm_models_llama2_load(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                const char *file)
{
    _CHECK_ARGS(context && model && file);
    memset(model, 0, sizeof(*model));
    model->b200.tp_size = 1;
    vkb::GgufFile gguf;
    std::string err = gguf.open(file);
    if (!err.empty())
    {
        log_error("failed to open gguf file %s: %s", file, err.c_str());
        return VKLLM_ERR_ARGS;
    }
    set_defaults(model);
    const vkb::GgufKV *tokens = nullptr, *scores = nullptr, *types = nullptr;
    for (const auto &kv : gguf.kvs())
    {
        apply_kv(model, kv);
        if (kv.key == "tokenizer.ggml.tokens" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_STRING)
            tokens = &kv;
        if (kv.key == "tokenizer.ggml.scores" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_F32)
            scores = &kv;
        if (kv.key == "tokenizer.ggml.token_type" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_I32)
            types = &kv;
    }
    vkllm_err_t e = VKLLM_ERR_OK;
    if (tokens)
    {
        _CHECK(vkllm_array_token_new(&model->meta.tokens, tokens->arr_str.size()));
        for (size_t i = 0; i < tokens->arr_str.size(); ++i)
        {
            vkllm_token t;
            t.text = strdup(tokens->arr_str[i].c_str());
            t.score = scores && i < scores->arr_num.size() ? (float)scores->arr_num[i] : 0.0f;
            t.type = types && i < types->arr_num.size() ? (int32_t)types->arr_num[i] : 0;
            _CHECK(vkllm_array_token_append(model->meta.tokens, t));
        }
    }
    _CHECK(vkllm_array_block_weights_new(&model->weights.blocks, model->meta.block_count));
    for (const auto &t : gguf.tensors())
    {
        vkllm_tensor **slot = nullptr;
        if (t.name == "token_embd.weight")
            slot = &model->weights.tok_embed_weights;
        else if (t.name == "output_norm.weight")
            slot = &model->weights.output_norm_weight;
        else if (t.name == "output.weight")
            slot = &model->weights.output_weight;
        else if (t.name.compare(0, 4, "blk.") == 0)
        {
            int idx = -1;
            char leaf[96] = {0};
            if (sscanf(t.name.c_str(), "blk.%d.%95s", &idx, leaf) == 2 && idx >= 0 && idx < 4096)
            {
                e = ensure_blocks(model, (size_t)idx + 1);
                if (e != VKLLM_ERR_OK)
                    goto fail;
                slot = block_slot(model->weights.blocks->data[idx], leaf);
            }
        }
        if (!slot)
            continue;
        if (*slot)
            vkllm_tensor_free(context, *slot);
        e = tensor_from_gguf(context, t, slot);
        if (e != VKLLM_ERR_OK)
            goto fail;
    }
    if (cudaStreamSynchronize(context->runtime->stream) != cudaSuccess)
    {
        e = VKLLM_ERR_VULKAN;
        goto fail;
    }
    e = create_kvcache(context, model);
    if (e != VKLLM_ERR_OK)
        goto fail;
    return VKLLM_ERR_OK;
fail:
    vkllm_models_llama2_free(context, model);
    return e;
}

extern "C" vkllm_err_t vkllm_b200_models_llama2_load_tp(struct vkllm_context *context,
                                                        struct vkllm_models_llama2 *model, const char *file,
                                                        uint32_t tp_rank, uint32_t tp_size)
{
    _CHECK_ARGS(context && model && file && tp_size >= 1 && tp_size <= 8 && tp_rank < tp_size);
    if (tp_size == 1)
        return vkllm_models_llama2_load(context, model, file);
    memset(model, 0, sizeof(*model));
    vkb::GgufFile gguf;
    std::string err = gguf.open(file);
    if (!err.empty())
    {
        log_error("failed to open gguf file %s: %s", file, err.c_str());
        return VKLLM_ERR_ARGS;
    }
    set_defaults(model);
    model->b200.tp_size = tp_size;
    model->b200.tp_rank = tp_rank;
    const vkb::GgufKV *tokens = nullptr, *scores = nullptr, *types = nullptr;
    for (const auto &kv : gguf.kvs())
    {
        apply_kv(model, kv);
        if (kv.key == "tokenizer.ggml.tokens" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_STRING)
            tokens = &kv;
        if (kv.key == "tokenizer.ggml.scores" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_F32)
            scores = &kv;
        if (kv.key == "tokenizer.ggml.token_type" && kv.type == vkb::GGUF_ARRAY && kv.arr_type == vkb::GGUF_I32)
            types = &kv;
    }
    if (model->meta.head_count % tp_size != 0 || model->meta.vocab_size % tp_size != 0)
    {
        log_error("head_count %u and vocab_size %u must be multiples of tp_size %u", model->meta.head_count,
                  model->meta.vocab_size, tp_size);
        return VKLLM_ERR_ARGS;
    }
    vkllm_err_t e = VKLLM_ERR_OK;
    if (tokens)
    {
        _CHECK(vkllm_array_token_new(&model->meta.tokens, tokens->arr_str.size()));
        for (size_t i = 0; i < tokens->arr_str.size(); ++i)
        {
            vkllm_token t;
            t.text = strdup(tokens->arr_str[i].c_str());
            t.score = scores && i < scores->arr_num.size() ? (float)scores->arr_num[i] : 0.0f;
            t.type = types && i < types->arr_num.size() ? (int32_t)types->arr_num[i] : 0;
            _CHECK(vkllm_array_token_append(model->meta.tokens, t));
        }
    }
    _CHECK(vkllm_array_block_weights_new(&model->weights.blocks, model->meta.block_count));
    for (const auto &t : gguf.tensors())
    {
        vkllm_tensor **slot = nullptr;
        if (t.name == "token_embd.weight")
            slot = &model->weights.tok_embed_weights;
        else if (t.name == "output_norm.weight")
            slot = &model->weights.output_norm_weight;
        else if (t.name == "output.weight")
            slot = &model->weights.output_weight;
        else if (t.name.compare(0, 4, "blk.") == 0)
        {
            int idx = -1;
            char leaf[96] = {0};
            if (sscanf(t.name.c_str(), "blk.%d.%95s", &idx, leaf) == 2 && idx >= 0 && idx < 4096)
            {
                e = ensure_blocks(model, (size_t)idx + 1);
                if (e != VKLLM_ERR_OK)
                    goto fail;
                slot = block_slot(model->weights.blocks->data[idx], leaf);
            }
        }
        if (!slot)
            continue;
        if (*slot)
            vkllm_tensor_free(context, *slot);
        e = tensor_from_gguf_shard(context, t, tp_rank, tp_size, slot);
        if (e != VKLLM_ERR_OK)
            goto fail;
    }
    if (cudaStreamSynchronize(context->runtime->stream) != cudaSuccess)
    {
        e = VKLLM_ERR_VULKAN;
        goto fail;
    }
    e = create_kvcache(context, model);
    if (e != VKLLM_ERR_OK)
        goto fail;
    return VKLLM_ERR_OK;
fail:
    vkllm_models_llama2_free(context, model);
    return e;
}

extern "C" vkllm_err_t vkllm_b200_gguf_read_shard(const char *file, const char *tensor, uint32_t tp_rank,
                                                 uint32_t tp_size, void *dst, uint64_t dst_bytes, uint32_t *shape)
{
    _CHECK_ARGS(file && tensor && shape && tp_size >= 1 && tp_rank < tp_size);
    vkb::GgufFile gguf;
    std::string err = gguf.open(file);
    if (!err.empty())
    {
        log_error("failed to open gguf file %s: %s", file, err.c_str());
        return VKLLM_ERR_ARGS;
    }
    for (const auto &t : gguf.tensors())
    {
        if (t.name != tensor)
            continue;
        uint32_t sp[4], esz = 0;
        _CHECK(tp_shard_of(t, tp_rank, tp_size, sp, &esz));
        shape[0] = sp[1];
        shape[1] = sp[3];
        if (!dst)
            return VKLLM_ERR_OK; // shape query
        _CHECK_ARGS(dst_bytes >= (uint64_t)sp[1] * sp[3] * esz);
        copy_tp_shard(t, sp, esz, (uint8_t *)dst);
        return VKLLM_ERR_OK;
    }
    log_error("tensor %s not in %s", tensor, file);
    return VKLLM_ERR_ARGS;
}

extern "C" vkllm_err_t vkllm_models_llama2_free(struct vkllm_context *context, struct vkllm_models_llama2 *model)
{
    _CHECK_ARGS(context && model);
    vkb::graph_cache_purge(context, model);
    vkb::engine_destroy(context, model);
    vkb::tp_comm_free(model);
    if (model->meta.tokens)
    {
        for (size_t i = 0; i < model->meta.tokens->used_n; ++i)
            free(model->meta.tokens->data[i].text);
        vkllm_array_token_free(model->meta.tokens);
        model->meta.tokens = NULL;
    }
    vkllm_tensor_free(context, model->weights.tok_embed_weights);
    vkllm_tensor_free(context, model->weights.output_norm_weight);
    vkllm_tensor_free(context, model->weights.output_weight);
    model->weights.tok_embed_weights = model->weights.output_norm_weight = model->weights.output_weight = NULL;
    if (model->weights.blocks)
    {
        for (size_t i = 0; i < model->weights.blocks->used_n; ++i)
        {
            block_weights *bw = model->weights.blocks->data[i];
            if (!bw)
                continue;
            vkllm_tensor *ts[] = {bw->attn_norm_weight, bw->ffn_norm_weight, bw->WQ, bw->WK, bw->WV,
                                  bw->WO,               bw->WU,              bw->WG, bw->WD};
            for (vkllm_tensor *t : ts)
                vkllm_tensor_free(context, t);
            free(bw);
        }
        vkllm_array_block_weights_free(model->weights.blocks);
        model->weights.blocks = NULL;
    }
    if (model->weights.kvcache)
    {
        vkllm_kvcache_free(context, model->weights.kvcache);
        model->weights.kvcache = NULL;
    }
    return VKLLM_ERR_OK;
}

static vkllm_err_t build_graph_nodes(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                     struct vkllm_tensor *input_toks, struct vkllm_graph *graph, uint32_t offsets);

extern "C" vkllm_err_t vkllm_models_llama2_build_graph(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                       struct vkllm_tensor *input_toks, struct vkllm_graph *graph,
                                                       uint32_t offsets)
{
    _CHECK_ARGS(context && model && input_toks && graph);
    _CHECK_ARGS(model->weights.tok_embed_weights && model->weights.output_norm_weight && model->weights.output_weight);
    _CHECK_ARGS(model->weights.blocks && model->weights.blocks->used_n > 0 && model->weights.kvcache);
    _CHECK_ARGS(input_toks->dtype == vkllm_dtype_uint32);
    const uint32_t S = input_toks->shapes[3];
    _CHECK_ARGS((uint64_t)offsets + S <= model->meta.context_length);

    // A plan left by an earlier build into this graph goes (its nodes stay in the graph).
    vkb::plan_free(context, graph);
    vkb::Plan *plan = (vkb::Plan *)calloc(1, sizeof(vkb::Plan));
    if (!plan)
        return VKLLM_ERR_ALLOC;
    plan->model = model;
    plan->input_toks = input_toks;
    plan->offsets = offsets;
    plan->seq_len = S;
    if (graph->nodes->used_n == 0 && vkb::graph_cache_take(context, model, input_toks, graph, offsets, plan))
    {
        plan->output = graph->output_node;
        plan->n_nodes = graph->nodes->used_n;
        graph->b200_plan = plan;
        return VKLLM_ERR_OK;
    }
    vkllm_err_t pe = build_graph_nodes(context, model, input_toks, graph, offsets);
    if (pe != VKLLM_ERR_OK)
    {
        free(plan);
        return pe;
    }
    plan->output = graph->output_node;
    plan->n_nodes = graph->nodes->used_n;
    graph->b200_plan = plan;
    vkb::graph_cache_register(context, model, graph, plan);
    return VKLLM_ERR_OK;
}

// The reference builder's node sequence (src/models/vkllm_models_llama2.c:488-602): the input, the
// embedding, the transformer blocks, the output norm, the logits and the mapped ARG_MAX output.
static vkllm_err_t build_graph_nodes(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                     struct vkllm_tensor *input_toks, struct vkllm_graph *graph, uint32_t offsets)
{
    uint32_t B = input_toks->shapes[0], S = input_toks->shapes[3];
    uint32_t D = model->meta.embedding_length, V = model->meta.vocab_size;
    _CHECK(vkllm_graph_add_input(context, graph, input_toks));
    uint32_t eshape[4] = {B, 1, S, D};
    vkllm_tensor *esrcs[] = {input_toks, model->weights.tok_embed_weights};
    uint32_t unk = model->meta.padding_token_id;
    vkllm_tensor *embedded;
    _CHECK(vkllm_tensor_new(context, "embedded", eshape, vkllm_dtype_float16, VKLLM_OP_EMBEDDING, esrcs, 2, &unk,
                            sizeof(unk), false, &embedded));
    vkllm_err_t e = vkllm_graph_add_node(context, graph, embedded);
    if (e != VKLLM_ERR_OK)
    {
        vkllm_tensor_free(context, embedded);
        return e;
    }
    vkllm_tensor *hidden = embedded;
    for (uint32_t i = 0; i < model->meta.block_count && i < model->weights.blocks->used_n; ++i)
    {
        block_weights *bw = model->weights.blocks->data[i];
        _CHECK_ARGS(bw);
        vkllm_llama2_transformer_block_params bp;
        memset(&bp, 0, sizeof(bp));
        bp.attn.WK = bw->WK;
        bp.attn.WQ = bw->WQ;
        bp.attn.WV = bw->WV;
        bp.attn.WO = bw->WO;
        bp.attn.norm_weight = bw->attn_norm_weight;
        bp.attn.norm_power = 2.0f;
        bp.attn.norm_eps = model->meta.layer_norm_rms_epsilon;
        bp.attn.freq_base = model->meta.rope_freq_base;
        bp.attn.offsets = offsets;
        bp.attn.num_head = model->meta.head_count;
        bp.ffn.WU = bw->WU;
        bp.ffn.WG = bw->WG;
        bp.ffn.WD = bw->WD;
        bp.ffn.norm_weight = bw->ffn_norm_weight;
        bp.ffn.norm_power = 2.0f;
        bp.ffn.norm_eps = model->meta.layer_norm_rms_epsilon;
        _CHECK(vkllm_llama2_build_transformer_block(context, graph, model->weights.kvcache, hidden, bp, i));
        hidden = graph->nodes->data[graph->nodes->used_n - 1];
    }
    vkllm_tensor *norm, *logits, *output;
    vkllm_tensor *nsrcs[] = {hidden, model->weights.output_norm_weight};
    vkllm_op_rmsnorm_params np = {2.0f, model->meta.layer_norm_rms_epsilon};
    _CHECK(vkllm_tensor_new(context, "output_norm", hidden->shapes, hidden->dtype, VKLLM_OP_RMSNORM, nsrcs, 2, &np,
                            sizeof(np), false, &norm));
    _CHECK(vkllm_graph_add_node(context, graph, norm));
    uint32_t lshape[4] = {B, 1, S, V};
    vkllm_tensor *lsrcs[] = {norm, model->weights.output_weight};
    vkllm_op_matmul_params mp = {1.0f, 0};
    _CHECK(vkllm_tensor_new(context, "logits", lshape, norm->dtype, VKLLM_OP_MATMUL, lsrcs, 2, &mp, sizeof(mp), false,
                            &logits));
    _CHECK(vkllm_graph_add_node(context, graph, logits));
    uint32_t oshape[4] = {B, 1, S, 1};
    _CHECK(vkllm_tensor_new(context, "output", oshape, vkllm_dtype_uint32, VKLLM_OP_ARG_MAX, &logits, 1, NULL, 0, true,
                            &output));
    _CHECK(vkllm_graph_add_node(context, graph, output));
    _CHECK(vkllm_graph_set_output(context, graph, output));
    return VKLLM_ERR_OK;
}

// Tokenizer (src/models/vkllm_models_llama2.c:604-816): "▁" prefix and "▁" for every space, split
// into UTF-8 characters, then repeatedly merge the adjacent pair whose concatenation is a vocabulary
// entry with the highest score (first pair on ties), until no pair merges. Output: [bos] + ids of
// the pieces found in the vocabulary (first entry with that text) + [eos].
extern "C" vkllm_err_t vkllm_models_llama2_tokenize(struct vkllm_models_llama2 *model, const char *sentence,
                                                    struct vkllm_array_token_id **token_ids)
{
    _CHECK_ARGS(model && sentence && token_ids);
    _CHECK_ARGS(model->meta.tokens && model->meta.tokens->used_n > 0);
    std::unordered_map<std::string, uint32_t> vocab;
    vocab.reserve(model->meta.tokens->used_n * 2);
    for (size_t i = 0; i < model->meta.tokens->used_n; ++i)
        vocab.emplace(model->meta.tokens->data[i].text ? model->meta.tokens->data[i].text : "", (uint32_t)i);
    size_t len = strlen(sentence);
    if (len == 0)
        return vkllm_array_token_id_new(token_ids, 1);
    static const char kSpace[] = "\xE2\x96\x81";
    std::string text = kSpace;
    for (size_t i = 0; i < len; ++i)
    {
        if (sentence[i] == ' ')
            text += kSpace;
        else
            text += sentence[i];
    }
    std::vector<std::string> pieces;
    for (size_t i = 0; i < text.size();)
    {
        unsigned char c = (unsigned char)text[i];
        size_t n = 1;
        if (c >= 0x80)
        {
            if ((c & 0xE0) == 0xC0)
                n = 2;
            else if ((c & 0xF0) == 0xE0)
                n = 3;
            else if ((c & 0xF8) == 0xF0)
                n = 4;
        }
        if (i + n > text.size())
            n = text.size() - i;
        pieces.push_back(text.substr(i, n));
        i += n;
    }
    while (pieces.size() > 1)
    {
        float best = -INFINITY;
        long best_i = -1;
        for (size_t i = 0; i + 1 < pieces.size(); ++i)
        {
            auto it = vocab.find(pieces[i] + pieces[i + 1]);
            if (it == vocab.end())
                continue;
            float sc = model->meta.tokens->data[it->second].score;
            if (sc > best)
            {
                best = sc;
                best_i = (long)i;
            }
        }
        if (best_i < 0)
            break;
        pieces[best_i] += pieces[best_i + 1];
        pieces.erase(pieces.begin() + best_i + 1);
    }
    _CHECK(vkllm_array_token_id_new(token_ids, pieces.size() + 2));
    if (model->meta.add_bos_token)
        _CHECK(vkllm_array_token_id_append(*token_ids, model->meta.bos_token_id));
    for (const auto &p : pieces)
    {
        auto it = vocab.find(p);
        if (it != vocab.end())
            _CHECK(vkllm_array_token_id_append(*token_ids, it->second));
    }
    if (model->meta.add_eos_token)
        _CHECK(vkllm_array_token_id_append(*token_ids, model->meta.eos_token_id));
    return VKLLM_ERR_OK;
}

// ------------------------------------------------------------------------------------------------
// Random initialisation on the device (no GGUF): same tensors, names and shapes as the GGUF loader
// produces, fp16 weights ~ N(0, std) from a counter-based generator, f32 norm gains = 1.
// Tensor-parallel shard of one matrix (rows x cols of the unsharded model) for rank r of N:
// split 1 = rows, split 2 = columns, 0 = whole. out = {row0, rows, col0, cols}.
extern "C" vkllm_err_t vkllm_b200_tp_shard(uint32_t rows, uint32_t cols, int split, uint32_t tp_rank,
                                           uint32_t tp_size, uint32_t *out)
{
    _CHECK_ARGS(out && tp_size >= 1 && tp_rank < tp_size && split >= 0 && split <= 2);
    _CHECK_ARGS(split != 1 || rows % tp_size == 0);
    _CHECK_ARGS(split != 2 || cols % tp_size == 0);
    const uint32_t lr = split == 1 ? rows / tp_size : rows, lc = split == 2 ? cols / tp_size : cols;
    out[0] = split == 1 ? tp_rank * lr : 0;
    out[1] = lr;
    out[2] = split == 2 ? tp_rank * lc : 0;
    out[3] = lc;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_models_llama2_init_random(struct vkllm_context *context,
                                                            struct vkllm_models_llama2 *model,
                                                            const struct vkllm_b200_llama2_config *cfg,
                                                            uint64_t seed)
{
    return vkllm_b200_models_llama2_init_random_tp(context, model, cfg, seed, 0, 1);
}

extern "C" vkllm_err_t vkllm_b200_models_llama2_init_random_tp(struct vkllm_context *context,
                                                               struct vkllm_models_llama2 *model,
                                                               const struct vkllm_b200_llama2_config *cfg,
                                                               uint64_t seed, uint32_t tp_rank, uint32_t tp_size)
{
    _CHECK_ARGS(context && model && cfg);
    _CHECK_ARGS(cfg->block_count > 0 && cfg->embedding_length > 0 && cfg->head_count > 0 && cfg->ffn_length > 0 &&
                cfg->vocab_size > 0 && cfg->context_length > 0);
    _CHECK_ARGS(cfg->embedding_length % cfg->head_count == 0);
    _CHECK_ARGS(tp_size >= 1 && tp_size <= 8 && tp_rank < tp_size);
    _CHECK_ARGS(cfg->head_count % tp_size == 0 && cfg->ffn_length % tp_size == 0 && cfg->vocab_size % tp_size == 0);
    memset(model, 0, sizeof(*model));
    model->b200.tp_size = tp_size;
    model->b200.tp_rank = tp_rank;
    set_defaults(model);
    model->meta.block_count = cfg->block_count;
    model->meta.context_length = cfg->context_length;
    model->meta.embedding_length = cfg->embedding_length;
    model->meta.head_count = cfg->head_count;
    model->meta.head_count_kv = cfg->head_count;
    model->meta.key_length = model->meta.value_length = cfg->embedding_length / cfg->head_count;
    model->meta.vocab_size = cfg->vocab_size;
    model->meta.rope_freq_base = cfg->rope_freq_base > 0 ? cfg->rope_freq_base : 10000.0f;
    model->meta.layer_norm_rms_epsilon = cfg->rms_eps > 0 ? cfg->rms_eps : 1e-5f;
    uint32_t D = cfg->embedding_length, F = cfg->ffn_length, V = cfg->vocab_size;
    float sd = cfg->init_std > 0 ? cfg->init_std : 0.02f;
    uint64_t tid = 0;
    vkllm_err_t e;
    // The tensor-parallel shard of rank r of N: rows [r rows/N, (r+1) rows/N) (split = 1: Wq/Wk/Wv,
    // Wgate/Wup, output) or columns [r cols/N, ...) (split = 2: Wo, Wdown) of the full matrix, with the
    // full matrix's element bits; split = 0 keeps the whole tensor (embedding).
    auto make16s = [&](const char *name, uint32_t rows, uint32_t cols, int split, vkllm_tensor **out) -> vkllm_err_t {
        uint32_t sp[4];
        _CHECK(vkllm_b200_tp_shard(rows, cols, split, tp_rank, tp_size, sp));
        const uint32_t r0 = sp[0], lr = sp[1], c0 = sp[2], lc = sp[3];
        uint32_t sh[4] = {1, 1, lr, lc};
        _CHECK(vkllm_tensor_new(context, name, sh, vkllm_dtype_float16, VKLLM_OP_NONE, NULL, 0, NULL, 0, false, out));
        void *d = vkb::dev_ptr(context, *out);
        if (!d)
            return VKLLM_ERR_ALLOC;
        if (tp_size == 1)
            return vkb::fill_random_f16(context, d, (uint64_t)rows * cols, seed, tid++, sd);
        return vkb::fill_random_f16_shard(context, d, lr, lc, cols, r0, c0, seed, tid++, sd);
    };
    auto make16 = [&](const char *name, uint32_t rows, uint32_t cols, vkllm_tensor **out) -> vkllm_err_t {
        return make16s(name, rows, cols, 0, out);
    };
    auto make32 = [&](const char *name, uint32_t n, vkllm_tensor **out) -> vkllm_err_t {
        uint32_t sh[4] = {1, 1, 1, n};
        _CHECK(vkllm_tensor_new(context, name, sh, vkllm_dtype_float32, VKLLM_OP_NONE, NULL, 0, NULL, 0, false, out));
        void *d = vkb::dev_ptr(context, *out);
        if (!d)
            return VKLLM_ERR_ALLOC;
        tid++;
        return vkb::fill_const_f32(context, d, n, 1.0f);
    };
    char name[128];
    e = vkllm_array_block_weights_new(&model->weights.blocks, cfg->block_count);
    if (e != VKLLM_ERR_OK)
        return e;
    // Tensor ids follow GGUF order: token_embd, blocks (attn_norm, ffn_norm, q, k, v, o, gate, up,
    // down), output_norm, output.
    if ((e = make16("token_embd.weight", V, D, &model->weights.tok_embed_weights)) != VKLLM_ERR_OK)
        goto fail;
    if ((e = ensure_blocks(model, cfg->block_count)) != VKLLM_ERR_OK)
        goto fail;
    for (uint32_t i = 0; i < cfg->block_count; ++i)
    {
        block_weights *bw = model->weights.blocks->data[i];
        snprintf(name, sizeof(name), "blk.%u.attn_norm.weight", i);
        if ((e = make32(name, D, &bw->attn_norm_weight)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.ffn_norm.weight", i);
        if ((e = make32(name, D, &bw->ffn_norm_weight)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.attn_q.weight", i);
        if ((e = make16s(name, D, D, 1, &bw->WQ)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.attn_k.weight", i);
        if ((e = make16s(name, D, D, 1, &bw->WK)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.attn_v.weight", i);
        if ((e = make16s(name, D, D, 1, &bw->WV)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.attn_output.weight", i);
        if ((e = make16s(name, D, D, 2, &bw->WO)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.ffn_gate.weight", i);
        if ((e = make16s(name, F, D, 1, &bw->WG)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.ffn_up.weight", i);
        if ((e = make16s(name, F, D, 1, &bw->WU)) != VKLLM_ERR_OK)
            goto fail;
        snprintf(name, sizeof(name), "blk.%u.ffn_down.weight", i);
        if ((e = make16s(name, D, F, 2, &bw->WD)) != VKLLM_ERR_OK)
            goto fail;
    }
    if ((e = make32("output_norm.weight", D, &model->weights.output_norm_weight)) != VKLLM_ERR_OK)
        goto fail;
    if ((e = make16s("output.weight", V, D, 1, &model->weights.output_weight)) != VKLLM_ERR_OK)
        goto fail;
    if (cudaStreamSynchronize(context->runtime->stream) != cudaSuccess)
    {
        e = VKLLM_ERR_VULKAN;
        goto fail;
    }
    if ((e = create_kvcache(context, model)) != VKLLM_ERR_OK)
        goto fail;
    return VKLLM_ERR_OK;
fail:
    vkllm_models_llama2_free(context, model);
    return e;
}
