// Structural graph cache for the LLaMA-2 token loop.
//
// The reference loop builds, initialises, runs and frees the whole model graph for every token
// (tests/vkllm_test_infer_gguf.c:181-272; the builder is src/models/vkllm_models_llama2.c:488-602):
// for 7B that is ~640 tensor structs created and freed per token. Between two tokens with the same
// model, batch and token count the graph differs only in values that follow the position: the RoPE
// offsets, the softmax offsets, the row extent of the KV-cache slices, and the key extent of the
// scores / probabilities nodes. So vkllm_graph_free hands the nodes of a model-built graph to this
// cache (input tensor excepted, which the caller creates per token) and the next build with the same
// structure takes them back and rewrites only those fields. Node buffers stay attached across tokens
// (a per-structure tensor arena); a node whose byte size grows past its buffer gets a new one on its
// next use. The context's allocation counters advance as if the nodes had been created and freed.
//
// What the caller sees is unchanged: the same node pointers order, names, ops, shapes, strides,
// params and sources as a fresh build. A caller that edits a built graph's nodes in place (params,
// shapes, sources) and then frees it should set VKLLM_B200_GRAPH_CACHE=0; a caller that adds or
// replaces nodes is detected (the node list no longer matches) and that graph is freed normally.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../engine/plan.h"
#include "../runtime/internal.h"
#include "vkllm_kvcache.h"
#include "vkllm_models_llama2.h"
#include "vkllm_op_rope.h"
#include "vkllm_op_softmax.h"

namespace vkb
{

enum PatchKind : uint8_t
{
    P_ROPE,   // RoPE params offset = offsets
    P_SLICE,  // KV-cache slice: rows = offsets + S
    P_SCORES, // [B, H, S, Lk] scores: Lk = offsets + S (contiguous strides, byte size)
    P_PROBS,  // the same for the softmax output, and its params offsets
};

struct GraphCacheEntry
{
    const vkllm_models_llama2 *model = nullptr;
    uint32_t B = 0, S = 0;
    Plan *owner = nullptr;             // plan of the live graph holding the nodes; null when idle
    std::vector<vkllm_tensor *> nodes; // graph nodes after the input tensor, in graph order
    vkllm_tensor *embedded = nullptr;  // its srcs[0] is the per-token input tensor
    vkllm_tensor *output = nullptr;    // the mapped ARG_MAX node
    std::vector<std::pair<vkllm_tensor *, uint8_t>> patches;
    std::vector<vkllm_tensor *> kv_src; // per layer: sources of the K and V cache tensors
    uint64_t last_use = 0;
};

namespace
{

constexpr size_t kMaxEntriesPerModel = 4;
uint64_t g_use_clock = 0;

// Frees an idle entry's nodes; their frees were counted when the graph holding them was freed.
void free_entry_nodes(vkllm_context *ctx, GraphCacheEntry *e)
{
    for (vkllm_tensor *t : e->nodes)
        vkllm_tensor_free(ctx, t);
    ctx->stats.tensor_free_counts -= (int)e->nodes.size();
    e->nodes.clear();
}

void set_contiguous(vkllm_context *ctx, vkllm_tensor *t)
{
    const uint64_t el = t->dtype == vkllm_dtype_float32 || t->dtype == vkllm_dtype_uint32 ? 4
                        : t->dtype == vkllm_dtype_int8                                     ? 1
                                                                                           : 2;
    const uint64_t row = t->shapes[3] * el, s1 = t->shapes[2] * row, s0 = t->shapes[1] * s1;
    t->strides[3] = (uint32_t)el;
    t->strides[2] = (uint32_t)row;
    t->strides[1] = (uint32_t)s1;
    t->strides[0] = (uint32_t)s0;
    t->bytes = (uint32_t)((s0 * t->shapes[0] + 63) / 64 * 64);
    if (!t->data.is_ref && !t->data.mapped && t->data.dev && t->bytes > t->data.capacity)
    {
        ctx->runtime->dev_alloc->release(t->data.dev); // re-backed at its next use (dev_ptr)
        t->data.dev = nullptr;
        t->data.capacity = 0;
    }
}

void apply_patches(vkllm_context *ctx, GraphCacheEntry *e, uint32_t offsets)
{
    const uint32_t lk = offsets + e->S;
    for (auto &pk : e->patches)
    {
        vkllm_tensor *t = pk.first;
        switch (pk.second)
        {
        case P_ROPE:
            ((vkllm_op_rope_params *)t->params)->offset = offsets;
            break;
        case P_SLICE:
            t->shapes[2] = lk;
            break;
        case P_PROBS:
            ((vkllm_op_softmax_params *)t->params)->offsets = offsets;
            t->shapes[3] = lk;
            set_contiguous(ctx, t);
            break;
        case P_SCORES:
            t->shapes[3] = lk;
            set_contiguous(ctx, t);
            break;
        }
    }
}

size_t entries_of(vkllm_context *ctx, const vkllm_models_llama2 *model)
{
    size_t n = 0;
    for (GraphCacheEntry *e : ctx->runtime->graph_cache)
        n += e->model == model;
    return n;
}

void drop_entry(vkllm_context *ctx, GraphCacheEntry *e)
{
    auto &v = ctx->runtime->graph_cache;
    v.erase(std::remove(v.begin(), v.end(), e), v.end());
    if (e->owner) // the live graph keeps its nodes and frees them itself
        e->owner->cache_entry = nullptr;
    else
        free_entry_nodes(ctx, e);
    delete e;
}

} // namespace

// Builds `graph` from an idle cache entry for (model, B, S) when one exists. Returns true when the
// graph was built from the cache, with `plan` attached to it.
bool graph_cache_take(vkllm_context *ctx, vkllm_models_llama2 *model, vkllm_tensor *input_toks, vkllm_graph *graph,
                      uint32_t offsets, Plan *plan)
{
    vkllm_b200_runtime *rt = ctx->runtime;
    if (!rt->graph_cache_on)
        return false;
    const uint32_t B = input_toks->shapes[0], S = input_toks->shapes[3];
    GraphCacheEntry *e = nullptr;
    for (GraphCacheEntry *c : rt->graph_cache)
        if (c->model == model && c->B == B && c->S == S && !c->owner)
        {
            e = c;
            break;
        }
    if (!e)
        return false;
    vkllm_kvcache *kv = model->weights.kvcache;
    const size_t L = e->kv_src.size() / 2;
    if (!kv || kv->kcaches->used_n < L || kv->vcaches->used_n < L)
        return false;
    for (size_t i = 0; i < L; ++i)
        if ((uint64_t)offsets + S > kv->kcaches->data[i]->shapes[2] ||
            (uint64_t)offsets + S > kv->vcaches->data[i]->shapes[2])
            return false; // the fresh build reports the error
    // nodes: the input, then the cached list
    const size_t n = 1 + e->nodes.size();
    if (graph->nodes->alloc_n < n)
    {
        vkllm_tensor **d = (vkllm_tensor **)realloc(graph->nodes->data, n * sizeof(vkllm_tensor *));
        if (!d)
            return false;
        graph->nodes->data = d;
        graph->nodes->alloc_n = n;
    }
    if (vkllm_array_tensor_append(graph->input_nodes, input_toks) != VKLLM_ERR_OK)
        return false;
    graph->nodes->data[0] = input_toks;
    memcpy(graph->nodes->data + 1, e->nodes.data(), e->nodes.size() * sizeof(vkllm_tensor *));
    graph->nodes->used_n = n;
    e->embedded->srcs[0] = input_toks;
    apply_patches(ctx, e, offsets);
    for (size_t i = 0; i < L; ++i) // what vkllm_kvcache_update does to the cache tensors
    {
        vkllm_tensor *kc = kv->kcaches->data[i], *vc = kv->vcaches->data[i];
        kc->srcs[0] = e->kv_src[2 * i];
        vc->srcs[0] = e->kv_src[2 * i + 1];
        memcpy(kc->params, &offsets, sizeof(offsets));
        memcpy(vc->params, &offsets, sizeof(offsets));
        kc->pipeline = NULL;
        vc->pipeline = NULL;
    }
    if (e->output->data.mapped && e->output->data.host) // fresh mapped memory reads as zero
        memset(e->output->data.host, 0, e->output->bytes);
    graph->output_node = e->output;
    ctx->stats.tensor_alloc_counts += e->nodes.size();
    plan->cache_entry = e;
    e->owner = plan;
    e->last_use = ++g_use_clock;
    return true;
}

// After a fresh build of `graph` (input tensor first, then the builder's nodes): registers a cache
// entry for its structure, owned by the graph until vkllm_graph_free hands the nodes back.
void graph_cache_register(vkllm_context *ctx, vkllm_models_llama2 *model, vkllm_graph *graph, Plan *plan)
{
    vkllm_b200_runtime *rt = ctx->runtime;
    if (!rt->graph_cache_on || graph->nodes->used_n < 2 || graph->nodes->data[0] != plan->input_toks)
        return;
    const uint32_t B = plan->input_toks->shapes[0], S = plan->seq_len;
    for (GraphCacheEntry *c : rt->graph_cache)
        if (c->model == model && c->B == B && c->S == S)
            return; // one entry per structure; this graph is freed normally
    if (entries_of(ctx, model) >= kMaxEntriesPerModel)
    {
        GraphCacheEntry *lru = nullptr;
        for (GraphCacheEntry *c : rt->graph_cache)
            if (c->model == model && !c->owner && (!lru || c->last_use < lru->last_use))
                lru = c;
        if (!lru)
            return;
        drop_entry(ctx, lru);
    }
    vkllm_kvcache *kv = model->weights.kvcache;
    if (!kv)
        return;
    GraphCacheEntry *e = new GraphCacheEntry();
    e->model = model;
    e->B = B;
    e->S = S;
    e->nodes.assign(graph->nodes->data + 1, graph->nodes->data + graph->nodes->used_n);
    e->embedded = e->nodes[0];
    e->output = plan->output;
    const size_t L = std::min(kv->kcaches->used_n, kv->vcaches->used_n);
    // The cache tensors' sources were just set by this build (vkllm_kvcache_update).
    e->kv_src.resize(2 * L);
    for (size_t i = 0; i < L; ++i)
    {
        e->kv_src[2 * i] = kv->kcaches->data[i]->srcs[0];
        e->kv_src[2 * i + 1] = kv->vcaches->data[i]->srcs[0];
    }
    auto is_cache = [&](const vkllm_tensor *t, bool keys_only) {
        for (size_t i = 0; i < L; ++i)
            if (t == kv->kcaches->data[i] || (!keys_only && t == kv->vcaches->data[i]))
                return true;
        return false;
    };
    bool ok = e->embedded->op == VKLLM_OP_EMBEDDING && e->embedded->srcs[0] == plan->input_toks;
    for (vkllm_tensor *t : e->nodes)
    {
        if (t->op == VKLLM_OP_ROPE)
            e->patches.push_back({t, P_ROPE});
        else if (t->data.is_ref && t->srcs[0] && is_cache(t->srcs[0], false))
            e->patches.push_back({t, P_SLICE});
        else if (t->op == VKLLM_OP_SOFTMAX)
            e->patches.push_back({t, P_PROBS});
        else if (t->op == VKLLM_OP_MATMUL && t->srcs[1] && t->srcs[1]->data.is_ref && t->srcs[1]->srcs[0] &&
                 is_cache(t->srcs[1]->srcs[0], true))
            e->patches.push_back({t, P_SCORES});
        if (t->op == VKLLM_OP_UPDATE_ROWS) // the builder adds no cache tensor to the graph
            ok = false;
    }
    if (!ok)
    {
        delete e;
        return;
    }
    e->owner = plan;
    e->last_use = ++g_use_clock;
    plan->cache_entry = e;
    rt->graph_cache.push_back(e);
}

// Called by vkllm_graph_free before it frees the nodes. Returns true when the nodes after the input
// went back to the cache (the caller then frees only the input tensor).
bool graph_cache_give(vkllm_context *ctx, vkllm_graph *graph)
{
    Plan *plan = (Plan *)graph->b200_plan;
    if (!plan || !plan->cache_entry)
        return false;
    GraphCacheEntry *e = plan->cache_entry;
    const bool same = graph->nodes->used_n == 1 + e->nodes.size() && graph->nodes->data[0] == plan->input_toks &&
                      graph->output_node == e->output && graph->input_nodes->used_n == 1 &&
                      memcmp(graph->nodes->data + 1, e->nodes.data(), e->nodes.size() * sizeof(vkllm_tensor *)) == 0;
    e->owner = nullptr;
    plan->cache_entry = nullptr;
    if (!same)
    {
        // The caller changed the node list: the graph frees what it holds, the entry goes.
        e->nodes.clear();
        drop_entry(ctx, e);
        return false;
    }
    ctx->stats.tensor_free_counts += e->nodes.size();
    return true;
}

// A graph whose plan is replaced or freed without vkllm_graph_free (e.g. a second build into the same
// graph) keeps its nodes: its entry is dropped.
void graph_cache_detach(vkllm_context *ctx, Plan *plan)
{
    if (!plan || !plan->cache_entry)
        return;
    GraphCacheEntry *e = plan->cache_entry;
    e->nodes.clear();
    drop_entry(ctx, e);
}

// Frees the cached nodes of `model` (all models when null).
void graph_cache_purge(vkllm_context *ctx, const vkllm_models_llama2 *model)
{
    if (!ctx || !ctx->runtime)
        return;
    std::vector<GraphCacheEntry *> drop;
    for (GraphCacheEntry *e : ctx->runtime->graph_cache)
        if (!model || e->model == model)
            drop.push_back(e);
    for (GraphCacheEntry *e : drop)
    {
        if (e->owner)
            e->nodes.clear(); // owned by a live graph
        drop_entry(ctx, e);
    }
}

} // namespace vkb
