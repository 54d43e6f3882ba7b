// Execution-mode control, stream/device queries and struct-layout queries of vkllm_b200.h.
#include <cstddef>
#include <cstring>

#include "internal.h"
#include "vkllm_b200.h"
#include "vkllm_kvcache.h"
#include "vkllm_models_llama2.h"

namespace vkb
{
void graph_cache_purge(vkllm_context *ctx, const vkllm_models_llama2 *model);
}

extern "C" const char *vkllm_b200_version(void)
{
    return "vkllm-b200 0.1 (sm_100a)";
}

extern "C" vkllm_err_t vkllm_b200_set_exec_mode(struct vkllm_context *context, int mode)
{
    _CHECK_ARGS(context && context->runtime);
    _CHECK_ARGS(mode == VKLLM_B200_EXEC_FUSED || mode == VKLLM_B200_EXEC_STRICT);
    if (context->runtime->exec_mode != mode) // cached nodes of one mode carry that mode's buffers
        vkb::graph_cache_purge(context, nullptr);
    context->runtime->exec_mode = mode;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_set_graph_cache(struct vkllm_context *context, int on)
{
    _CHECK_ARGS(context && context->runtime);
    if (!on)
        vkb::graph_cache_purge(context, nullptr);
    context->runtime->graph_cache_on = on != 0;
    return VKLLM_ERR_OK;
}

extern "C" int vkllm_b200_get_exec_mode(struct vkllm_context *context)
{
    return context && context->runtime ? context->runtime->exec_mode : -1;
}

extern "C" void *vkllm_b200_context_stream(struct vkllm_context *context)
{
    return context && context->runtime ? (void *)context->runtime->stream : nullptr;
}

extern "C" int vkllm_b200_context_device(struct vkllm_context *context)
{
    return context && context->device ? context->device->ordinal : -1;
}

extern "C" vkllm_err_t vkllm_b200_allocator_stats(struct vkllm_context *context, uint64_t *dev_in_use,
                                                  uint64_t *dev_cached, uint64_t *host_in_use)
{
    _CHECK_ARGS(context && context->runtime);
    if (dev_in_use)
        *dev_in_use = context->runtime->dev_alloc->bytes_in_use();
    if (dev_cached)
        *dev_cached = context->runtime->dev_alloc->bytes_cached();
    if (host_in_use)
        *host_in_use = context->runtime->host_alloc->bytes_in_use();
    return VKLLM_ERR_OK;
}

#define VKB_FIELD(S, F)                                                                                                \
    if (strcmp(field, #F) == 0)                                                                                        \
        return offsetof(S, F);

extern "C" size_t vkllm_b200_sizeof(const char *name)
{
    if (!name)
        return 0;
    if (!strcmp(name, "vkllm_tensor"))
        return sizeof(vkllm_tensor);
    if (!strcmp(name, "vkllm_graph"))
        return sizeof(vkllm_graph);
    if (!strcmp(name, "vkllm_context"))
        return sizeof(vkllm_context);
    if (!strcmp(name, "vkllm_commands"))
        return sizeof(vkllm_commands);
    if (!strcmp(name, "vkllm_models_llama2"))
        return sizeof(vkllm_models_llama2);
    if (!strcmp(name, "vkllm_kvcache"))
        return sizeof(vkllm_kvcache);
    if (!strcmp(name, "block_weights"))
        return sizeof(block_weights);
    return 0;
}

extern "C" size_t vkllm_b200_offsetof(const char *name, const char *field)
{
    if (!name || !field)
        return (size_t)-1;
    if (!strcmp(name, "vkllm_tensor"))
    {
        VKB_FIELD(vkllm_tensor, name)
        VKB_FIELD(vkllm_tensor, dtype)
        VKB_FIELD(vkllm_tensor, shapes)
        VKB_FIELD(vkllm_tensor, strides)
        VKB_FIELD(vkllm_tensor, bytes)
        VKB_FIELD(vkllm_tensor, data)
        VKB_FIELD(vkllm_tensor, op)
        VKB_FIELD(vkllm_tensor, pipeline)
        VKB_FIELD(vkllm_tensor, srcs)
        VKB_FIELD(vkllm_tensor, params)
    }
    if (!strcmp(name, "vkllm_models_llama2"))
    {
        VKB_FIELD(vkllm_models_llama2, meta)
        VKB_FIELD(vkllm_models_llama2, weights)
        VKB_FIELD(vkllm_models_llama2, b200)
    }
    if (!strcmp(name, "vkllm_graph"))
    {
        VKB_FIELD(vkllm_graph, nodes)
        VKB_FIELD(vkllm_graph, input_nodes)
        VKB_FIELD(vkllm_graph, output_node)
        VKB_FIELD(vkllm_graph, commands)
        VKB_FIELD(vkllm_graph, b200_plan)
    }
    return (size_t)-1;
}
