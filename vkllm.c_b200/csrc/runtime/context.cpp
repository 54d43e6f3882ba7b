// vkllm_context over the CUDA runtime (reference: src/core/vkllm_context.c:8-35).
#include <cstdlib>
#include <cstring>

#include "internal.h"
#include "vkllm_hashmap.h"

extern "C" vkllm_err_t vkllm_context_new(uint32_t dev, struct vkllm_context **context)
{
    _CHECK_ARGS(context);
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
    {
        (void)cudaGetLastError();
        log_error("no CUDA device visible (%s)", cudaGetErrorString(e));
        return VKLLM_ERR_DEV_NOT_FOUND;
    }
    if ((int)dev >= n)
    {
        log_error("device %u not found (%d devices)", dev, n);
        return VKLLM_ERR_DEV_NOT_FOUND;
    }
    VKB_CUDA(cudaSetDevice((int)dev));

    vkllm_context *p = (vkllm_context *)calloc(1, sizeof(vkllm_context));
    if (!p)
        return VKLLM_ERR_ALLOC;
    p->appname = "vkllm";
    p->device = (vkllm_gpu_device *)calloc(1, sizeof(vkllm_gpu_device));
    p->runtime = new vkllm_b200_runtime();
    if (!p->device || !p->runtime)
        return VKLLM_ERR_ALLOC;

    cudaDeviceProp prop;
    VKB_CUDA(cudaGetDeviceProperties(&prop, (int)dev));
    p->device->ordinal = (int)dev;
    p->device->sm_count = prop.multiProcessorCount;
    p->device->cc_major = prop.major;
    p->device->cc_minor = prop.minor;
    p->device->smem_optin = prop.sharedMemPerBlockOptin;
    strncpy(p->device->name, prop.name, sizeof(p->device->name) - 1);

    vkllm_b200_runtime *rt = p->runtime;
    VKB_CUDA(cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking));
    rt->dev_alloc = new vkb::CachingAllocator(false);
    rt->host_alloc = new vkb::CachingAllocator(true);
    VKB_CUDA(cudaMalloc(&rt->dev_error_word, sizeof(int)));
    VKB_CUDA(cudaMemset(rt->dev_error_word, 0, sizeof(int)));
    const char *strict = getenv("VKLLM_B200_STRICT");
    rt->exec_mode = (strict && atoi(strict) != 0) ? VKLLM_EXEC_STRICT : VKLLM_EXEC_FUSED;
    const char *timing = getenv("VKLLM_NODE_TIMING");
    rt->node_timing = timing && atoi(timing) != 0;
    const char *gc = getenv("VKLLM_B200_GRAPH_CACHE");
    rt->graph_cache_on = !(gc && atoi(gc) == 0);

    vkllm_err_t err = vkllm_hashmap_new(&p->stats.node_time_cost, 1024);
    if (err != VKLLM_ERR_OK)
        return err;
    *context = p;
    return VKLLM_ERR_OK;
}

struct vkllm_models_llama2;

namespace vkb
{
void engine_release_all(vkllm_context *ctx);
void graph_cache_purge(vkllm_context *ctx, const vkllm_models_llama2 *model);
}

extern "C" void vkllm_context_free(struct vkllm_context *p)
{
    if (!p)
        return;
    vkllm_b200_runtime *rt = p->runtime;
    if (rt)
    {
        if (rt->stream)
            cudaStreamSynchronize(rt->stream);
        vkb::graph_cache_purge(p, nullptr); // cached nodes hold buffers of both allocators
        for (auto &kv : rt->pipelines)
        {
            if (kv.second->ev_start)
                cudaEventDestroy((cudaEvent_t)kv.second->ev_start);
            if (kv.second->ev_end)
                cudaEventDestroy((cudaEvent_t)kv.second->ev_end);
            free(kv.second);
        }
        for (void *b : rt->tensor_pool)
            free(b);
        for (void *ev : rt->event_pool)
            cudaEventDestroy((cudaEvent_t)ev);
        delete rt->dev_alloc;
        delete rt->host_alloc;
        if (rt->dev_error_word)
            cudaFree(rt->dev_error_word);
        if (rt->stream)
            cudaStreamDestroy(rt->stream);
        delete rt;
    }
    vkllm_hashmap_free(p->stats.node_time_cost);
    free(p->device);
    free(p);
}

namespace vkb
{

uint32_t dtype_bytes(vkllm_dtype_t dt)
{
    vkllm_dtype_info info;
    if (vkllm_get_dtype_info(dt, &info) != VKLLM_ERR_OK)
        return 0;
    return info.bytes;
}

vkllm_pipeline *get_pipeline(vkllm_context *ctx, const char *name, vkllm_op_t op, int variant)
{
    auto &tab = ctx->runtime->pipelines;
    auto it = tab.find(name);
    if (it != tab.end())
        return it->second;
    vkllm_pipeline *p = (vkllm_pipeline *)calloc(1, sizeof(vkllm_pipeline));
    strncpy(p->name, name, sizeof(p->name) - 1);
    p->op = op;
    p->variant = variant;
    tab[name] = p;
    return p;
}

cudaStream_t stream_of(vkllm_context *ctx, vkllm_commands *cmd)
{
    if (cmd && cmd->stream)
        return (cudaStream_t)cmd->stream;
    return ctx->runtime->stream;
}

void timing_begin(vkllm_context *ctx, vkllm_pipeline *p, cudaStream_t s)
{
    if (!ctx->runtime->node_timing || !p)
        return;
    if (!p->ev_start)
    {
        cudaEventCreate((cudaEvent_t *)&p->ev_start);
        cudaEventCreate((cudaEvent_t *)&p->ev_end);
    }
    cudaEventRecord((cudaEvent_t)p->ev_start, s);
}

void timing_end(vkllm_context *ctx, vkllm_pipeline *p, cudaStream_t s)
{
    if (!ctx->runtime->node_timing || !p || !p->ev_end)
        return;
    cudaEventRecord((cudaEvent_t)p->ev_end, s);
    p->timed = 1;
}

} // namespace vkb

extern "C" vkllm_err_t vkllm_pipeline_query_exec_time(struct vkllm_context *context, struct vkllm_pipeline *pipeline,
                                                      uint64_t *time_ns)
{
    _CHECK_ARGS(context && pipeline && time_ns);
    *time_ns = 0;
    if (!pipeline->timed)
        return VKLLM_ERR_OK;
    float ms = 0.f;
    VKB_CUDA(cudaEventSynchronize((cudaEvent_t)pipeline->ev_end));
    VKB_CUDA(cudaEventElapsedTime(&ms, (cudaEvent_t)pipeline->ev_start, (cudaEvent_t)pipeline->ev_end));
    *time_ns = (uint64_t)(ms * 1.0e6);
    return VKLLM_ERR_OK;
}
