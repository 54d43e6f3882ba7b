// vkllm_commands over one CUDA stream (reference: src/core/vkllm_commands.c).
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "internal.h"

namespace
{

struct DownloadTask
{
    vkllm_tensor *staging;
    uint8_t *dst;
    size_t bytes;
};

vkllm_err_t run_download_task(void *arg)
{
    vkllm_commands_task *task = (vkllm_commands_task *)arg;
    DownloadTask *d = (DownloadTask *)task->priv;
    memcpy(d->dst, d->staging->data.host, d->bytes);
    vkllm_tensor_free(task->context, d->staging);
    delete d;
    return VKLLM_ERR_OK;
}

} // namespace

extern "C" vkllm_err_t vkllm_commands_new(struct vkllm_context *context, struct vkllm_commands **commands)
{
    _CHECK_ARGS(context && commands && context->runtime);
    vkllm_commands *p = (vkllm_commands *)calloc(1, sizeof(vkllm_commands));
    if (!p)
        return VKLLM_ERR_ALLOC;
    p->device = context->device;
    // All commands objects of a context share its in-order stream, as every reference commands
    // object shares device queue 0 (src/core/vkllm_commands.c:87-94).
    p->stream = (void *)context->runtime->stream;
    // The reference loop creates a commands object per token (with its graph); completion events
    // are recycled through the context.
    cudaEvent_t ev;
    auto &pool = context->runtime->event_pool;
    if (!pool.empty())
    {
        ev = (cudaEvent_t)pool.back();
        pool.pop_back();
    }
    else
    {
        cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess)
        {
            free(p);
            return vkb::cuda_check(e, "cudaEventCreateWithFlags", __FILE__, __LINE__);
        }
    }
    p->done = (void *)ev;
    vkllm_err_t err = vkllm_array_commands_task_new(&p->defer_tasks, 16);
    if (err != VKLLM_ERR_OK)
    {
        cudaEventDestroy(ev);
        free(p);
        return err;
    }
    *commands = p;
    return VKLLM_ERR_OK;
}

extern "C" void vkllm_commands_free(struct vkllm_context *context, struct vkllm_commands *commands)
{
    if (!commands)
        return;
    cudaStreamSynchronize((cudaStream_t)commands->stream);
    // Run pending deferred tasks so staging buffers go back to the allocator.
    for (size_t i = 0; i < commands->defer_tasks->used_n; ++i)
        commands->defer_tasks->data[i].func(&commands->defer_tasks->data[i]);
    vkllm_array_commands_task_free(commands->defer_tasks);
    if (context && context->runtime && context->runtime->event_pool.size() < 64)
        context->runtime->event_pool.push_back(commands->done);
    else
        cudaEventDestroy((cudaEvent_t)commands->done);
    free(commands);
}

extern "C" vkllm_err_t vkllm_commands_begin(struct vkllm_context *context, struct vkllm_commands *commands)
{
    _CHECK_ARGS(context && commands);
    commands->recording = 1;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_commands_end(struct vkllm_context *context, struct vkllm_commands *commands)
{
    _CHECK_ARGS(context && commands);
    commands->recording = 0;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_commands_upload(struct vkllm_context *context, struct vkllm_commands *commands,
                                             struct vkllm_tensor *tensor, const uint8_t *data, size_t bytes)
{
    _CHECK_ARGS(context && commands && tensor && data);
    _CHECK_ARGS(bytes <= tensor->bytes);
    vkllm_tensor *owner = vkb::storage_owner(tensor);
    if (owner->data.mapped)
    {
        memcpy(owner->data.host, data, bytes);
        return vkllm_tensor_flush_cache(context, owner);
    }
    void *dst = vkb::dev_ptr(context, tensor);
    if (!dst)
        return VKLLM_ERR_ALLOC;
    // The copy is staged before cudaMemcpyAsync returns, so `data` may be reused at once.
    VKB_CUDA(cudaMemcpyAsync(dst, data, bytes, cudaMemcpyHostToDevice, (cudaStream_t)commands->stream));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_commands_download(struct vkllm_context *context, struct vkllm_commands *commands,
                                               struct vkllm_tensor *tensor, uint8_t *data, size_t bytes)
{
    _CHECK_ARGS(context && commands && tensor && data);
    _CHECK_ARGS(bytes <= tensor->bytes);
    vkllm_tensor *owner = vkb::storage_owner(tensor);
    if (owner->data.mapped)
    {
        // As in the reference, a mapped tensor is read directly (its producer has completed once
        // the caller waited on the graph / commands that wrote it).
        memcpy(data, owner->data.host, bytes);
        return VKLLM_ERR_OK;
    }
    void *src = vkb::dev_ptr(context, tensor);
    if (!src)
        return VKLLM_ERR_ALLOC;
    vkllm_tensor *staging = nullptr;
    _CHECK(vkllm_tensor_new_staging(context, tensor, &staging));
    VKB_CUDA(cudaMemcpyAsync(staging->data.host, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)commands->stream));
    DownloadTask *d = new DownloadTask{staging, data, bytes};
    vkllm_commands_task task = {run_download_task, context, d};
    return vkllm_array_commands_task_append(commands->defer_tasks, task);
}

extern "C" vkllm_err_t vkllm_commands_submit(struct vkllm_context *context, struct vkllm_commands *commands)
{
    _CHECK_ARGS(context && commands);
    VKB_CUDA(cudaEventRecord((cudaEvent_t)commands->done, (cudaStream_t)commands->stream));
    commands->submitted = 1;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_commands_wait_exec(struct vkllm_context *context, struct vkllm_commands *commands)
{
    _CHECK_ARGS(context && commands);
    cudaEvent_t ev = (cudaEvent_t)commands->done;
    if (!commands->submitted)
        VKB_CUDA(cudaEventRecord(ev, (cudaStream_t)commands->stream));
    // Same 60 s bound as the reference's fence wait (src/core/vkllm_commands.c:344-359).
    auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    for (;;)
    {
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess)
            break;
        if (q != cudaErrorNotReady)
            return vkb::cuda_check(q, "cudaEventQuery", __FILE__, __LINE__);
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60))
        {
            log_error("device work did not complete within 60 s");
            return VKLLM_ERR_VULKAN;
        }
        // Yield for the first ~200 ms (decode steps finish in a few ms), then back off.
        if (++spins < 200000)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    commands->submitted = 0;
    vkllm_err_t err = VKLLM_ERR_OK;
    for (size_t i = 0; i < commands->defer_tasks->used_n; ++i)
    {
        vkllm_err_t e = commands->defer_tasks->data[i].func(&commands->defer_tasks->data[i]);
        if (e != VKLLM_ERR_OK)
            err = e;
    }
    commands->defer_tasks->used_n = 0;
    return err;
}
