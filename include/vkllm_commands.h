/* Command recording and submission (reference: src/core/vkllm_commands.h:36-56, src/core/vkllm_commands.c).
 *
 * The reference records a Vulkan command buffer, submits it to a queue and waits on a fence with a
 * 60 s timeout. Here a commands object owns a CUDA stream: work is enqueued on the stream as it is
 * recorded, vkllm_commands_submit records a completion event and vkllm_commands_wait_exec waits for
 * it (polling, 60 s limit -> VKLLM_ERR_VULKAN) and then runs the deferred host tasks (staging
 * copies into caller buffers), exactly where the reference runs them.
 */
#ifndef VKLLM_COMMANDS_H
#define VKLLM_COMMANDS_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_array.h"

struct vkllm_gpu_device;
struct vkllm_tensor;
struct vkllm_context;

struct vkllm_commands_task
{
    vkllm_err_t (*func)(void *);
    struct vkllm_context *context;
    void *priv;
};

VKLLM_DEF_ARRAY(commands_task, struct vkllm_commands_task)

struct vkllm_commands
{
    struct vkllm_gpu_device *device;
    void *stream;    /* cudaStream_t */
    void *done;      /* cudaEvent_t recorded by submit */
    int recording;   /* between begin and end */
    int submitted;   /* submit called, wait_exec pending */
    struct vkllm_array_commands_task *defer_tasks;
};

extern vkllm_err_t vkllm_commands_new(struct vkllm_context *context, struct vkllm_commands **commands);
extern void vkllm_commands_free(struct vkllm_context *context, struct vkllm_commands *commands);
extern vkllm_err_t vkllm_commands_begin(struct vkllm_context *context, struct vkllm_commands *commands);
extern vkllm_err_t vkllm_commands_end(struct vkllm_context *context, struct vkllm_commands *commands);
/* Host -> tensor. Mapped tensors: memcpy into data.host. Others: async copy on the stream; the
 * caller's buffer may be reused as soon as this returns (reference: src/core/vkllm_commands.c:172-211). */
extern vkllm_err_t vkllm_commands_upload(struct vkllm_context *context, struct vkllm_commands *commands,
                                         struct vkllm_tensor *tensor, const uint8_t *data, size_t bytes);
/* Tensor -> host. `data` is filled once vkllm_commands_wait_exec returns (reference: src/core/vkllm_commands.c:236-269). */
extern vkllm_err_t vkllm_commands_download(struct vkllm_context *context, struct vkllm_commands *commands,
                                           struct vkllm_tensor *tensor, uint8_t *data, size_t bytes);
extern vkllm_err_t vkllm_commands_submit(struct vkllm_context *context, struct vkllm_commands *commands);
extern vkllm_err_t vkllm_commands_wait_exec(struct vkllm_context *context, struct vkllm_commands *commands);

#ifdef __cplusplus
}
#endif
#endif
