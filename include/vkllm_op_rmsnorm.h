/* VKLLM_OP_RMSNORM (reference: src/core/vkllm_op_rmsnorm.h:14-24, src/core/vkllm_op_rmsnorm.c).
 *
 * y = fp16((x * g) * rsqrt(mean(x^2) + eps)) per row of W. x: f16 [B,C,H,W]; g: f32 [1,1,1,W]; y: f16.
 */
#ifndef VKLLM_OP_RMSNORM_H
#define VKLLM_OP_RMSNORM_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

struct vkllm_op_rmsnorm_params
{
    float power; /* carried for API compatibility; unused, as in the reference shader */
    float eps;
};

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_rmsnorm_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_rmsnorm_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_rmsnorm_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
