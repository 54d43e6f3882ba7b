/* VKLLM_OP_UPDATE_ROWS (reference: src/core/vkllm_op_update_rows.h:12-24, src/core/vkllm_op_update_rows.c).
 *
 * out[b,c,offset_rows + h,w] = src[b,c,h,w] (the KV-cache write); bit-exact copy, f16 or f32.
 */
#ifndef VKLLM_OP_UPDATE_ROWS_H
#define VKLLM_OP_UPDATE_ROWS_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

struct vkllm_op_update_rows_params
{
    uint32_t offset_rows;
};

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_update_rows_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_update_rows_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_update_rows_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
