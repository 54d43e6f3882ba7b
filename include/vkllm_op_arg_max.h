/* VKLLM_OP_ARG_MAX (reference: src/core/vkllm_op_arg_max.h, src/core/vkllm_op_arg_max.c).
 *
 * Per-row argmax to u32 [B,C,H,1]. Ties are broken by the reference rule: index i competes in
 * lane (i mod 32) keeping its first strict maximum, then a 16/8/4/2/1 tree keeps the left operand
 * unless the right one is strictly greater (src/shaders/vkllm_arg_max.comp:54-90).
 */
#ifndef VKLLM_OP_ARG_MAX_H
#define VKLLM_OP_ARG_MAX_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;


/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_arg_max_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_arg_max_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_arg_max_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
