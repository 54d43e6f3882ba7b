/* VKLLM_OP_BIN (reference: src/core/vkllm_op_bin.h, src/core/vkllm_op_bin.c).
 *
 * Elementwise out = in0 (op) in1, all three addressed with the output strides, no broadcasting.
 * f16.f16 -> f16/f32 (fp32 math) or f32.f32 -> f32.
 */
#ifndef VKLLM_OP_BIN_H
#define VKLLM_OP_BIN_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

/* The params block of a VKLLM_OP_BIN node is one int32_t: 0 add, 1 sub, 2 mul, 3 div
 * (src/shaders/vkllm_bin_op.comp:24-25). */

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_bin_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_bin_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_bin_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
