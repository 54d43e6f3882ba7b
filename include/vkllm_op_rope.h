/* VKLLM_OP_ROPE (reference: src/core/vkllm_op_rope.h:12-31, src/core/vkllm_op_rope.c).
 *
 * Rotary embedding: theta = (offset + h) / base^(2i/W); input may be a strided view, output is
 * written with its own strides. f16 (fp32 math) or f32.
 */
#ifndef VKLLM_OP_ROPE_H
#define VKLLM_OP_ROPE_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

struct vkllm_op_rope_params
{
    uint32_t offset; /* position of row h = offset + h */
    float base;      /* frequency base, typically 10000 */
    bool neox_style; /* false: rotate (2i, 2i+1); true: rotate (i, i + W/2) */
};

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_rope_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_rope_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_rope_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
