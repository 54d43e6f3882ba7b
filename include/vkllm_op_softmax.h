/* VKLLM_OP_SOFTMAX (reference: src/core/vkllm_op_softmax.h:12-25, src/core/vkllm_op_softmax.c).
 *
 * Row softmax over W. As in the reference shader the row maximum is taken over ALL entries, masked
 * ones included; masked entries are excluded from the sum and written as 0. Input is read with the
 * output strides (the reference passes only the output layout).
 */
#ifndef VKLLM_OP_SOFTMAX_H
#define VKLLM_OP_SOFTMAX_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

struct vkllm_op_softmax_params
{
    int32_t seq_mask; /* > 0: causal mask, entry i of row h is zeroed when i > h + offsets */
    uint32_t offsets;
};

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_softmax_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_softmax_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_softmax_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
