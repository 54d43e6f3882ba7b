/* VKLLM_OP_FFN_UP_AND_GATE (reference: src/core/vkllm_op_ffn_up_and_gate.h, src/core/vkllm_op_ffn_up_and_gate.c).
 *
 * y = (x . Wu^T) * silu(x . Wg^T) for x [B,C,M,K], Wu/Wg [1,1,N,K] (srcs = {x, Wu, Wg}).
 * This is the operator's intended math. The reference host code pushes its constants in a layout
 * the shader does not expect (src/core/vkllm_op_ffn_up_and_gate.c:131-138 vs
 * src/shaders/vkllm_ffn_up_and_gate.comp:24-30) and its test never checks the output, so there is
 * no meaningful reference output to match; the LLaMA-2 graph does not use this op.
 */
#ifndef VKLLM_OP_FFN_UP_AND_GATE_H
#define VKLLM_OP_FFN_UP_AND_GATE_H

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
extern vkllm_err_t vkllm_op_ffn_up_and_gate_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_ffn_up_and_gate_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_ffn_up_and_gate_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
