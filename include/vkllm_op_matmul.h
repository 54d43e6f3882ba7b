/* VKLLM_OP_MATMUL (reference: src/core/vkllm_op_matmul.h:12-23, src/core/vkllm_op_matmul.c).
 *
 * C[b,c] = act(scale * A[b,c] . B[b,c]) with broadcasting over B and C (a size-1 axis is reused).
 * B is taken as [N,K] ("transposed", the weight layout) exactly when the reference predicate holds:
 * A.H == M && B.H == N && A.W == K && B.W == K (src/core/vkllm_op_matmul.c:14-24); otherwise as [K,N].
 * Note this predicate is shape-only: a [K,N] operand with K == N is read as [N,K], as in the reference.
 * When additionally A.H == 1 the GEMV kernel runs (decode); otherwise the GEMM kernels (tcgen05
 * tensor cores for fp16 operands with 16-byte-aligned rows, a CUDA-core kernel otherwise).
 * dtypes: f16.f16 -> f16 or f32.f32 -> f32; accumulation is fp32.
 */
#ifndef VKLLM_OP_MATMUL_H
#define VKLLM_OP_MATMUL_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

struct vkllm_op_matmul_params
{
    float scale;   /* output = act(scale * A.B) */
    int32_t act;   /* 0: none, 1: SiLU */
};

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_matmul_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_matmul_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_matmul_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
