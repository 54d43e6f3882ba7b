/* Operator set of the tensor DAG (reference: src/core/vkllm_ops.h:8-23). Values are part of the ABI. */
#ifndef VKLLM_OPS_H
#define VKLLM_OPS_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum
{
    VKLLM_OP_NONE = 0,
    VKLLM_OP_COPY,
    VKLLM_OP_BIN,
    VKLLM_OP_EMBEDDING,
    VKLLM_OP_RMSNORM,
    VKLLM_OP_MATMUL,
    VKLLM_OP_ROPE,
    VKLLM_OP_SOFTMAX,
    VKLLM_OP_FFN_UP_AND_GATE,
    VKLLM_OP_UPDATE_ROWS,
    VKLLM_OP_ARG_MAX,
    VKLLM_OP_REF,
    VKLLM_OP_COUNTS,
} vkllm_op_t;

/* reference: src/core/vkllm_ops.c:3-13 */
extern const char *vkllm_op_s(const vkllm_op_t op);

#ifdef __cplusplus
}
#endif
#endif
