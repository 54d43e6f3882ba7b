/* VKLLM_OP_EMBEDDING (reference: src/core/vkllm_op_embedding.h, src/core/vkllm_op_embedding.c).
 *
 * Row gather out[s,:] = E[id_s,:] for u32 ids [1,1,1,S] and table [1,1,V,D]; bit-exact.
 */
#ifndef VKLLM_OP_EMBEDDING_H
#define VKLLM_OP_EMBEDDING_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdbool.h>
#include <stdint.h>

struct vkllm_context;
struct vkllm_commands;
struct vkllm_tensor;

/* The params block of a VKLLM_OP_EMBEDDING node is one uint32_t: the token substituted for
 * ids >= vocabulary size (src/core/vkllm_op_embedding.c:91, src/shaders/vkllm_embedding.comp:57-60). */

/* Validates shapes/dtypes and selects the kernel (sets tensor->pipeline). */
extern vkllm_err_t vkllm_op_embedding_init(struct vkllm_context *context, struct vkllm_commands *commands,
                                  struct vkllm_tensor *tensor);
/* Enqueues the kernel on commands' stream. */
extern vkllm_err_t vkllm_op_embedding_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                 struct vkllm_tensor *tensor);
/* No-op, kept for the lifecycle. */
extern vkllm_err_t vkllm_op_embedding_post_run(struct vkllm_context *context, struct vkllm_commands *commands,
                                      struct vkllm_tensor *tensor);

#ifdef __cplusplus
}
#endif
#endif
