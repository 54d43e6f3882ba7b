/* Per-layer KV cache (reference: src/models/vkllm_kvcache.h:14-25, src/models/vkllm_kvcache.c).
 *
 * kcaches/vcaches hold one persistent fp16 tensor [1, H, context, head_dim] per layer. Each is a
 * VKLLM_OP_UPDATE_ROWS node whose srcs[0] and offset are re-pointed by vkllm_kvcache_update every
 * step, which then replaces *key / *value by a slice0 view of the cache covering rows [0, offset + S)
 * (reference: src/models/vkllm_kvcache.c:65-102). HBM layout: head-major, rows of head_dim halves,
 * so one decode step appends one 2*head_dim-byte row per head and attention streams contiguous rows.
 */
#ifndef VKLLM_KVCACHE_H
#define VKLLM_KVCACHE_H

#include "vkllm_errors.h"
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct vkllm_array_tensor;
struct vkllm_tensor;
struct vkllm_context;
struct vkllm_graph;

struct vkllm_kvcache
{
    struct vkllm_array_tensor *kcaches;
    struct vkllm_array_tensor *vcaches;
    uint32_t kcache_shape[4];
    uint32_t vcache_shape[4];
    uint32_t layer_counts;
};

vkllm_err_t vkllm_kvcache_new(struct vkllm_context *context, uint32_t kcache_shape[4], uint32_t vcache_shape[4],
                              uint32_t layer_counts, struct vkllm_kvcache **kvcache);
vkllm_err_t vkllm_kvcache_update(struct vkllm_context *context, struct vkllm_kvcache *kvcache,
                                 struct vkllm_tensor **key, struct vkllm_tensor **value, uint32_t layer,
                                 uint32_t offset);
void vkllm_kvcache_free(struct vkllm_context *context, struct vkllm_kvcache *kvcache);

#ifdef __cplusplus
}
#endif
#endif
