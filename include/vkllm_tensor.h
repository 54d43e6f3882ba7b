/* 4-D tensors and DAG nodes (reference: src/core/vkllm_tensor.h:19-65, src/core/vkllm_tensor.c).
 *
 * Layout [B, C, H, W]; `strides` are in BYTES, W innermost. A tensor is also a node of the op DAG:
 * `op` is the operator producing it, `srcs` its inputs and the trailing `params` the operator's
 * parameter block (copied at creation).
 *
 * Storage. The reference gives every tensor its own Vulkan buffer at creation. Here:
 *   - `mapped` tensors get pinned, device-mapped host memory at creation (`data.host` is valid at
 *     once, as in the reference) and `data.dev` is the device alias of the same bytes;
 *   - other tensors get device memory from the context's caching allocator when first needed
 *     (upload, download, op init/run, graph init), so `data.dev` may be NULL right after
 *     vkllm_tensor_new. Nodes that the fused decode path never materialises cost no device memory.
 *   - views (copy_ref, slice0) own nothing (`data.is_ref`); their bytes are those of srcs[0].
 * Fields that held Vulkan handles (VmaAllocation, VkBuffer, access/stage flags, descriptor set)
 * are replaced, so the struct is source-compatible with the reference, not binary-compatible.
 */
#ifndef VKLLM_TENSOR_H
#define VKLLM_TENSOR_H

#ifdef __cplusplus
extern "C" {
#endif

#include <stdbool.h>
#include <stdint.h>

#include "vkllm_common.h"
#include "vkllm_dtypes.h"
#include "vkllm_ops.h"

struct vkllm_context;
struct vkllm_pipeline;
struct vkllm_gpu_device;

struct vkllm_tensor
{
    const char name[128];
    vkllm_dtype_t dtype;
    uint32_t shapes[4];
    uint32_t strides[4];
    uint32_t bytes;

    struct vkllm_gpu_device *device;
    struct
    {
        void *dev;         /* device address of element [0,0,0,0] (NULL until first use, see above) */
        void *host;        /* host address, mapped tensors only */
        bool mapped;       /* host-visible; coherent with the device after vkllm_graph_run returns */
        bool is_ref;       /* view: the bytes belong to srcs[0] */
        uint64_t capacity; /* bytes reserved behind `dev` (>= bytes) */
    } data;

    uint32_t state_flags; /* runtime bookkeeping (replaces the Vulkan access/stage flags) */

    vkllm_op_t op;
    struct vkllm_pipeline *pipeline; /* kernel chosen by the op's init; non-NULL after vkllm_graph_init */
    struct vkllm_tensor *srcs[VKLLM_MAX_SRCS];
    uint8_t params[];
};

/* reference: src/core/vkllm_tensor.c:66-145. Every shape entry must be >= 1 (VKLLM_ERR_ARGS). */
extern vkllm_err_t vkllm_tensor_new(struct vkllm_context *context, const char *name, const uint32_t *shapes,
                                    vkllm_dtype_t dtype, vkllm_op_t op, struct vkllm_tensor **srcs,
                                    const uint32_t n_srcs, const void *params, size_t params_bytes, bool mapped,
                                    struct vkllm_tensor **p);
/* reference: src/core/vkllm_tensor.c:147-160. Returns owned storage to the context's allocator. */
extern void vkllm_tensor_free(struct vkllm_context *context, struct vkllm_tensor *tensor);
/* Mapped tensors only (VKLLM_ERR_ARGS otherwise). Pinned mapped memory is coherent, so these only
 * order host accesses against the device (reference: src/core/vkllm_tensor.c:162-196). */
extern vkllm_err_t vkllm_tensor_invalid_cache(struct vkllm_context *context, struct vkllm_tensor *tensor);
extern vkllm_err_t vkllm_tensor_flush_cache(struct vkllm_context *context, struct vkllm_tensor *tensor);
/* A mapped tensor with the same shape and dtype (reference: src/core/vkllm_tensor.c:198-205). */
extern vkllm_err_t vkllm_tensor_new_staging(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                            struct vkllm_tensor **staging);
/* In-place reshape of a contiguous tensor; strides recomputed (reference: src/core/vkllm_tensor.c:221-238). */
extern vkllm_err_t vkllm_tensor_reshape(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                        const uint32_t *shapes);
/* In-place axis permutation of shapes and strides (reference: src/core/vkllm_tensor.c:240-259). */
extern vkllm_err_t vkllm_tensor_permute(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                        const uint32_t *axis);
/* Non-owning view, op VKLLM_OP_REF, srcs[0] = tensor, name "<name>_ref" (reference: src/core/vkllm_tensor.c:261-299). */
extern vkllm_err_t vkllm_tensor_copy_ref(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                         struct vkllm_tensor **p);
/* View of the leading `extents` of every axis, name "<name>_slice0" (reference: src/core/vkllm_tensor.c:301-320). */
extern vkllm_err_t vkllm_tensor_slice0(struct vkllm_context *context, struct vkllm_tensor *tensor, uint32_t extents[4],
                                       struct vkllm_tensor **slice);
/* "<name><dtype>[B, C, H, W]" (reference: src/core/vkllm_tensor.c:322-336). */
extern vkllm_err_t vkllm_tensor_s(struct vkllm_context *context, struct vkllm_tensor *tensor, char *buf, size_t len);

#ifdef __cplusplus
}
#endif
#endif
