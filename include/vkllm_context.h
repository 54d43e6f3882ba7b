/* Device context (reference: src/core/vkllm_context.h:19-112, src/core/vkllm_context.c:8-35).
 *
 * The reference context owns a Vulkan device and ~150 prebuilt SPIR-V pipelines. Here it owns a
 * CUDA device (ordinal `dev`), its streams, a caching device/pinned-host allocator and the kernel
 * table; those live behind the opaque `runtime` pointer. `appname`, `device` and `stats` keep their
 * names and meaning (the reference token loop reads stats under _LOG_NODE_TIME_COST).
 */
#ifndef VKLLM_CONTEXT_H
#define VKLLM_CONTEXT_H

#include "vkllm_common.h"
#ifdef __cplusplus
extern "C" {
#endif

#include <stdint.h>

#include "vkllm_errors.h"
#include "vkllm_ops.h"

struct vkllm_gpu_device; /* opaque: CUDA device ordinal, properties, SM count */
struct vkllm_hashmap;
struct vkllm_b200_runtime; /* opaque: streams, allocator, engine caches */

struct vkllm_context
{
    const char *appname;
    struct vkllm_gpu_device *device;
    struct vkllm_b200_runtime *runtime;

    struct
    {
        int tensor_alloc_counts;
        int tensor_free_counts;
        uint64_t op_time_costs[(int)VKLLM_OP_COUNTS]; /* nanoseconds, filled when node timing is enabled */
        struct vkllm_hashmap *node_time_cost;         /* node name -> accumulated nanoseconds */
    } stats;
};

/* Creates a context on CUDA device `dev`. VKLLM_ERR_DEV_NOT_FOUND when the ordinal does not exist
 * (or no CUDA device is visible); VKLLM_ERR_VULKAN on any other CUDA error. */
extern vkllm_err_t vkllm_context_new(uint32_t dev, struct vkllm_context **context);
extern void vkllm_context_free(struct vkllm_context *pcontext);

#ifdef __cplusplus
}
#endif
#endif
