/* Kernel table entries (replaces the Vulkan pipelines of src/core/vkllm_pipeline.h:43-74).
 *
 * A pipeline here names one CUDA kernel variant chosen by an op's init (e.g. "mat_mul_vec_f16f32").
 * Per-pipeline timing follows src/core/vkllm_pipeline.c:318-331: when node timing is enabled
 * (environment VKLLM_NODE_TIMING=1) every launch in the op-by-op executor is bracketed by CUDA events
 * and the last duration is kept on the pipeline, so, as in the reference, nodes sharing a pipeline
 * see the last launch only.
 */
#ifndef VKLLM_PIPELINE_H
#define VKLLM_PIPELINE_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include "vkllm_ops.h"
#include <stdint.h>

struct vkllm_context;

struct vkllm_pipeline
{
    char name[64];
    vkllm_op_t op;
    int variant;
    void *ev_start, *ev_end; /* cudaEvent_t, created when timing is enabled */
    int timed;               /* ev_start/ev_end bracket a completed launch */
};

/* Nanoseconds of the last timed launch through `pipeline` (0 when timing is off). */
extern vkllm_err_t vkllm_pipeline_query_exec_time(struct vkllm_context *context, struct vkllm_pipeline *pipeline,
                                                  uint64_t *time_ns);

#ifdef __cplusplus
}
#endif
#endif
