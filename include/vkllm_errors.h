/* Error codes of the vkllm C API.
 *
 * Replaces src/core/vkllm_errors.h:9-13 + src/core/vkllm_errors.inc:6-11 of the reference.
 * The enumerator values are part of the ABI and are kept identical: VKLLM_ERR_OK == 1.
 * VKLLM_ERR_VULKAN keeps its name and now means "device / CUDA runtime error".
 */
#ifndef VKLLM_ERRORS_H
#define VKLLM_ERRORS_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum
{
    VKLLM_ERR_START = 0,
    VKLLM_ERR_OK,                 /* 1 */
    VKLLM_ERR_ALLOC,              /* 2: host or device allocation failed */
    VKLLM_ERR_VULKAN,             /* 3: device runtime error (a CUDA call failed, or a device wait timed out) */
    VKLLM_ERR_DEV_NOT_FOUND,      /* 4: no such device ordinal */
    VKLLM_ERR_PIPELINE_NOT_FOUND, /* 5: no kernel for this dtype combination */
    VKLLM_ERR_ARGS,               /* 6: invalid arguments / shapes */
} vkllm_err_t;

/* Name of an error code; vkllm_err_s(VKLLM_ERR_OK) == "VKLLM_ERR_OK" (reference: src/core/vkllm_errors.c:3-13). */
extern const char *vkllm_err_s(vkllm_err_t err);

#ifdef __cplusplus
}
#endif
#endif
