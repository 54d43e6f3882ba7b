/* Element types (reference: src/core/vkllm_dtypes.h:11-31, src/core/vkllm_dtypes.inc:5-8). Values kept. */
#ifndef VKLLM_DTYPES_H
#define VKLLM_DTYPES_H

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include <stdint.h>

typedef enum
{
    vkllm_dtype_start = 0,
    vkllm_dtype_float32, /* 1 */
    vkllm_dtype_float16, /* 2 */
    vkllm_dtype_int8,    /* 3 */
    vkllm_dtype_uint32,  /* 4 */
} vkllm_dtype_t;

struct vkllm_dtype_info
{
    vkllm_dtype_t dtype;
    uint32_t bytes;
    uint32_t items_per_block;
    uint32_t bytes_per_block;
};

/* reference: src/core/vkllm_dtypes.c:3-13 */
extern const char *vkllm_dtype_s(vkllm_dtype_t dtype);
/* reference: src/core/vkllm_dtypes.c:15-48; VKLLM_ERR_ARGS for an unknown dtype */
extern vkllm_err_t vkllm_get_dtype_info(vkllm_dtype_t dtype, struct vkllm_dtype_info *info);

#ifdef __cplusplus
}
#endif
#endif
