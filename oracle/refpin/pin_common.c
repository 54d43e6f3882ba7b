/* TEST INFRASTRUCTURE (oracle pin). Exports the reference's own fp16 <-> fp32 helpers
 * (src/core/vkllm_common.h:125-186), which its tests' CPU references use for every fp16 store, and
 * compiles its dtype table (src/core/vkllm_dtypes.c) for vkllm_get_dtype_info. */
#include "src/core/vkllm_common.h"
#include "src/core/vkllm_dtypes.c"
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT uint16_t refpin_fp32_to_fp16(float v)
{
    vkllm_fp16_pack p = vkllm_fp32_to_fp16(v);
    uint16_t bits;
    memcpy(&bits, &p, sizeof(bits));
    return bits;
}

REFPIN_EXPORT float refpin_fp16_to_fp32(uint16_t bits)
{
    vkllm_fp16_pack p;
    memcpy(&p, &bits, sizeof(bits));
    return vkllm_fp16_to_fp32(p);
}
