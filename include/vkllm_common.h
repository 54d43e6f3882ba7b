/* Shared macros, limits and fp16 helpers of the C API (reference: src/core/vkllm_common.h:13-186).
 *
 * The check macros keep their names and behaviour because callers use them (the reference's tests
 * and token loop do). The fp16 helpers keep the reference's conversion semantics, which callers
 * rely on to prepare inputs: fp32 -> fp16 TRUNCATES the mantissa and clamps the exponent
 * (src/core/vkllm_common.h:157-186); it is not round-to-nearest. Device kernels round to nearest even.
 */
#ifndef VKLLM_COMMON_H
#define VKLLM_COMMON_H

#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef __cplusplus
extern "C" {
#endif

#include "vkllm_errors.h"
#include "vkllm_log.h"

#define _NEW_AND_CHECK(_p, _type)                                                                                      \
    do                                                                                                                 \
    {                                                                                                                  \
        (_p) = (_type *)malloc(sizeof(_type));                                                                         \
        if (!(_p))                                                                                                     \
            return VKLLM_ERR_ALLOC;                                                                                    \
    } while (0)

#define _NEW_N_AND_CHECK(_p, _type, _n)                                                                                \
    do                                                                                                                 \
    {                                                                                                                  \
        (_p) = (_type *)malloc(sizeof(_type) * (_n));                                                                  \
        if (!(_p))                                                                                                     \
            return VKLLM_ERR_ALLOC;                                                                                    \
    } while (0)

#define _CHECK(fn)                                                                                                     \
    do                                                                                                                 \
    {                                                                                                                  \
        vkllm_err_t __r = (fn);                                                                                        \
        if (__r != VKLLM_ERR_OK)                                                                                       \
            return __r;                                                                                                \
    } while (0)

#define _CHECK_JUMP(_fn, _ret, _label)                                                                                 \
    do                                                                                                                 \
    {                                                                                                                  \
        _ret = (_fn);                                                                                                  \
        if (_ret != VKLLM_ERR_OK)                                                                                      \
            goto _label;                                                                                               \
    } while (0)

#define BOOL_S(_cond) (!!(_cond) ? "true" : "false")

#define _CHECK_ARGS(_cond)                                                                                             \
    do                                                                                                                 \
    {                                                                                                                  \
        if (!(_cond))                                                                                                  \
        {                                                                                                              \
            log_error("%s is false", #_cond);                                                                             \
            return VKLLM_ERR_ARGS;                                                                                     \
        }                                                                                                              \
    } while (0)

#define _DIV4_S(__vec4, __den, __out)                                                                                  \
    do                                                                                                                 \
    {                                                                                                                  \
        (__out)[0] = (__vec4)[0] / (__den);                                                                            \
        (__out)[1] = (__vec4)[1] / (__den);                                                                            \
        (__out)[2] = (__vec4)[2] / (__den);                                                                            \
        (__out)[3] = (__vec4)[3] / (__den);                                                                            \
    } while (0)

#define _MUL4(__vec4) ((__vec4)[0] * (__vec4)[1] * (__vec4)[2] * (__vec4)[3])
#define _ASSIGN4(_lhs, _rhs)                                                                                           \
    do                                                                                                                 \
    {                                                                                                                  \
        (_lhs)[0] = (_rhs)[0];                                                                                         \
        (_lhs)[1] = (_rhs)[1];                                                                                         \
        (_lhs)[2] = (_rhs)[2];                                                                                         \
        (_lhs)[3] = (_rhs)[3];                                                                                         \
    } while (0)

#define _ARRAY_SIZE(_arr) (sizeof(_arr) / sizeof((_arr)[0]))
#define __PACKED__ __attribute__((packed))
#define __UNUSED(__x) ((void)__x)

#define VKLLM_MAX_PHY_DEVS 16
#define VKLLM_MAX_SRCS 4

/* IEEE binary16 bit pattern. The reference declares it as a packed bit-field struct; here it is
 * a plain 16-bit word wrapped in a struct so the type stays distinct and 2 bytes wide. */
typedef struct vkllm_fp16_pack
{
    uint16_t bits;
} vkllm_fp16_pack;

static inline float vkllm_fp16_to_fp32(vkllm_fp16_pack h)
{
    uint32_t sign = (uint32_t)(h.bits >> 15) & 1u;
    uint32_t exp = (uint32_t)(h.bits >> 10) & 0x1fu;
    uint32_t frac = (uint32_t)h.bits & 0x3ffu;
    uint32_t out;
    if (exp == 31u && frac != 0u)
        out = (sign << 31) | (255u << 23) | 1u; /* NaN */
    else
    {
        /* Exponent 31 maps to 255, 0 stays 0 (the fraction is kept, giving an fp32 denormal), the rest re-biased. */
        uint32_t e = exp == 31u ? 255u : (exp == 0u ? 0u : exp - 15u + 127u);
        out = (sign << 31) | (e << 23) | (frac << 13);
    }
    float f;
    memcpy(&f, &out, sizeof(f));
    return f;
}

static inline vkllm_fp16_pack vkllm_fp32_to_fp16(float f)
{
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    uint32_t sign = u >> 31, exp = (u >> 23) & 0xffu, frac = u & 0x7fffffu;
    vkllm_fp16_pack h;
    if (exp == 255u && frac != 0u)
    {
        h.bits = (uint16_t)((sign << 15) | (31u << 10) | 1u);
        return h;
    }
    int e = (int)exp - 127;
    uint32_t he = e < -14 ? 0u : (e > 15 ? 31u : (uint32_t)(e + 15));
    h.bits = (uint16_t)((sign << 15) | (he << 10) | (frac >> 13));
    return h;
}

#ifdef __cplusplus
}
#endif
#endif
