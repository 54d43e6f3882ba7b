// Device-side helpers shared by the op kernels and the fused engine (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace vkb
{

// A 4-D view in ELEMENT strides, [B, C, H, W] with W innermost.
struct Desc4
{
    uint32_t shape[4];
    uint32_t stride[4];
};

__host__ __device__ inline uint64_t d4_offset(const Desc4 &d, uint32_t b, uint32_t c, uint32_t h, uint32_t w)
{
    return (uint64_t)b * d.stride[0] + (uint64_t)c * d.stride[1] + (uint64_t)h * d.stride[2] +
           (uint64_t)w * d.stride[3];
}

__host__ __device__ inline uint64_t d4_count(const Desc4 &d)
{
    return (uint64_t)d.shape[0] * d.shape[1] * d.shape[2] * d.shape[3];
}

// Linear index -> (b, c, h, w) over shape `s`, W fastest.
__host__ __device__ inline void d4_unravel(const uint32_t *s, uint64_t i, uint32_t &b, uint32_t &c, uint32_t &h,
                                           uint32_t &w)
{
    w = (uint32_t)(i % s[3]);
    i /= s[3];
    h = (uint32_t)(i % s[2]);
    i /= s[2];
    c = (uint32_t)(i % s[1]);
    b = (uint32_t)(i / s[1]);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v)
{
    return v;
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v)
{
    return __half2float(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v)
{
    return v;
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v)
{
    return __float2half_rn(v);
}

// Rounds an fp32 value through fp16 and back (the reference materialises every node as fp16).
__device__ __forceinline__ float round_f16(float v)
{
    return __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// SiLU as the reference evaluates it: v / (1 + exp(-v)) in fp32.
__device__ __forceinline__ float silu_f32(float v)
{
    return v / (1.0f + expf(-v));
}

// 16-byte streaming load that bypasses L1 (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Dot product of 8 fp16 pairs packed in two uint4, accumulated in fp32.
__device__ __forceinline__ float dot8_f16(const uint4 &a, const uint4 &b, float acc)
{
    const __half2 *x = reinterpret_cast<const __half2 *>(&a);
    const __half2 *y = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        float2 fx = __half22float2(x[i]);
        float2 fy = __half22float2(y[i]);
        acc = fmaf(fx.x, fy.x, acc);
        acc = fmaf(fx.y, fy.y, acc);
    }
    return acc;
}

// fp16 -> fp32 without the conversion pipe: placing the fp16 exponent/mantissa bits of a half at
// fp32 bit 13 (sign at bit 31) gives exactly h * 2^-112 for every finite half, subnormals included
// (they become fp32 denormals with the same ratio). Two halves packed in a word take a shift and a
// LOP3 each. Multiplying by an operand pre-scaled by 2^112 then yields exactly the fp32 product of
// the original values, so sums are bit-identical to fma(float(x), float(h), acc).
constexpr float kHalfBitsScale = 0x1p112f;

__device__ __forceinline__ float2 half2_bits_scaled(uint32_t v)
{
    const float lo = __uint_as_float(((v << 13) & 0x0fffe000u) | ((v << 16) & 0x80000000u));
    const float hi = __uint_as_float(((v >> 3) & 0x0fffe000u) | (v & 0x80000000u));
    return make_float2(lo, hi);
}

// acc + sum_i xs[i] * w[i] for 8 fp16 weights `w` and 8 staged activations `xs` that were
// multiplied by kHalfBitsScale (xs0 holds elements 0-3, xs1 elements 4-7).
__device__ __forceinline__ float dot8_scaled(const float4 &xs0, const float4 &xs1, const uint4 &w, float acc)
{
    const float2 w0 = half2_bits_scaled(w.x), w1 = half2_bits_scaled(w.y), w2 = half2_bits_scaled(w.z),
                 w3 = half2_bits_scaled(w.w);
    acc = fmaf(xs0.x, w0.x, acc);
    acc = fmaf(xs0.y, w0.y, acc);
    acc = fmaf(xs0.z, w1.x, acc);
    acc = fmaf(xs0.w, w1.y, acc);
    acc = fmaf(xs1.x, w2.x, acc);
    acc = fmaf(xs1.y, w2.y, acc);
    acc = fmaf(xs1.z, w3.x, acc);
    acc = fmaf(xs1.w, w3.y, acc);
    return acc;
}

} // namespace vkb
