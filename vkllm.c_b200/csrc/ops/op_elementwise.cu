// Row/elementwise operators of the op-by-op executor: RMSNORM, ROPE, SOFTMAX, UPDATE_ROWS, BIN, COPY,
// EMBEDDING, ARG_MAX. Each op keeps the reference host checks (src/core/vkllm_op_*.c) and computes
// what the reference shader computes (src/shaders/*.comp), with fp32 arithmetic on fp16 storage
// (the reference's f16f32 variants).
#include <cfloat>

#include "../kernels/common.cuh"
#include "../runtime/internal.h"
#include "vkllm_op_arg_max.h"
#include "vkllm_op_bin.h"
#include "vkllm_op_copy.h"
#include "vkllm_op_embedding.h"
#include "vkllm_op_rmsnorm.h"
#include "vkllm_op_rope.h"
#include "vkllm_op_softmax.h"
#include "vkllm_op_update_rows.h"

using namespace vkb;

namespace
{

Desc4 desc_of(const vkllm_tensor *t)
{
    Desc4 d;
    Strides4 s = elem_strides(t);
    for (int i = 0; i < 4; ++i)
    {
        d.shape[i] = t->shapes[i];
        d.stride[i] = s.s[i];
    }
    return d;
}

bool same_shape(const vkllm_tensor *a, const vkllm_tensor *b)
{
    return a->shapes[0] == b->shapes[0] && a->shapes[1] == b->shapes[1] && a->shapes[2] == b->shapes[2] &&
           a->shapes[3] == b->shapes[3];
}

vkllm_err_t launch_status(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return cuda_check(e, what, __FILE__, __LINE__);
    return VKLLM_ERR_OK;
}

// ------------------------------------------------------------------------------------------------
// RMSNORM (src/shaders/vkllm_rmsnorm.comp:31-82): per row, mean of squares in fp32, alpha =
// rsqrt(mean + eps), y = fp16((x * g) * alpha).
__global__ void k_rmsnorm(const __half *x, Desc4 dx, const float *g, __half *y, Desc4 dy, float eps)
{
    __shared__ float red[32];
    uint32_t row = blockIdx.x;
    uint32_t h = row % dx.shape[2];
    uint32_t c = (row / dx.shape[2]) % dx.shape[1];
    uint32_t b = row / (dx.shape[2] * dx.shape[1]);
    const __half *xr = x + d4_offset(dx, b, c, h, 0);
    __half *yr = y + d4_offset(dy, b, c, h, 0);
    uint32_t W = dx.shape[3];
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < W; i += blockDim.x)
    {
        float v = __half2float(xr[(uint64_t)i * dx.stride[3]]);
        s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32)
    {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0)
            red[0] = t;
    }
    __syncthreads();
    float alpha = rsqrtf(red[0] / (float)W + eps);
    for (uint32_t i = threadIdx.x; i < W; i += blockDim.x)
    {
        float v = __half2float(xr[(uint64_t)i * dx.stride[3]]);
        yr[(uint64_t)i * dy.stride[3]] = __float2half_rn((v * g[i]) * alpha);
    }
}

// Contiguous rows (W % 8 == 0, 16-byte aligned): the same node with 16-byte loads and stores, the
// row held in registers between the two passes (W <= 8 * blockDim.x).
__global__ void k_rmsnorm_vec(const __half *x, Desc4 dx, const float *g, __half *y, Desc4 dy, float eps)
{
    __shared__ float red[32];
    const uint32_t row = blockIdx.x;
    const uint32_t h = row % dx.shape[2], c = (row / dx.shape[2]) % dx.shape[1], b = row / (dx.shape[2] * dx.shape[1]);
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + d4_offset(dx, b, c, h, 0));
    uint4 *yr = reinterpret_cast<uint4 *>(y + d4_offset(dy, b, c, h, 0));
    const uint32_t W = dx.shape[3], n8 = W / 8;
    const uint4 v = threadIdx.x < n8 ? xr[threadIdx.x] : make_uint4(0, 0, 0, 0);
    const __half2 *vh = reinterpret_cast<const __half2 *>(&v);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
    {
        const float2 f = __half22float2(vh[e]);
        s = fmaf(f.x, f.x, s);
        s = fmaf(f.y, f.y, s);
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32)
    {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0)
            red[0] = t;
    }
    __syncthreads();
    const float alpha = rsqrtf(red[0] / (float)W + eps);
    if (threadIdx.x < n8)
    {
        const float4 ga = reinterpret_cast<const float4 *>(g)[2 * threadIdx.x];
        const float4 gb = reinterpret_cast<const float4 *>(g)[2 * threadIdx.x + 1];
        const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 f = __half22float2(vh[e]);
            oh[e] = __floats2half2_rn((f.x * gg[2 * e]) * alpha, (f.y * gg[2 * e + 1]) * alpha);
        }
        yr[threadIdx.x] = o;
    }
}

// The residual BIN (op 0, fp16(float(x) + float(y)), src/shaders/vkllm_bin_op.comp:43-72) and the
// RMSNORM of its result (as k_rmsnorm_vec) in one pass over a dense row: x = x + y, n = rmsnorm(x).
__global__ void k_residual_rmsnorm_vec(__half *__restrict__ x, const __half *__restrict__ y, const float *g,
                                       __half *__restrict__ n, uint32_t W, float eps)
{
    __shared__ float red[32];
    const uint64_t row = blockIdx.x;
    uint4 *xr = reinterpret_cast<uint4 *>(x + row * W);
    const uint4 *yr = reinterpret_cast<const uint4 *>(y + row * W);
    uint4 *nr = reinterpret_cast<uint4 *>(n + row * W);
    const uint32_t n8 = W / 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < n8)
    {
        const uint4 a = xr[threadIdx.x], b = yr[threadIdx.x];
        const __half2 *ah = reinterpret_cast<const __half2 *>(&a), *bh = reinterpret_cast<const __half2 *>(&b);
        __half2 *vh = reinterpret_cast<__half2 *>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 fa = __half22float2(ah[e]), fb = __half22float2(bh[e]);
            vh[e] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
        }
        xr[threadIdx.x] = v;
    }
    const __half2 *vh = reinterpret_cast<const __half2 *>(&v);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
    {
        const float2 f = __half22float2(vh[e]);
        s = fmaf(f.x, f.x, s);
        s = fmaf(f.y, f.y, s);
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32)
    {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0)
            red[0] = t;
    }
    __syncthreads();
    const float alpha = rsqrtf(red[0] / (float)W + eps);
    if (threadIdx.x < n8)
    {
        const float4 ga = reinterpret_cast<const float4 *>(g)[2 * threadIdx.x];
        const float4 gb = reinterpret_cast<const float4 *>(g)[2 * threadIdx.x + 1];
        const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 f = __half22float2(vh[e]);
            oh[e] = __floats2half2_rn((f.x * gg[2 * e]) * alpha, (f.y * gg[2 * e + 1]) * alpha);
        }
        nr[threadIdx.x] = o;
    }
}

// ------------------------------------------------------------------------------------------------
// ROPE (src/shaders/vkllm_rope.comp:39-79): one thread per rotated pair.
template <typename T>
__global__ void k_rope(const T *in, Desc4 di, T *out, Desc4 dout, uint32_t offset, float base, int neox)
{
    uint32_t half_w = di.shape[3] / 2;
    uint64_t n = (uint64_t)di.shape[0] * di.shape[1] * di.shape[2] * half_w;
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        uint32_t w = (uint32_t)(t % half_w);
        uint64_t r = t / half_w;
        uint32_t h = (uint32_t)(r % di.shape[2]);
        r /= di.shape[2];
        uint32_t c = (uint32_t)(r % di.shape[1]);
        uint32_t b = (uint32_t)(r / di.shape[1]);
        uint64_t i0, i1, o0, o1;
        if (neox)
        {
            i0 = d4_offset(di, b, c, h, w);
            i1 = i0 + (uint64_t)di.stride[3] * half_w;
            o0 = d4_offset(dout, b, c, h, w);
            o1 = o0 + (uint64_t)dout.stride[3] * (dout.shape[3] / 2);
        }
        else
        {
            i0 = d4_offset(di, b, c, h, 2 * w);
            i1 = i0 + di.stride[3];
            o0 = d4_offset(dout, b, c, h, 2 * w);
            o1 = o0 + dout.stride[3];
        }
        float theta = (float)(offset + h) / powf(base, (float)(2 * w) / (float)di.shape[3]);
        float cs = cosf(theta), sn = sinf(theta);
        float v0 = to_f32(in[i0]), v1 = to_f32(in[i1]);
        out[o0] = from_f32<T>(cs * v0 - sn * v1);
        out[o1] = from_f32<T>(sn * v0 + cs * v1);
    }
}

// fp16, normal-style pairs, unit innermost strides: the same rotation with one half2 load and store
// per pair of the input and output, 32-bit index arithmetic (n < 2^32).
// The denominators base^(2w / W) are computed once per block into shared memory (the same powf of
// the same arguments, so theta keeps its bits) when W / 2 <= kRopeTab.
constexpr uint32_t kRopeTab = 512;
__global__ void k_rope_h2(const __half *in, Desc4 di, __half *out, Desc4 dout, uint32_t offset, float base)
{
    __shared__ float den_s[kRopeTab];
    const uint32_t half_w = di.shape[3] / 2, H = di.shape[2], Cc = di.shape[1];
    const uint32_t n = di.shape[0] * Cc * H * half_w;
    const bool tab = half_w <= kRopeTab;
    if (tab)
    {
        for (uint32_t w = threadIdx.x; w < half_w; w += blockDim.x)
            den_s[w] = powf(base, (float)(2 * w) / (float)di.shape[3]);
        __syncthreads();
    }
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x)
    {
        const uint32_t w = t % half_w, r = t / half_w, h = r % H, r2 = r / H, c = r2 % Cc, b = r2 / Cc;
        const float den = tab ? den_s[w] : powf(base, (float)(2 * w) / (float)di.shape[3]);
        const float theta = (float)(offset + h) / den;
        const float cs = cosf(theta), sn = sinf(theta);
        const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(in + d4_offset(di, b, c, h, 2 * w)));
        *reinterpret_cast<__half2 *>(out + d4_offset(dout, b, c, h, 2 * w)) =
            __floats2half2_rn(cs * v.x - sn * v.y, sn * v.x + cs * v.y);
    }
}

// As k_rope_h2, four pairs (one 16-byte load and store) per thread, so that the index arithmetic is
// paid once per four rotations: W % 8 == 0, W / 2 <= kRopeTab, 16-byte aligned rows.
__global__ void k_rope_h8(const __half *in, Desc4 di, __half *out, Desc4 dout, uint32_t offset, float base)
{
    __shared__ float den_s[kRopeTab];
    const uint32_t half_w = di.shape[3] / 2, q8 = di.shape[3] / 8, H = di.shape[2], Cc = di.shape[1];
    const uint32_t n = di.shape[0] * Cc * H * q8;
    for (uint32_t w = threadIdx.x; w < half_w; w += blockDim.x)
        den_s[w] = powf(base, (float)(2 * w) / (float)di.shape[3]);
    __syncthreads();
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x)
    {
        const uint32_t qd = t % q8, r = t / q8, h = r % H, r2 = r / H, c = r2 % Cc, b = r2 / Cc;
        const uint4 v = *reinterpret_cast<const uint4 *>(in + d4_offset(di, b, c, h, 8 * qd));
        const __half2 *vh = reinterpret_cast<const __half2 *>(&v);
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e)
        {
            const float theta = (float)(offset + h) / den_s[4 * qd + e];
            const float cs = cosf(theta), sn = sinf(theta);
            const float2 f = __half22float2(vh[e]);
            oh[e] = __floats2half2_rn(cs * f.x - sn * f.y, sn * f.x + cs * f.y);
        }
        *reinterpret_cast<uint4 *>(out + d4_offset(dout, b, c, h, 8 * qd)) = o;
    }
}

// ------------------------------------------------------------------------------------------------
// SOFTMAX (src/shaders/vkllm_softmax.comp:42-96): one warp per row; max over ALL entries, sum over
// unmasked ones, masked outputs 0. Input addressed with the output layout, as in the reference.
template <typename T> __global__ void k_softmax(const T *in, T *out, Desc4 d, int seq_mask, uint32_t offsets)
{
    uint64_t rows = (uint64_t)d.shape[0] * d.shape[1] * d.shape[2];
    uint64_t row = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    uint32_t h = (uint32_t)(row % d.shape[2]);
    uint32_t c = (uint32_t)((row / d.shape[2]) % d.shape[1]);
    uint32_t b = (uint32_t)(row / ((uint64_t)d.shape[2] * d.shape[1]));
    uint64_t base = d4_offset(d, b, c, h, 0);
    uint32_t W = d.shape[3];
    float m = to_f32(in[base]);
    for (uint32_t i = lane; i < W; i += 32)
        m = fmaxf(m, to_f32(in[base + (uint64_t)i * d.stride[3]]));
    m = warp_max(m);
    float s = 0.f;
    for (uint32_t i = lane; i < W; i += 32)
    {
        if (seq_mask > 0 && i > h + offsets)
            continue;
        s += expf(to_f32(in[base + (uint64_t)i * d.stride[3]]) - m);
    }
    s = warp_sum(s);
    for (uint32_t i = lane; i < W; i += 32)
    {
        uint64_t o = base + (uint64_t)i * d.stride[3];
        if (seq_mask > 0 && i > h + offsets)
            out[o] = from_f32<T>(0.f);
        else
            out[o] = from_f32<T>(expf(to_f32(in[o]) - m) / s);
    }
}

// Long rows (W >= 1024, e.g. decode scores over a long cache): one block per row, same node.
template <typename T> __global__ void k_softmax_block(const T *in, T *out, Desc4 d, int seq_mask, uint32_t offsets)
{
    __shared__ float red[32];
    const uint32_t row = blockIdx.x;
    const uint32_t h = row % d.shape[2], c = (row / d.shape[2]) % d.shape[1], b = row / (d.shape[2] * d.shape[1]);
    const uint64_t base = d4_offset(d, b, c, h, 0);
    const uint32_t W = d.shape[3], nw = blockDim.x >> 5, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // each pass reads this thread's elements i = tid + k * blockDim eight at a time (all loads of a
    // group issued before their uses); the sums still run in increasing k
    const uint32_t nt = blockDim.x;
    auto load8 = [&](uint32_t i0, float (&xs)[8]) {
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = i0 + u * nt;
            xs[u] = i < W ? to_f32(in[base + (uint64_t)i * d.stride[3]]) : 0.f;
        }
    };
    float m = to_f32(in[base]);
    for (uint32_t i0 = threadIdx.x; i0 < W; i0 += 8 * nt)
    {
        float xs[8];
        load8(i0, xs);
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
            if (i0 + u * nt < W)
                m = fmaxf(m, xs[u]);
    }
    m = warp_max(m);
    if (lane == 0)
        red[warp] = m;
    __syncthreads();
    m = red[0];
    for (uint32_t w = 1; w < nw; ++w)
        m = fmaxf(m, red[w]);
    __syncthreads();
    float s = 0.f;
    for (uint32_t i0 = threadIdx.x; i0 < W; i0 += 8 * nt)
    {
        float xs[8];
        load8(i0, xs);
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = i0 + u * nt;
            if (i < W && !(seq_mask > 0 && i > h + offsets))
                s += expf(xs[u] - m);
        }
    }
    s = warp_sum(s);
    if (lane == 0)
        red[warp] = s;
    __syncthreads();
    float tot = 0.f;
    for (uint32_t w = 0; w < nw; ++w)
        tot += red[w];
    for (uint32_t i0 = threadIdx.x; i0 < W; i0 += 8 * nt)
    {
        float xs[8];
        load8(i0, xs); // each element is read and then written by the same thread (in may be out)
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = i0 + u * nt;
            if (i >= W)
                continue;
            const uint64_t o = base + (uint64_t)i * d.stride[3];
            if (seq_mask > 0 && i > h + offsets)
                out[o] = from_f32<T>(0.f);
            else
                out[o] = from_f32<T>(expf(xs[u] - m) / tot);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// UPDATE_ROWS / COPY: strided element copies (src/shaders/vkllm_update_rows.comp:21-46,
// src/shaders/vkllm_copy.comp:35-50).
template <typename T> __global__ void k_update_rows(const T *in, Desc4 di, T *out, Desc4 dout, uint32_t off_rows)
{
    uint64_t n = d4_count(di);
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        uint32_t b, c, h, w;
        d4_unravel(di.shape, t, b, c, h, w);
        uint32_t oh = h + off_rows;
        if (oh >= dout.shape[2])
            continue;
        out[d4_offset(dout, b, c, oh, w)] = in[d4_offset(di, b, c, h, w)];
    }
}

template <typename T> __global__ void k_copy(const T *in, Desc4 di, T *out, Desc4 dout)
{
    uint64_t n = d4_count(di);
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        uint32_t b, c, h, w;
        d4_unravel(di.shape, t, b, c, h, w);
        out[d4_offset(dout, b, c, h, w)] = in[d4_offset(di, b, c, h, w)];
    }
}

// ------------------------------------------------------------------------------------------------
// BIN (src/shaders/vkllm_bin_op.comp:41-73): same offset (output layout) for all three operands.
template <typename TI, typename TO> __global__ void k_bin(const TI *a, const TI *bb, TO *out, Desc4 d, int op)
{
    uint64_t n = d4_count(d);
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        uint32_t b, c, h, w;
        d4_unravel(d.shape, t, b, c, h, w);
        uint64_t o = d4_offset(d, b, c, h, w);
        float x = to_f32(a[o]), y = to_f32(bb[o]);
        float r = op == 0 ? x + y : (op == 1 ? x - y : (op == 2 ? x * y : x / y));
        out[o] = from_f32<TO>(r);
    }
}

// Dense fp16 operands, 8 elements per thread (16-byte loads and stores).
template <typename TO> __global__ void k_bin_h8(const __half *a, const __half *bb, TO *out, uint64_t n8, int op)
{
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n8; t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint4 va = reinterpret_cast<const uint4 *>(a)[t], vb = reinterpret_cast<const uint4 *>(bb)[t];
        const __half *ha = reinterpret_cast<const __half *>(&va), *hb = reinterpret_cast<const __half *>(&vb);
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float x = __half2float(ha[i]), y = __half2float(hb[i]);
            r[i] = op == 0 ? x + y : (op == 1 ? x - y : (op == 2 ? x * y : x / y));
        }
        if constexpr (sizeof(TO) == 2)
        {
            uint4 o;
            __half *ho = reinterpret_cast<__half *>(&o);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                ho[i] = __float2half_rn(r[i]);
            reinterpret_cast<uint4 *>(out)[t] = o;
        }
        else
        {
            reinterpret_cast<float4 *>(out)[2 * t] = make_float4(r[0], r[1], r[2], r[3]);
            reinterpret_cast<float4 *>(out)[2 * t + 1] = make_float4(r[4], r[5], r[6], r[7]);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// EMBEDDING (src/shaders/vkllm_embedding.comp:41-70): one block per id. The reference addresses the
// output with strides shifted by one axis (out = c*s0 + h*s1 + w*s2), which for ids [1,1,1,S] and
// output [1,1,S,D] is row s; that addressing is kept.
template <typename T>
__global__ void k_embedding(const uint32_t *ids, Desc4 di, const T *table, Desc4 dt, T *out, Desc4 dout,
                            uint32_t unk)
{
    uint64_t id = blockIdx.x;
    uint32_t b, c, h, w;
    d4_unravel(di.shape, id, b, c, h, w);
    uint32_t tok = ids[d4_offset(di, b, c, h, w)];
    if (tok >= dt.shape[2])
        tok = unk;
    uint64_t o = (uint64_t)c * dout.stride[0] + (uint64_t)h * dout.stride[1] + (uint64_t)w * dout.stride[2];
    const T *src = table + (uint64_t)tok * dt.stride[2];
    T *dst = out + o;
    uint32_t dim = dt.shape[3];
    // 16-byte vector path when both rows are aligned.
    constexpr uint32_t V = 16 / sizeof(T);
    if ((((uintptr_t)src | (uintptr_t)dst) & 15) == 0 && dim % V == 0)
    {
        const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
        uint4 *d4 = reinterpret_cast<uint4 *>(dst);
        const uint32_t n4 = dim / V, nt = blockDim.x;
        for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += 4 * nt) // four 16-byte loads in flight, then the stores
        {
            uint4 t[4];
#pragma unroll
            for (uint32_t u = 0; u < 4; ++u)
                if (i0 + u * nt < n4)
                    t[u] = s4[i0 + u * nt];
#pragma unroll
            for (uint32_t u = 0; u < 4; ++u)
                if (i0 + u * nt < n4)
                    d4[i0 + u * nt] = t[u];
        }
    }
    else
    {
        for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x)
            dst[i] = src[i];
    }
}

// ------------------------------------------------------------------------------------------------
// ARG_MAX (src/shaders/vkllm_arg_max.comp:40-97) with the reference tie rule: lane l scans
// i = l, l+32, ... keeping its first strict maximum; then offsets 16,8,4,2,1 keep the left value
// unless the right one is strictly greater. One warp per row.
template <typename T> __global__ void k_arg_max(const T *in, Desc4 di, uint32_t *out, Desc4 dout)
{
    uint64_t rows = (uint64_t)di.shape[0] * di.shape[1] * di.shape[2];
    uint64_t row = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    uint32_t h = (uint32_t)(row % di.shape[2]);
    uint32_t c = (uint32_t)((row / di.shape[2]) % di.shape[1]);
    uint32_t b = (uint32_t)(row / ((uint64_t)di.shape[2] * di.shape[1]));
    uint64_t base = d4_offset(di, b, c, h, 0);
    uint32_t W = di.shape[3];
    float mv = -FLT_MAX;
    uint32_t mi = lane;
    if (lane < W)
        mv = to_f32(in[base + (uint64_t)lane * di.stride[3]]);
    for (uint32_t i = lane + 32; i < W; i += 32)
    {
        float v = to_f32(in[base + (uint64_t)i * di.stride[3]]);
        if (v > mv)
        {
            mv = v;
            mi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        float ov = __shfl_down_sync(0xffffffffu, mv, o);
        uint32_t oi = __shfl_down_sync(0xffffffffu, mi, o);
        if ((int)lane < o && ov > mv)
        {
            mv = ov;
            mi = oi;
        }
    }
    if (lane == 0)
        out[d4_offset(dout, b, c, h, 0)] = mi;
}

// Long rows: one block per row with the same result. Lane l of the reference scans class l (i = l,
// l + 32, ...) from its first element and replaces on a strict maximum, so the class result is (its
// first element, index l) when that element is NaN (nothing compares greater), else the largest
// non-NaN value at its smallest index. The warps split each class's elements, the per-class results
// are combined in shared memory, then the reference's 16/8/4/2/1 tree runs unchanged.
template <typename T> __global__ void k_arg_max_block(const T *in, Desc4 di, uint32_t *out, Desc4 dout)
{
    __shared__ float cv[32][32];
    __shared__ uint32_t ci[32][32];
    const uint32_t row = blockIdx.x;
    const uint32_t h = row % di.shape[2], c = (row / di.shape[2]) % di.shape[1], b = row / (di.shape[2] * di.shape[1]);
    const uint64_t base = d4_offset(di, b, c, h, 0);
    const uint32_t W = di.shape[3], nw = blockDim.x >> 5, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float v = -FLT_MAX;
    uint32_t idx = 0xffffffffu;
    // this thread's elements i = lane + 32 warp + k * 32 nw: eight loads in flight at a time, then the
    // comparisons in increasing k
    const uint32_t stride = 32 * nw;
    for (uint32_t i0 = lane + 32 * warp; i0 < W; i0 += 8 * stride)
    {
        float xs[8];
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = i0 + u * stride;
            xs[u] = i < W ? to_f32(in[base + (uint64_t)i * di.stride[3]]) : 0.f;
        }
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = i0 + u * stride;
            if (i < W && xs[u] == xs[u] && (idx == 0xffffffffu || xs[u] > v)) // NaN never wins a strict comparison
            {
                v = xs[u];
                idx = i;
            }
        }
    }
    cv[warp][lane] = v;
    ci[warp][lane] = idx;
    __syncthreads();
    if (warp != 0)
        return;
    float mv = -FLT_MAX;
    uint32_t mi = 0xffffffffu;
    for (uint32_t w = 0; w < nw; ++w) // the warps interleave a class's elements: ties go to the smaller index
        if (ci[w][lane] != 0xffffffffu &&
            (mi == 0xffffffffu || cv[w][lane] > mv || (cv[w][lane] == mv && ci[w][lane] < mi)))
        {
            mv = cv[w][lane];
            mi = ci[w][lane];
        }
    if (lane < W)
    {
        const float first = to_f32(in[base + (uint64_t)lane * di.stride[3]]);
        if (first != first || mi == 0xffffffffu)
        {
            mv = first;
            mi = lane;
        }
    }
    else
    {
        mv = -FLT_MAX; // no element in this class: the reference's initial lane state
        mi = lane;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const float ov = __shfl_down_sync(0xffffffffu, mv, o);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, mi, o);
        if ((int)lane < o && ov > mv)
        {
            mv = ov;
            mi = oi;
        }
    }
    if (lane == 0)
        out[d4_offset(dout, b, c, h, 0)] = mi;
}

} // namespace

// =================================================================================================
// RMSNORM (reference host: src/core/vkllm_op_rmsnorm.c:11-124)
extern "C" vkllm_err_t vkllm_op_rmsnorm_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0] && tensor->srcs[1]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_RMSNORM);
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    _CHECK_ARGS(same_shape(in0, tensor));
    _CHECK_ARGS(in1->shapes[0] == 1 && in1->shapes[1] == 1 && in1->shapes[2] == 1);
    _CHECK_ARGS(in1->shapes[3] == in0->shapes[3]);
    if (!(tensor->dtype == vkllm_dtype_float16 && in0->dtype == vkllm_dtype_float16 &&
          in1->dtype == vkllm_dtype_float32))
        return VKLLM_ERR_PIPELINE_NOT_FOUND;
    tensor->pipeline = get_pipeline(context, "rmsnorm_f16f32f16", VKLLM_OP_RMSNORM, 0);
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_rmsnorm_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0] && tensor->srcs[1]);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_rmsnorm_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    const vkllm_op_rmsnorm_params *p = (const vkllm_op_rmsnorm_params *)tensor->params;
    void *x = dev_ptr(context, in0), *g = dev_ptr(context, in1), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && g && y);
    cudaStream_t s = stream_of(context, commands);
    uint32_t rows = in0->shapes[0] * in0->shapes[1] * in0->shapes[2];
    timing_begin(context, tensor->pipeline, s);
    const Desc4 dx = desc_of(in0), dy = desc_of(tensor);
    const uint32_t W = in0->shapes[3];
    const bool vec = dx.stride[3] == 1 && dy.stride[3] == 1 && W % 8 == 0 && W / 8 <= 1024 && dx.stride[2] % 8 == 0 &&
                     dy.stride[2] % 8 == 0 && dx.stride[1] % 8 == 0 && dy.stride[1] % 8 == 0 && dx.stride[0] % 8 == 0 &&
                     dy.stride[0] % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0 &&
                     ((uintptr_t)g & 15) == 0;
    if (vec)
        k_rmsnorm_vec<<<rows, (W / 8 + 31) / 32 * 32, 0, s>>>((const __half *)x, dx, (const float *)g, (__half *)y, dy,
                                                               p->eps);
    else
        k_rmsnorm<<<rows, 512, 0, s>>>((const __half *)x, dx, (const float *)g, (__half *)y, dy, p->eps);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_rmsnorm");
}

extern "C" vkllm_err_t vkllm_op_rmsnorm_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// ROPE (reference host: src/core/vkllm_op_rope.c:9-153)
extern "C" vkllm_err_t vkllm_op_rope_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_ROPE);
    vkllm_tensor *in0 = tensor->srcs[0];
    _CHECK_ARGS(same_shape(in0, tensor));
    _CHECK_ARGS(in0->dtype == tensor->dtype);
    const vkllm_op_rope_params *p = (const vkllm_op_rope_params *)tensor->params;
    int neox = p->neox_style ? 1 : 0;
    if (in0->dtype == vkllm_dtype_float16)
        tensor->pipeline = get_pipeline(context, neox ? "rope_f16f32_neox" : "rope_f16f32", VKLLM_OP_ROPE, neox);
    else if (in0->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, neox ? "rope_f32f32_neox" : "rope_f32f32", VKLLM_OP_ROPE, neox);
    else
    {
        log_error("unsupported op input dtype: %s", vkllm_dtype_s(in0->dtype));
        return VKLLM_ERR_ARGS;
    }
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_rope_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_ROPE);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_rope_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0];
    const vkllm_op_rope_params *p = (const vkllm_op_rope_params *)tensor->params;
    void *x = dev_ptr(context, in0), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && y);
    cudaStream_t s = stream_of(context, commands);
    uint64_t n = (uint64_t)in0->shapes[0] * in0->shapes[1] * in0->shapes[2] * (in0->shapes[3] / 2);
    if (n == 0)
        return VKLLM_ERR_OK;
    unsigned grid = grid_1d(n, 256);
    timing_begin(context, tensor->pipeline, s);
    const Desc4 di = desc_of(in0), dout = desc_of(tensor);
    const bool h2 = in0->dtype == vkllm_dtype_float16 && !p->neox_style && di.stride[3] == 1 && dout.stride[3] == 1 &&
                    in0->shapes[3] % 2 == 0 && di.stride[2] % 2 == 0 && di.stride[1] % 2 == 0 &&
                    di.stride[0] % 2 == 0 && dout.stride[2] % 2 == 0 && dout.stride[1] % 2 == 0 &&
                    dout.stride[0] % 2 == 0 && ((uintptr_t)x & 3) == 0 && ((uintptr_t)y & 3) == 0 && n < (1ull << 32);
    const bool h8 = h2 && in0->shapes[3] % 8 == 0 && in0->shapes[3] / 2 <= kRopeTab && di.stride[2] % 8 == 0 &&
                    di.stride[1] % 8 == 0 && di.stride[0] % 8 == 0 && dout.stride[2] % 8 == 0 &&
                    dout.stride[1] % 8 == 0 && dout.stride[0] % 8 == 0 && ((uintptr_t)x & 15) == 0 &&
                    ((uintptr_t)y & 15) == 0;
    if (h8)
        k_rope_h8<<<grid_1d(n / 4, 256), 256, 0, s>>>((const __half *)x, di, (__half *)y, dout, p->offset, p->base);
    else if (h2)
        k_rope_h2<<<grid, 256, 0, s>>>((const __half *)x, di, (__half *)y, dout, p->offset, p->base);
    else if (in0->dtype == vkllm_dtype_float16)
        k_rope<__half><<<grid, 256, 0, s>>>((const __half *)x, di, (__half *)y, dout, p->offset, p->base,
                                             p->neox_style ? 1 : 0);
    else
        k_rope<float><<<grid, 256, 0, s>>>((const float *)x, desc_of(in0), (float *)y, desc_of(tensor), p->offset,
                                            p->base, p->neox_style ? 1 : 0);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_rope");
}

extern "C" vkllm_err_t vkllm_op_rope_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// SOFTMAX (reference host: src/core/vkllm_op_softmax.c:9-128)
extern "C" vkllm_err_t vkllm_op_softmax_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_SOFTMAX);
    vkllm_tensor *in0 = tensor->srcs[0];
    _CHECK_ARGS(same_shape(in0, tensor));
    if (tensor->dtype != in0->dtype)
    {
        log_error("softmax input and output dtype mismatch: input=%s, output=%s", vkllm_dtype_s(in0->dtype),
                  vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    if (in0->dtype == vkllm_dtype_float16)
        tensor->pipeline = get_pipeline(context, "softmax_f16f32", VKLLM_OP_SOFTMAX, 0);
    else if (in0->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, "softmax_f32f32", VKLLM_OP_SOFTMAX, 1);
    else
    {
        log_error("unsupported softmax dtype: %s", vkllm_dtype_s(in0->dtype));
        return VKLLM_ERR_ARGS;
    }
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_softmax_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_SOFTMAX);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_softmax_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0];
    const vkllm_op_softmax_params *p = (const vkllm_op_softmax_params *)tensor->params;
    void *x = dev_ptr(context, in0), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && y);
    cudaStream_t s = stream_of(context, commands);
    uint64_t rows = (uint64_t)tensor->shapes[0] * tensor->shapes[1] * tensor->shapes[2];
    unsigned grid = grid_1d(rows * 32, 256);
    timing_begin(context, tensor->pipeline, s);
    const bool block = tensor->shapes[3] >= 1024 && rows <= 0x7fffffffu;
    if (block && in0->dtype == vkllm_dtype_float16)
        k_softmax_block<__half><<<(unsigned)rows, 256, 0, s>>>((const __half *)x, (__half *)y, desc_of(tensor),
                                                                p->seq_mask, p->offsets);
    else if (block)
        k_softmax_block<float><<<(unsigned)rows, 256, 0, s>>>((const float *)x, (float *)y, desc_of(tensor), p->seq_mask,
                                                               p->offsets);
    else if (in0->dtype == vkllm_dtype_float16)
        k_softmax<__half><<<grid, 256, 0, s>>>((const __half *)x, (__half *)y, desc_of(tensor), p->seq_mask,
                                                p->offsets);
    else
        k_softmax<float><<<grid, 256, 0, s>>>((const float *)x, (float *)y, desc_of(tensor), p->seq_mask, p->offsets);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_softmax");
}

extern "C" vkllm_err_t vkllm_op_softmax_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// UPDATE_ROWS (reference host: src/core/vkllm_op_update_rows.c:9-118)
extern "C" vkllm_err_t vkllm_op_update_rows_init(vkllm_context *context, vkllm_commands *commands,
                                                 vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_UPDATE_ROWS);
    vkllm_tensor *in0 = tensor->srcs[0];
    _CHECK_ARGS(in0->shapes[0] == tensor->shapes[0]);
    _CHECK_ARGS(in0->shapes[1] == tensor->shapes[1]);
    _CHECK_ARGS(in0->shapes[3] == tensor->shapes[3]);
    const vkllm_op_update_rows_params *p = (const vkllm_op_update_rows_params *)tensor->params;
    _CHECK_ARGS((uint64_t)p->offset_rows + in0->shapes[2] <= tensor->shapes[2]);
    if (tensor->dtype != in0->dtype)
    {
        log_error("update_rows input and output dtype mismatch: input=%s, output=%s", vkllm_dtype_s(in0->dtype),
                  vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    if (in0->dtype == vkllm_dtype_float16)
        tensor->pipeline = get_pipeline(context, "update_rows_f16", VKLLM_OP_UPDATE_ROWS, 0);
    else if (in0->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, "update_rows_f32", VKLLM_OP_UPDATE_ROWS, 1);
    else
    {
        log_error("unsupported update_rows dtype: %s", vkllm_dtype_s(in0->dtype));
        return VKLLM_ERR_ARGS;
    }
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_update_rows_run(vkllm_context *context, vkllm_commands *commands,
                                                vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_UPDATE_ROWS);
    // The KV-cache nodes are re-pointed every step, so re-validate on every run.
    _CHECK(vkllm_op_update_rows_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0];
    const vkllm_op_update_rows_params *p = (const vkllm_op_update_rows_params *)tensor->params;
    void *x = dev_ptr(context, in0), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && y);
    cudaStream_t s = stream_of(context, commands);
    uint64_t n = (uint64_t)_MUL4(in0->shapes);
    unsigned grid = grid_1d(n, 256);
    timing_begin(context, tensor->pipeline, s);
    if (in0->dtype == vkllm_dtype_float16)
        k_update_rows<__half><<<grid, 256, 0, s>>>((const __half *)x, desc_of(in0), (__half *)y, desc_of(tensor),
                                                    p->offset_rows);
    else
        k_update_rows<float><<<grid, 256, 0, s>>>((const float *)x, desc_of(in0), (float *)y, desc_of(tensor),
                                                   p->offset_rows);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_update_rows");
}

extern "C" vkllm_err_t vkllm_op_update_rows_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// BIN (reference host: src/core/vkllm_op_bin.c:9-123)
extern "C" vkllm_err_t vkllm_op_bin_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0] && tensor->srcs[1]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_BIN);
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    _CHECK_ARGS(same_shape(in0, in1) && same_shape(in0, tensor));
    int32_t op = *(const int32_t *)tensor->params;
    _CHECK_ARGS(op >= 0 && op <= 3);
    if (tensor->dtype != vkllm_dtype_float32 && tensor->dtype != vkllm_dtype_float16)
    {
        log_error("tensor: %s unsupported op result dtype: %s", tensor->name, vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    static const char *const f16n[2][4] = {{"bin_f16f32f16_add", "bin_f16f32f16_sub", "bin_f16f32f16_mul",
                                            "bin_f16f32f16_div"},
                                           {"bin_f16f32f32_add", "bin_f16f32f32_sub", "bin_f16f32f32_mul",
                                            "bin_f16f32f32_div"}};
    static const char *const f32n[4] = {"bin_f32f32f32_add", "bin_f32f32f32_sub", "bin_f32f32f32_mul",
                                        "bin_f32f32f32_div"};
    if (in0->dtype == vkllm_dtype_float16 && in1->dtype == vkllm_dtype_float16)
        tensor->pipeline =
            get_pipeline(context, f16n[tensor->dtype == vkllm_dtype_float32 ? 1 : 0][op], VKLLM_OP_BIN, op);
    else if (in0->dtype == vkllm_dtype_float32 && in1->dtype == vkllm_dtype_float32 &&
             tensor->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, f32n[op], VKLLM_OP_BIN, op);
    else
        return VKLLM_ERR_ARGS;
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_bin_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0] && tensor->srcs[1]);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_bin_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    int32_t op = *(const int32_t *)tensor->params;
    void *a = dev_ptr(context, in0), *b = dev_ptr(context, in1), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(a && b && y);
    cudaStream_t s = stream_of(context, commands);
    Desc4 d = desc_of(tensor);
    unsigned grid = grid_1d(d4_count(d), 256);
    timing_begin(context, tensor->pipeline, s);
    const uint64_t n = d4_count(d);
    const bool dense = d.stride[3] == 1 && d.stride[2] == d.shape[3] && d.stride[1] == (uint64_t)d.shape[2] * d.shape[3] &&
                       d.stride[0] == (uint64_t)d.shape[1] * d.shape[2] * d.shape[3] && n % 8 == 0 &&
                       (((uintptr_t)a | (uintptr_t)b | (uintptr_t)y) & 15) == 0;
    if (in0->dtype == vkllm_dtype_float16 && dense)
    {
        const unsigned g8 = grid_1d(n / 8, 256);
        if (tensor->dtype == vkllm_dtype_float16)
            k_bin_h8<__half><<<g8, 256, 0, s>>>((const __half *)a, (const __half *)b, (__half *)y, n / 8, op);
        else
            k_bin_h8<float><<<g8, 256, 0, s>>>((const __half *)a, (const __half *)b, (float *)y, n / 8, op);
    }
    else if (in0->dtype == vkllm_dtype_float16)
    {
        if (tensor->dtype == vkllm_dtype_float16)
            k_bin<__half, __half><<<grid, 256, 0, s>>>((const __half *)a, (const __half *)b, (__half *)y, d, op);
        else
            k_bin<__half, float><<<grid, 256, 0, s>>>((const __half *)a, (const __half *)b, (float *)y, d, op);
    }
    else
        k_bin<float, float><<<grid, 256, 0, s>>>((const float *)a, (const float *)b, (float *)y, d, op);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_bin");
}

extern "C" vkllm_err_t vkllm_op_bin_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// COPY (reference host: src/core/vkllm_op_copy.c:11-123)
extern "C" vkllm_err_t vkllm_op_copy_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_COPY);
    vkllm_tensor *in0 = tensor->srcs[0];
    _CHECK_ARGS(same_shape(in0, tensor));
    if (tensor->dtype != in0->dtype)
    {
        log_error("copy op requires same dtype for src and dst. src: %s, dst: %s", vkllm_dtype_s(in0->dtype),
                  vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    if (tensor->dtype == vkllm_dtype_float16)
        tensor->pipeline = get_pipeline(context, "copy_f16", VKLLM_OP_COPY, 0);
    else if (tensor->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, "copy_f32", VKLLM_OP_COPY, 1);
    else
    {
        log_error("unsupported copy dtype: %s", vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_copy_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0]);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_copy_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0];
    void *x = dev_ptr(context, in0), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && y);
    cudaStream_t s = stream_of(context, commands);
    unsigned grid = grid_1d(_MUL4(tensor->shapes), 256);
    timing_begin(context, tensor->pipeline, s);
    if (tensor->dtype == vkllm_dtype_float16)
        k_copy<uint16_t><<<grid, 256, 0, s>>>((const uint16_t *)x, desc_of(in0), (uint16_t *)y, desc_of(tensor));
    else
        k_copy<uint32_t><<<grid, 256, 0, s>>>((const uint32_t *)x, desc_of(in0), (uint32_t *)y, desc_of(tensor));
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_copy");
}

extern "C" vkllm_err_t vkllm_op_copy_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// EMBEDDING (reference host: src/core/vkllm_op_embedding.c:10-110)
extern "C" vkllm_err_t vkllm_op_embedding_init(vkllm_context *context, vkllm_commands *commands,
                                               vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0] && tensor->srcs[1]);
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    _CHECK_ARGS(in0->dtype == vkllm_dtype_uint32);
    _CHECK_ARGS(in1->dtype == vkllm_dtype_float16 || in1->dtype == vkllm_dtype_float32);
    _CHECK_ARGS(in0->shapes[0] == 1 && in1->shapes[0] == 1 && in1->shapes[1] == 1);
    if ((tensor->dtype != vkllm_dtype_float32 && tensor->dtype != vkllm_dtype_float16) || tensor->dtype != in1->dtype)
    {
        log_error("unsupported op result dtype: %s, dtype of table: %s", vkllm_dtype_s(tensor->dtype),
                  vkllm_dtype_s(in1->dtype));
        return VKLLM_ERR_ARGS;
    }
    // Every gathered row must land inside the output (the reference does not check this).
    {
        Strides4 so = elem_strides(tensor);
        uint64_t last = (uint64_t)(in0->shapes[1] - 1) * so.s[0] + (uint64_t)(in0->shapes[2] - 1) * so.s[1] +
                        (uint64_t)(in0->shapes[3] - 1) * so.s[2] + in1->shapes[3];
        _CHECK_ARGS(last <= (uint64_t)_MUL4(tensor->shapes));
    }
    tensor->pipeline = get_pipeline(context, in1->dtype == vkllm_dtype_float16 ? "embedding_f16" : "embedding_f32",
                                    VKLLM_OP_EMBEDDING, in1->dtype == vkllm_dtype_float16 ? 0 : 1);
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_embedding_run(vkllm_context *context, vkllm_commands *commands,
                                              vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0] && tensor->srcs[1]);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_embedding_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    uint32_t unk = *(const uint32_t *)tensor->params;
    void *ids = dev_ptr(context, in0), *tab = dev_ptr(context, in1), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(ids && tab && y);
    cudaStream_t s = stream_of(context, commands);
    uint32_t n = _MUL4(in0->shapes);
    timing_begin(context, tensor->pipeline, s);
    if (in1->dtype == vkllm_dtype_float16)
        k_embedding<__half><<<n, 128, 0, s>>>((const uint32_t *)ids, desc_of(in0), (const __half *)tab, desc_of(in1),
                                               (__half *)y, desc_of(tensor), unk);
    else
        k_embedding<float><<<n, 128, 0, s>>>((const uint32_t *)ids, desc_of(in0), (const float *)tab, desc_of(in1),
                                              (float *)y, desc_of(tensor), unk);
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_embedding");
}

extern "C" vkllm_err_t vkllm_op_embedding_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// ARG_MAX (reference host: src/core/vkllm_op_arg_max.c:9-121)
extern "C" vkllm_err_t vkllm_op_arg_max_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_ARG_MAX);
    vkllm_tensor *in0 = tensor->srcs[0];
    _CHECK_ARGS(in0->shapes[0] == tensor->shapes[0]);
    _CHECK_ARGS(in0->shapes[1] == tensor->shapes[1]);
    _CHECK_ARGS(in0->shapes[2] == tensor->shapes[2]);
    _CHECK_ARGS(tensor->shapes[3] == 1);
    if (tensor->dtype != vkllm_dtype_uint32)
    {
        log_error("arg_max output dtype must be uint32, got %s", vkllm_dtype_s(tensor->dtype));
        return VKLLM_ERR_ARGS;
    }
    if (in0->dtype == vkllm_dtype_float16)
        tensor->pipeline = get_pipeline(context, "arg_max_f16f32", VKLLM_OP_ARG_MAX, 0);
    else if (in0->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, "arg_max_f32f32", VKLLM_OP_ARG_MAX, 1);
    else
    {
        log_error("unsupported arg_max dtype: %s", vkllm_dtype_s(in0->dtype));
        return VKLLM_ERR_ARGS;
    }
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_arg_max_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0]);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_arg_max_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0];
    void *x = dev_ptr(context, in0), *y = dev_ptr(context, tensor);
    _CHECK_ARGS(x && y);
    cudaStream_t s = stream_of(context, commands);
    uint64_t rows = (uint64_t)in0->shapes[0] * in0->shapes[1] * in0->shapes[2];
    unsigned grid = grid_1d(rows * 32, 128);
    timing_begin(context, tensor->pipeline, s);
    const unsigned bt = in0->shapes[3] >= 8192 ? 1024u : 256u;
    const bool block = in0->shapes[3] >= 1024 && rows <= 0x7fffffffu;
    if (block && in0->dtype == vkllm_dtype_float16)
        k_arg_max_block<__half><<<(unsigned)rows, bt, 0, s>>>((const __half *)x, desc_of(in0), (uint32_t *)y,
                                                              desc_of(tensor));
    else if (block)
        k_arg_max_block<float><<<(unsigned)rows, bt, 0, s>>>((const float *)x, desc_of(in0), (uint32_t *)y,
                                                             desc_of(tensor));
    else if (in0->dtype == vkllm_dtype_float16)
        k_arg_max<__half><<<grid, 128, 0, s>>>((const __half *)x, desc_of(in0), (uint32_t *)y, desc_of(tensor));
    else
        k_arg_max<float><<<grid, 128, 0, s>>>((const float *)x, desc_of(in0), (uint32_t *)y, desc_of(tensor));
    timing_end(context, tensor->pipeline, s);
    return launch_status("k_arg_max");
}

extern "C" vkllm_err_t vkllm_op_arg_max_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
// Launchers for the fused prefill step (engine/engine.cu): the same kernels as the RMSNORM, BIN and
// ARG_MAX nodes on dense row-major operands, without tensor structs.
namespace vkb
{

bool launch_rmsnorm_rows(const __half *x, const float *g, __half *y, uint32_t rows, uint32_t W, float eps,
                         cudaStream_t s)
{
    if (W % 8 != 0 || W / 8 > 1024 || ((uintptr_t)x & 15) || ((uintptr_t)y & 15) || ((uintptr_t)g & 15))
        return false;
    Desc4 d{{1, 1, rows, W}, {0, 0, W, 1}};
    const unsigned threads = ((W / 8 + 31) / 32) * 32;
    k_rmsnorm_vec<<<rows, threads < 32 ? 32 : threads, 0, s>>>(x, d, g, y, d, eps);
    return true;
}

bool launch_residual_rmsnorm_rows(__half *x, const __half *y, const float *g, __half *n, uint32_t rows, uint32_t W,
                                  float eps, cudaStream_t s)
{
    if (W % 8 != 0 || W / 8 > 1024 || (((uintptr_t)x | (uintptr_t)y | (uintptr_t)n | (uintptr_t)g) & 15))
        return false;
    const unsigned threads = ((W / 8 + 31) / 32) * 32;
    k_residual_rmsnorm_vec<<<rows, threads < 32 ? 32 : threads, 0, s>>>(x, y, g, n, W, eps);
    return true;
}

bool launch_bin_h(const __half *a, const __half *b, __half *out, uint64_t n, int op, cudaStream_t s)
{
    if (n % 8 != 0 || (((uintptr_t)a | (uintptr_t)b | (uintptr_t)out) & 15))
        return false;
    const uint64_t n8 = n / 8;
    uint64_t grid = (n8 + 255) / 256;
    if (grid > 148ull * 16)
        grid = 148ull * 16;
    k_bin_h8<__half><<<(unsigned)grid, 256, 0, s>>>(a, b, out, n8, op);
    return true;
}

bool launch_argmax_rows(const __half *x, uint32_t rows, uint32_t W, uint32_t *out, cudaStream_t s)
{
    Desc4 di{{1, 1, rows, W}, {0, 0, W, 1}};
    Desc4 dout{{1, 1, rows, 1}, {0, 0, 1, 1}};
    k_arg_max_block<__half><<<rows, 1024, 0, s>>>(x, di, out, dout);
    return true;
}

} // namespace vkb
