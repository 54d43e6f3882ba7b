// TEST INFRASTRUCTURE ONLY - the parity oracle for vkllm-b200.
//
// A CPU restatement of the reference vkllm.c LLaMA-2 path (ComingToy/vkllm.c): every operator
// follows the math, accumulation structure and fp16 rounding points of the reference's GLSL
// compute shaders (src/shaders/*.comp) in their "f16f32" variants (fp16 storage, fp32 arithmetic;
// the variants a device without shaderFloat16 selects), and the model step follows the reference
// graph (src/models/vkllm_models_llama2.c:488-602, src/models/vkllm_llama2_layers.c:13-340,
// src/models/vkllm_kvcache.c:65-102). Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline may load this library; the product never does.
//
// Parity pins: the reference ships no golden vectors. The per-op formulas are pinned to the CPU
// references inside the reference's own tests (tests/vkllm_test_op_*.c), compiled from its checkout
// by oracle/refpin/Makefile; tests/golden/ref_ops.npz holds their outputs and tests/test_oracle.py
// checks this restatement against them. The reference's GPU path cannot run here (Vulkan, VMA,
// gguf-tools and Bazel are absent), so end-to-end token parity is pinned to this restatement.
//
// Two arithmetic modes (oracle_set_arith): 0 = the f16f32 variants above (the default, and the parity
// target); 1 = the variants a device with shaderFloat16 selects (src/core/vkllm_gpu_device.c:232,
// src/core/vkllm_op_matmul.c:92-102, vkllm_op_softmax.c:22-33, vkllm_op_rope.c:20-30): the GEMV
// accumulates in fp16 (vkllm_mat_mul_vec.comp f16f16), the GEMM forms each dot(f16vec2) in fp16
// (vkllm_matmul_t*.comp f16f16f16), and softmax and RoPE compute in fp16 (LOAD_DTYPE float16_t).
// Each fp16 operation is modelled as the fp32 operation rounded to fp16 (exact for products and
// sums of two fp16 values up to a rare double rounding); the GPU's own fp16 exp/sin/cos/pow are
// modelled as the fp32 libm result rounded to fp16. BIN and ARG_MAX give the same results in both
// modes on fp16 data, RMSNORM is fp32 in both.
//
// fp16 <-> fp32 conversions use round-to-nearest-even (GPU conversion semantics). Transcendentals
// (expf, powf, sinf, cosf, 1/sqrtf) come from the host libm in fp32.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include <immintrin.h>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace
{

// ------------------------------------------------------------------------------------------------
// fp16 helpers
float g_h2f[65536];
struct H2FInit
{
    H2FInit()
    {
        for (uint32_t h = 0; h < 65536; ++h)
        {
            uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, man = h & 0x3ff, f;
            if (exp == 0)
            {
                if (man == 0)
                    f = sign << 31;
                else
                {
                    int e = -1;
                    do
                    {
                        e++;
                        man <<= 1;
                    } while (!(man & 0x400));
                    f = (sign << 31) | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
                }
            }
            else if (exp == 31)
                f = (sign << 31) | 0x7f800000u | (man << 13);
            else
                f = (sign << 31) | ((exp - 15 + 127) << 23) | (man << 13);
            memcpy(&g_h2f[h], &f, 4);
        }
    }
} g_h2f_init;

inline float h2f(uint16_t h)
{
    return g_h2f[h];
}

inline uint16_t f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, mant = x & 0x7fffffu;
    int exp = (int)((x >> 23) & 0xff);
    if (exp == 255)
        return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    int e = exp - 127 + 15;
    if (e >= 31)
        return (uint16_t)(sign | 0x7c00u);
    if (e <= 0)
    {
        if (e < -10)
            return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u)))
            hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
        h++;
    return (uint16_t)h;
}

// One fp16 rounding of an fp32 value (the value of f2h followed by h2f): the F16C conversion, which
// is IEEE round-to-nearest-even with fp16 subnormals and overflow to infinity, part of the x86-64-v3
// baseline this library is built for. round16x8 rounds eight lanes the same way.
inline float round16(float f)
{
    return _cvtsh_ss(_cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT));
}

inline __m256 round16x8(__m256 v)
{
    return _mm256_cvtph_ps(_mm256_cvtps_ph(v, _MM_FROUND_TO_NEAREST_INT));
}

int g_arith16 = 0; // 1: the shaderFloat16 variants (oracle_set_arith)

// ------------------------------------------------------------------------------------------------
// Strided views: dtype 1 = f32, 2 = f16, 4 = u32 (vkllm_dtype_t values); element strides.
struct View
{
    int dtype;
    uint32_t shape[4];
    uint32_t stride[4];
    void *data;
    uint64_t off(uint32_t b, uint32_t c, uint32_t h, uint32_t w) const
    {
        return (uint64_t)b * stride[0] + (uint64_t)c * stride[1] + (uint64_t)h * stride[2] + (uint64_t)w * stride[3];
    }
    float get(uint64_t o) const
    {
        return dtype == 2 ? h2f(((const uint16_t *)data)[o]) : ((const float *)data)[o];
    }
    void set(uint64_t o, float v) const
    {
        if (dtype == 2)
            ((uint16_t *)data)[o] = f2h(v);
        else
            ((float *)data)[o] = v;
    }
};

View mkview(int dtype, const uint32_t *shape, const uint32_t *stride, const void *data)
{
    View v;
    v.dtype = dtype;
    memcpy(v.shape, shape, 16);
    memcpy(v.stride, stride, 16);
    v.data = const_cast<void *>(data);
    return v;
}

View contiguous(int dtype, uint32_t b, uint32_t c, uint32_t h, uint32_t w, void *data)
{
    View v;
    v.dtype = dtype;
    v.shape[0] = b, v.shape[1] = c, v.shape[2] = h, v.shape[3] = w;
    v.stride[3] = 1, v.stride[2] = w, v.stride[1] = h * w, v.stride[0] = c * h * w;
    v.data = data;
    return v;
}

// 32-lane subgroup reduction as a butterfly (offsets 16, 8, 4, 2, 1); lane 0's value is returned.
float subgroup_add(float *lanes)
{
    float t[32];
    memcpy(t, lanes, sizeof(t));
    for (int o = 16; o > 0; o >>= 1)
        for (int l = 0; l < o; ++l)
            t[l] = t[l] + t[l + o];
    return t[0];
}

float subgroup_max(float *lanes)
{
    float t[32];
    memcpy(t, lanes, sizeof(t));
    for (int o = 16; o > 0; o >>= 1)
        for (int l = 0; l < o; ++l)
            t[l] = std::max(t[l], t[l + o]);
    return t[0];
}

float silu(float v)
{
    return v / (1.0f + expf(-v));
}

bool is_transposed_b(const View &a, const View &b, const View &c)
{
    // src/core/vkllm_op_matmul.c:14-24
    uint32_t M = c.shape[2], N = c.shape[3], K = a.shape[3];
    return a.shape[2] == M && b.shape[2] == N && a.shape[3] == K && b.shape[3] == K;
}

// GEMV (src/shaders/vkllm_mat_mul_vec.comp:94-150, f16f32 variant): lane l accumulates
// fp32 dot(vec4) partials over i = 4l + 128j; subgroupAdd; * scale; SiLU; store. Batch offsets use
// the channel index only (the GEMV pipelines are unspecialised, AXIS0); a size-1 channel is reused.
void gemv(const View &a, const View &w, const View &out, float scale, int act)
{
    uint64_t n = (uint64_t)out.shape[0] * out.shape[1] * out.shape[2] * out.shape[3];
    uint32_t K = a.shape[3];
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)n; ++idx)
    {
        uint64_t t = (uint64_t)idx;
        uint32_t col = t % out.shape[3];
        t /= out.shape[3];
        uint32_t h = t % out.shape[2];
        t /= out.shape[2];
        uint32_t c = t % out.shape[1];
        uint32_t b = (uint32_t)(t / out.shape[1]);
        uint64_t ao = (uint64_t)(a.shape[1] == 1 ? 0 : c) * a.stride[1] + (uint64_t)h * a.stride[2];
        uint64_t wo = (uint64_t)(w.shape[1] == 1 ? 0 : c) * w.stride[1] + (uint64_t)col * w.stride[2];
        float lanes[32];
        for (int l = 0; l < 32; ++l)
        {
            float acc = 0.f;
            for (uint32_t i = 4 * l; i < K; i += 128)
            {
                float d = 0.f;
                for (uint32_t q = 0; q < 4; ++q)
                {
                    // The reference reads 4 elements unconditionally (K % 4 == 0 in every config);
                    // elements past K count as 0 here.
                    if (i + q < K)
                        d += a.get(ao + (uint64_t)(i + q) * a.stride[3]) * w.get(wo + (uint64_t)(i + q) * w.stride[3]);
                }
                // f16f16: acc = ACC_DTYPE(dot(vec4, vec4)) + acc, both in fp16
                acc = g_arith16 ? round16(round16(d) + acc) : d + acc;
            }
            lanes[l] = acc;
        }
        float v;
        if (g_arith16)
        {
            for (int o = 16; o > 0; o >>= 1) // subgroupAdd in fp16
                for (int l = 0; l < o; ++l)
                    lanes[l] = round16(lanes[l] + lanes[l + o]);
            v = round16(lanes[0] * round16(scale));
            if (act == 1)
                v = round16(v / round16(1.0f + round16(expf(-v))));
        }
        else
        {
            v = subgroup_add(lanes) * scale;
            if (act == 1)
                v = silu(v);
        }
        out.set(out.off(b, c, h, col), v);
    }
}

// GEMM (src/shaders/vkllm_matmul_t1.comp:90-251 for B [N,K], vkllm_matmul_t0.comp:92-245 for B [K,N]):
// fp32 sum over K in order of pairwise fp32 dot(vec2) terms; * scale; SiLU; store. Broadcast: a
// size-1 batch/channel axis is reused (src/core/vkllm_op_matmul.c:65-91).
//
// Every output element is acc_{k+2} = acc_k + (a_k b_k + a_{k+1} b_{k+1}) over k = 0, 2, 4, ..., with
// an odd K padded by a zero pair. The loops below compute 8-32 columns of a row at once (a panel of
// B converted to fp32 and laid out k-major per block of columns), which the compiler vectorises
// across columns; each column still sees exactly that sequence of operations.
constexpr uint32_t kGemmNB = 32; // columns per panel (a multiple of the 8 lanes of round16x8)
static_assert(kGemmNB % 8 == 0, "panel width");
constexpr uint32_t kGemmMB = 4;  // rows per register block

void gemm(const View &a, const View &bm, const View &out, bool trans_b, float scale, int act)
{
    const uint32_t M = out.shape[2], N = out.shape[3], K = a.shape[3], Kp = K + (K & 1u);
    const uint32_t nb = (N + kGemmNB - 1) / kGemmNB, batches = out.shape[0] * out.shape[1];
    // A rows in fp32, zero-padded to Kp, for every batch.
    std::vector<float> af((size_t)batches * M * Kp, 0.f);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)batches * M; ++idx)
    {
        uint32_t m = (uint32_t)(idx % M), z = (uint32_t)(idx / M);
        uint32_t c = z % out.shape[1], b = z / out.shape[1];
        uint64_t ao = (uint64_t)(a.shape[0] == 1 ? 0 : b) * a.stride[0] + (uint64_t)(a.shape[1] == 1 ? 0 : c) * a.stride[1] +
                      (uint64_t)m * a.stride[2];
        float *dst = &af[(size_t)idx * Kp];
        for (uint32_t k = 0; k < K; ++k)
            dst[k] = a.get(ao + (uint64_t)k * a.stride[3]);
    }
#pragma omp parallel
    {
        std::vector<float> panel((size_t)Kp * kGemmNB);
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < (int64_t)batches * nb; ++t)
        {
            const uint32_t z = (uint32_t)(t / nb), n0 = (uint32_t)(t % nb) * kGemmNB;
            const uint32_t c = z % out.shape[1], b = z / out.shape[1];
            const uint32_t nn = std::min(kGemmNB, N - n0);
            const uint64_t bo = (uint64_t)(bm.shape[0] == 1 ? 0 : b) * bm.stride[0] +
                                (uint64_t)(bm.shape[1] == 1 ? 0 : c) * bm.stride[1];
            for (uint32_t k = 0; k < Kp; ++k)
                for (uint32_t j = 0; j < kGemmNB; ++j)
                {
                    float v = 0.f;
                    if (k < K && j < nn)
                        v = trans_b ? bm.get(bo + (uint64_t)(n0 + j) * bm.stride[2] + (uint64_t)k * bm.stride[3])
                                    : bm.get(bo + (uint64_t)k * bm.stride[2] + (uint64_t)(n0 + j) * bm.stride[3]);
                    panel[(size_t)k * kGemmNB + j] = v;
                }
            const float *A = &af[(size_t)z * M * Kp];
            for (uint32_t m0 = 0; m0 < M; m0 += kGemmMB)
            {
                const uint32_t mm = std::min(kGemmMB, M - m0);
                float acc[kGemmMB][kGemmNB] = {};
                for (uint32_t k = 0; k < Kp; k += 2)
                {
                    const float *b0 = &panel[(size_t)k * kGemmNB], *b1 = b0 + kGemmNB;
                    for (uint32_t r = 0; r < kGemmMB; ++r)
                    {
                        const float a0 = r < mm ? A[(size_t)(m0 + r) * Kp + k] : 0.f;
                        const float a1 = r < mm ? A[(size_t)(m0 + r) * Kp + k + 1] : 0.f;
                        if (g_arith16) // f16f16f16: float(dot(f16vec2, f16vec2)), the dot in fp16
                            for (uint32_t j = 0; j < kGemmNB; j += 8)
                            {
                                const __m256 p0 = round16x8(_mm256_mul_ps(_mm256_set1_ps(a0), _mm256_loadu_ps(b0 + j)));
                                const __m256 p1 = round16x8(_mm256_mul_ps(_mm256_set1_ps(a1), _mm256_loadu_ps(b1 + j)));
                                _mm256_storeu_ps(&acc[r][j], _mm256_add_ps(_mm256_loadu_ps(&acc[r][j]),
                                                                           round16x8(_mm256_add_ps(p0, p1))));
                            }
                        else
                            for (uint32_t j = 0; j < kGemmNB; ++j)
                                acc[r][j] += a0 * b0[j] + a1 * b1[j];
                    }
                }
                for (uint32_t r = 0; r < mm; ++r)
                    for (uint32_t j = 0; j < nn; ++j)
                    {
                        float v = acc[r][j] * scale;
                        if (act == 1)
                            v = silu(v);
                        out.set(out.off(b, c, m0 + r, n0 + j), v);
                    }
            }
        }
    }
}

void matmul(const View &a, const View &b, const View &out, float scale, int act)
{
    bool tb = is_transposed_b(a, b, out);
    if (a.shape[2] == 1 && tb) // src/core/vkllm_op_matmul.c:26-30
        gemv(a, b, out, scale, act);
    else
        gemm(a, b, out, tb, scale, act);
}

// RMSNORM (src/shaders/vkllm_rmsnorm.comp:31-82): 512 thread-strided partial sums of squares, a
// halving tree, alpha = inversesqrt(sum / W + eps), y = fp16((x * g) * alpha).
void rmsnorm(const View &x, const float *g, const View &y, float eps)
{
    uint32_t rows = x.shape[0] * x.shape[1] * x.shape[2], W = x.shape[3];
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r)
    {
        uint32_t h = r % x.shape[2], c = (r / x.shape[2]) % x.shape[1], b = (uint32_t)(r / (x.shape[2] * x.shape[1]));
        uint64_t xo = x.off(b, c, h, 0), yo = y.off(b, c, h, 0);
        float part[512];
        for (uint32_t t = 0; t < 512; ++t)
        {
            float s = 0.f;
            for (uint32_t i = t; i < W; i += 512)
            {
                float v = x.get(xo + i);
                s += v * v;
            }
            part[t] = s;
        }
        for (uint32_t o = 256; o > 0; o >>= 1)
            for (uint32_t t = 0; t < o; ++t)
                part[t] += part[t + o];
        float mean = part[0] / (float)W;
        float alpha = 1.0f / sqrtf(mean + eps);
        for (uint32_t i = 0; i < W; ++i)
            y.set(yo + i, (x.get(xo + i) * g[i]) * alpha);
    }
}

// ROPE (src/shaders/vkllm_rope.comp:39-79), normal or neox pairing.
void rope(const View &in, const View &out, uint32_t offset, float base, int neox)
{
    uint32_t hw = in.shape[3] / 2;
    for (uint32_t b = 0; b < in.shape[0]; ++b)
        for (uint32_t c = 0; c < in.shape[1]; ++c)
            for (uint32_t h = 0; h < in.shape[2]; ++h)
                for (uint32_t w = 0; w < hw; ++w)
                {
                    uint64_t i0, i1, o0, o1;
                    if (neox)
                    {
                        i0 = in.off(b, c, h, w);
                        i1 = i0 + (uint64_t)in.stride[3] * hw;
                        o0 = out.off(b, c, h, w);
                        o1 = o0 + (uint64_t)out.stride[3] * (out.shape[3] / 2);
                    }
                    else
                    {
                        i0 = in.off(b, c, h, 2 * w);
                        i1 = i0 + in.stride[3];
                        o0 = out.off(b, c, h, 2 * w);
                        o1 = o0 + out.stride[3];
                    }
                    float v0 = in.get(i0), v1 = in.get(i1);
                    if (g_arith16) // LOAD_DTYPE float16_t: every value and operation in fp16
                    {
                        float e = round16(round16((float)(2 * w)) / round16((float)in.shape[3]));
                        float f = round16(round16((float)(offset + h)) / round16(powf(round16(base), e)));
                        float cs = round16(cosf(f)), sn = round16(sinf(f));
                        out.set(o0, round16(cs * v0) - round16(sn * v1));
                        out.set(o1, round16(sn * v0) + round16(cs * v1));
                        continue;
                    }
                    float f = (float)(offset + h) / powf(base, (float)(2 * w) / (float)in.shape[3]);
                    float cs = cosf(f), sn = sinf(f);
                    out.set(o0, cs * v0 - sn * v1);
                    out.set(o1, sn * v0 + cs * v1);
                }
}

// SOFTMAX (src/shaders/vkllm_softmax.comp:42-96): lane max (seeded with element 0) over ALL
// entries, subgroupMax; lane sums of exp(x - max) over unmasked entries, subgroupAdd; masked -> 0.
// The input is addressed with the output layout.
void softmax(const View &in_as_out, const View &out, int seq_mask, uint32_t offsets)
{
    uint32_t W = out.shape[3];
    for (uint32_t b = 0; b < out.shape[0]; ++b)
        for (uint32_t c = 0; c < out.shape[1]; ++c)
            for (uint32_t h = 0; h < out.shape[2]; ++h)
            {
                uint64_t base = out.off(b, c, h, 0);
                float lm[32], ls[32];
                for (uint32_t l = 0; l < 32; ++l)
                {
                    float m = in_as_out.get(base);
                    for (uint32_t i = l; i < W; i += 32)
                        m = std::max(m, in_as_out.get(base + (uint64_t)i * out.stride[3]));
                    lm[l] = m;
                }
                float gm = subgroup_max(lm);
                // f16f16 (LOAD_DTYPE float16_t): differences, exponentials, sums and quotients in fp16
                auto ex = [&](float x) { return g_arith16 ? round16(expf(round16(x - gm))) : expf(x - gm); };
                for (uint32_t l = 0; l < 32; ++l)
                {
                    float s = 0.f;
                    for (uint32_t i = l; i < W; i += 32)
                    {
                        if (seq_mask > 0 && i > h + offsets)
                            continue;
                        s = g_arith16 ? round16(s + ex(in_as_out.get(base + (uint64_t)i * out.stride[3])))
                                      : s + ex(in_as_out.get(base + (uint64_t)i * out.stride[3]));
                    }
                    ls[l] = s;
                }
                float gs;
                if (g_arith16)
                {
                    for (int o = 16; o > 0; o >>= 1)
                        for (int l = 0; l < o; ++l)
                            ls[l] = round16(ls[l] + ls[l + o]);
                    gs = ls[0];
                }
                else
                    gs = subgroup_add(ls);
                for (uint32_t i = 0; i < W; ++i)
                {
                    uint64_t o = base + (uint64_t)i * out.stride[3];
                    if (seq_mask > 0 && i > h + offsets)
                        out.set(o, 0.f);
                    else
                        out.set(o, ex(in_as_out.get(o)) / gs);
                }
            }
}

// ARG_MAX (src/shaders/vkllm_arg_max.comp:40-97): lane l scans i = l, l+32, ... keeping its first
// strict maximum (lanes >= W start at -FLT_MAX with their own index); tree 16..1 keeps the left
// operand unless the right is strictly greater.
void arg_max(const View &in, uint32_t *out, const uint32_t *out_stride)
{
    uint32_t W = in.shape[3];
    for (uint32_t b = 0; b < in.shape[0]; ++b)
        for (uint32_t c = 0; c < in.shape[1]; ++c)
            for (uint32_t h = 0; h < in.shape[2]; ++h)
            {
                uint64_t base = in.off(b, c, h, 0);
                float v[32];
                uint32_t ix[32];
                for (uint32_t l = 0; l < 32; ++l)
                {
                    v[l] = -FLT_MAX;
                    ix[l] = l;
                    if (l < W)
                        v[l] = in.get(base + (uint64_t)l * in.stride[3]);
                    for (uint32_t i = l + 32; i < W; i += 32)
                    {
                        float x = in.get(base + (uint64_t)i * in.stride[3]);
                        if (x > v[l])
                        {
                            v[l] = x;
                            ix[l] = i;
                        }
                    }
                }
                for (int o = 16; o > 0; o >>= 1)
                    for (int l = 0; l < o; ++l)
                        if (v[l + o] > v[l])
                        {
                            v[l] = v[l + o];
                            ix[l] = ix[l + o];
                        }
                out[(uint64_t)b * out_stride[0] + (uint64_t)c * out_stride[1] + (uint64_t)h * out_stride[2]] = ix[0];
            }
}

// ------------------------------------------------------------------------------------------------
// Counter-based random weights (same definition as the library's device generator, restated
// here so the oracle can build a 7B-shaped model on its own).
uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ------------------------------------------------------------------------------------------------
struct Layer
{
    const float *attn_norm, *ffn_norm;
    const uint16_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
};

struct Model
{
    uint32_t D, H, hd, F, V, L, ctx, unk;
    float eps, base;
    const uint16_t *embed, *wout;
    const float *out_norm;
    std::vector<Layer> layers;
    std::vector<std::vector<uint16_t>> kc, vc; // [H, ctx, hd] per layer
};

} // namespace

extern "C" {

struct oracle_view
{
    int dtype;
    uint32_t shape[4];
    uint32_t stride[4];
    void *data;
};

static View from(const oracle_view *v)
{
    return mkview(v->dtype, v->shape, v->stride, v->data);
}

// 0: f16f32 arithmetic (fp32 math, the default); 1: the shaderFloat16 variants. Returns the previous mode.
int oracle_set_arith(int mode)
{
    int old = g_arith16;
    g_arith16 = mode ? 1 : 0;
    return old;
}

int oracle_threads(int n)
{
#ifdef _OPENMP
    if (n > 0)
        omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

void oracle_f32_to_f16(const float *in, uint16_t *out, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i)
        out[i] = f2h(in[i]);
}

// round16 over an array (lets a test compare the F16C rounding with f2h/h2f and with numpy).
void oracle_round16(const float *in, float *out, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i)
        out[i] = round16(in[i]);
}

void oracle_f16_to_f32(const uint16_t *in, float *out, uint64_t n)
{
    for (uint64_t i = 0; i < n; ++i)
        out[i] = h2f(in[i]);
}

int oracle_op_matmul(const oracle_view *a, const oracle_view *b, const oracle_view *c, float scale, int act)
{
    matmul(from(a), from(b), from(c), scale, act);
    return 0;
}

int oracle_op_rmsnorm(const oracle_view *x, const float *g, const oracle_view *y, float eps)
{
    rmsnorm(from(x), g, from(y), eps);
    return 0;
}

int oracle_op_rope(const oracle_view *in, const oracle_view *out, uint32_t offset, float base, int neox)
{
    rope(from(in), from(out), offset, base, neox);
    return 0;
}

int oracle_op_softmax(const oracle_view *in, const oracle_view *out, int seq_mask, uint32_t offsets)
{
    View i = from(in), o = from(out);
    View io = o;
    io.data = i.data;
    io.dtype = i.dtype;
    softmax(io, o, seq_mask, offsets);
    return 0;
}

// UPDATE_ROWS (src/shaders/vkllm_update_rows.comp:21-46) / COPY (src/shaders/vkllm_copy.comp:35-50):
// element copies; `elem_bytes` 2 or 4.
int oracle_op_update_rows(const oracle_view *in, const oracle_view *out, uint32_t offset_rows, int elem_bytes)
{
    View i = from(in), o = from(out);
    for (uint32_t b = 0; b < i.shape[0]; ++b)
        for (uint32_t c = 0; c < i.shape[1]; ++c)
            for (uint32_t h = 0; h < i.shape[2]; ++h)
                for (uint32_t w = 0; w < i.shape[3]; ++w)
                {
                    if (h + offset_rows >= o.shape[2])
                        continue;
                    uint64_t si = i.off(b, c, h, w), so = o.off(b, c, h + offset_rows, w);
                    memcpy((char *)o.data + so * elem_bytes, (const char *)i.data + si * elem_bytes, elem_bytes);
                }
    return 0;
}

int oracle_op_copy(const oracle_view *in, const oracle_view *out, int elem_bytes)
{
    return oracle_op_update_rows(in, out, 0, elem_bytes);
}

// BIN (src/shaders/vkllm_bin_op.comp:41-73): fp32 op, all operands at the output layout's offsets.
int oracle_op_bin(const oracle_view *a, const oracle_view *b, const oracle_view *out, int op)
{
    View x = from(a), y = from(b), o = from(out);
    for (uint32_t i0 = 0; i0 < o.shape[0]; ++i0)
        for (uint32_t i1 = 0; i1 < o.shape[1]; ++i1)
            for (uint32_t i2 = 0; i2 < o.shape[2]; ++i2)
                for (uint32_t i3 = 0; i3 < o.shape[3]; ++i3)
                {
                    uint64_t off = o.off(i0, i1, i2, i3);
                    float u = x.get(off), v = y.get(off);
                    float r = op == 0 ? u + v : (op == 1 ? u - v : (op == 2 ? u * v : u / v));
                    o.set(off, r);
                }
    return 0;
}

// EMBEDDING (src/shaders/vkllm_embedding.comp:41-70): id >= rows -> unk; output addressed
// c*s0 + h*s1 + w*s2 (the shader's shifted indexing).
int oracle_op_embedding(const oracle_view *ids, const oracle_view *table, const oracle_view *out, uint32_t unk,
                        int elem_bytes)
{
    View i = from(ids), t = from(table), o = from(out);
    for (uint32_t b = 0; b < i.shape[0]; ++b)
        for (uint32_t c = 0; c < i.shape[1]; ++c)
            for (uint32_t h = 0; h < i.shape[2]; ++h)
                for (uint32_t w = 0; w < i.shape[3]; ++w)
                {
                    uint32_t tok = ((const uint32_t *)i.data)[i.off(b, c, h, w)];
                    if (tok >= t.shape[2])
                        tok = unk;
                    uint64_t oo = (uint64_t)c * o.stride[0] + (uint64_t)h * o.stride[1] + (uint64_t)w * o.stride[2];
                    memcpy((char *)o.data + oo * elem_bytes, (const char *)t.data + (uint64_t)tok * t.stride[2] * elem_bytes,
                           (size_t)t.shape[3] * elem_bytes);
                }
    return 0;
}

int oracle_op_arg_max(const oracle_view *in, uint32_t *out, const uint32_t *out_stride)
{
    arg_max(from(in), out, out_stride);
    return 0;
}

// FFN_UP_AND_GATE intended math (src/shaders/vkllm_ffn_up_and_gate.comp:137-146):
// y = u * g / (1 + exp(-g)), u = x.Wu^T, g = x.Wg^T, fp32 sums over K in order.
int oracle_op_ffn_up_gate(const oracle_view *x, const oracle_view *wu, const oracle_view *wg, const oracle_view *out)
{
    View xv = from(x), u = from(wu), g = from(wg), o = from(out);
    for (uint32_t b = 0; b < o.shape[0]; ++b)
        for (uint32_t c = 0; c < o.shape[1]; ++c)
            for (uint32_t m = 0; m < o.shape[2]; ++m)
                for (uint32_t n = 0; n < o.shape[3]; ++n)
                {
                    float su = 0.f, sg = 0.f;
                    for (uint32_t k = 0; k < xv.shape[3]; ++k)
                    {
                        float a = xv.get(xv.off(b, c, m, k));
                        su += a * u.get((uint64_t)n * u.stride[2] + (uint64_t)k * u.stride[3]);
                        sg += a * g.get((uint64_t)n * g.stride[2] + (uint64_t)k * g.stride[3]);
                    }
                    o.set(o.off(b, c, m, n), su * sg / (1.0f + expf(-sg)));
                }
    return 0;
}

void oracle_random_f16(uint64_t seed, uint64_t tensor_id, float std_dev, uint64_t first, uint64_t n, uint16_t *out)
{
    uint64_t key = splitmix64(seed ^ splitmix64(tensor_id + 0x5851F42D4C957F2Dull));
    float scale = std_dev * (1.0f / 65536.0f);
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii)
    {
        uint64_t i = first + (uint64_t)ii;
        int64_t s = 0;
        for (int j = 0; j < 3; ++j)
        {
            uint64_t h = splitmix64(key + 3 * i + (uint64_t)j);
            s += (int64_t)(h & 0xffff) + (int64_t)((h >> 16) & 0xffff) + (int64_t)((h >> 32) & 0xffff) +
                 (int64_t)(h >> 48);
        }
        out[ii] = f2h((float)(int32_t)(s - 393210) * scale);
    }
}

struct oracle_llama2_cfg
{
    uint32_t D, H, F, V, L, ctx, unk;
    float eps, rope_base;
};

// layer_ptrs: 9 per layer in the order attn_norm (f32), ffn_norm (f32), q, k, v, o, gate, up, down (fp16).
void *oracle_llama2_new(const oracle_llama2_cfg *cfg, const uint16_t *embed, const float *out_norm,
                        const uint16_t *wout, const void *const *layer_ptrs)
{
    Model *m = new Model();
    m->D = cfg->D, m->H = cfg->H, m->hd = cfg->D / cfg->H, m->F = cfg->F, m->V = cfg->V, m->L = cfg->L;
    m->ctx = cfg->ctx, m->unk = cfg->unk, m->eps = cfg->eps, m->base = cfg->rope_base;
    m->embed = embed, m->out_norm = out_norm, m->wout = wout;
    for (uint32_t l = 0; l < m->L; ++l)
    {
        const void *const *p = layer_ptrs + 9 * l;
        Layer ly = {(const float *)p[0],    (const float *)p[1],    (const uint16_t *)p[2],
                    (const uint16_t *)p[3], (const uint16_t *)p[4], (const uint16_t *)p[5],
                    (const uint16_t *)p[6], (const uint16_t *)p[7], (const uint16_t *)p[8]};
        m->layers.push_back(ly);
        m->kc.emplace_back((size_t)m->H * m->ctx * m->hd, 0);
        m->vc.emplace_back((size_t)m->H * m->ctx * m->hd, 0);
    }
    return m;
}

void oracle_llama2_free(void *p)
{
    delete (Model *)p;
}

// One reference graph run for S tokens at position `offset` (src/models/vkllm_models_llama2.c:488-602).
// logits_out: fp16 [S, V] (or NULL); tokens_out: argmax per row [S].
int oracle_llama2_step(void *p, const uint32_t *toks, uint32_t S, uint32_t offset, uint16_t *logits_out,
                       uint32_t *tokens_out)
{
    Model *m = (Model *)p;
    if (offset + S > m->ctx)
        return -1;
    const uint32_t D = m->D, H = m->H, hd = m->hd, F = m->F, V = m->V, HD = H * hd, Lk = offset + S;
    std::vector<uint16_t> x((size_t)S * D), n((size_t)S * D), Q((size_t)S * HD), K((size_t)S * HD),
        Vv((size_t)S * HD), RQ((size_t)S * HD), RK((size_t)S * HD), sc((size_t)H * S * Lk), pr((size_t)H * S * Lk),
        ao((size_t)H * S * hd), cat((size_t)S * HD), y((size_t)S * D), u((size_t)S * F), g((size_t)S * F),
        mm((size_t)S * F), dn((size_t)S * D), lg((size_t)S * V);
    // embedded = EMBEDDING(input_toks)
    for (uint32_t s = 0; s < S; ++s)
    {
        uint32_t t = toks[s] >= V ? m->unk : toks[s];
        memcpy(&x[(size_t)s * D], m->embed + (size_t)t * D, (size_t)D * 2);
    }
    View X = contiguous(2, 1, 1, S, D, x.data()), N = contiguous(2, 1, 1, S, D, n.data());
    for (uint32_t l = 0; l < m->L; ++l)
    {
        const Layer &ly = m->layers[l];
        rmsnorm(X, ly.attn_norm, N, m->eps);
        View WQ = contiguous(2, 1, 1, HD, D, (void *)ly.wq), WK = contiguous(2, 1, 1, HD, D, (void *)ly.wk),
             WV = contiguous(2, 1, 1, HD, D, (void *)ly.wv);
        View Qv = contiguous(2, 1, 1, S, HD, Q.data()), Kv = contiguous(2, 1, 1, S, HD, K.data()),
             VvV = contiguous(2, 1, 1, S, HD, Vv.data());
        matmul(N, WQ, Qv, 1.0f, 0);
        matmul(N, WK, Kv, 1.0f, 0);
        matmul(N, WV, VvV, 1.0f, 0);
        // views [1,S,H,hd] permuted to [1,H,S,hd]: strides (S*HD, hd, HD, 1)
        auto heads = [&](std::vector<uint16_t> &buf) {
            View v;
            v.dtype = 2;
            v.shape[0] = 1, v.shape[1] = H, v.shape[2] = S, v.shape[3] = hd;
            v.stride[0] = S * HD, v.stride[1] = hd, v.stride[2] = HD, v.stride[3] = 1;
            v.data = buf.data();
            return v;
        };
        View RQv = contiguous(2, 1, H, S, hd, RQ.data()), RKv = contiguous(2, 1, H, S, hd, RK.data());
        rope(heads(Q), RQv, offset, m->base, 0);
        rope(heads(K), RKv, offset, m->base, 0);
        // kvcache_update: cache[h][offset + s] = RK[h][s], V[s][h]
        for (uint32_t h = 0; h < H; ++h)
            for (uint32_t s = 0; s < S; ++s)
            {
                memcpy(&m->kc[l][((size_t)h * m->ctx + offset + s) * hd], &RK[((size_t)h * S + s) * hd], hd * 2);
                memcpy(&m->vc[l][((size_t)h * m->ctx + offset + s) * hd], &Vv[(size_t)s * HD + (size_t)h * hd], hd * 2);
            }
        View Ks, Vs;
        Ks.dtype = Vs.dtype = 2;
        Ks.shape[0] = 1, Ks.shape[1] = H, Ks.shape[2] = Lk, Ks.shape[3] = hd;
        Ks.stride[0] = H * m->ctx * hd, Ks.stride[1] = m->ctx * hd, Ks.stride[2] = hd, Ks.stride[3] = 1;
        Vs = Ks;
        Ks.data = m->kc[l].data();
        Vs.data = m->vc[l].data();
        View SC = contiguous(2, 1, H, S, Lk, sc.data()), PR = contiguous(2, 1, H, S, Lk, pr.data());
        matmul(RQv, Ks, SC, 1.0f / sqrtf((float)hd), 0);
        softmax(SC, PR, 1, offset);
        View AO = contiguous(2, 1, H, S, hd, ao.data());
        matmul(PR, Vs, AO, 1.0f, 0);
        // concated_heads = COPY(permute(attn)) -> [S, H*hd]
        for (uint32_t h = 0; h < H; ++h)
            for (uint32_t s = 0; s < S; ++s)
                memcpy(&cat[(size_t)s * HD + (size_t)h * hd], &ao[((size_t)h * S + s) * hd], hd * 2);
        View CAT = contiguous(2, 1, 1, S, HD, cat.data()), Y = contiguous(2, 1, 1, S, D, y.data());
        matmul(CAT, contiguous(2, 1, 1, D, HD, (void *)ly.wo), Y, 1.0f, 0);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] = f2h(h2f(x[i]) + h2f(y[i]));
        // FFN
        rmsnorm(X, ly.ffn_norm, N, m->eps);
        View U = contiguous(2, 1, 1, S, F, u.data()), G = contiguous(2, 1, 1, S, F, g.data());
        matmul(N, contiguous(2, 1, 1, F, D, (void *)ly.wu), U, 1.0f, 0);
        matmul(N, contiguous(2, 1, 1, F, D, (void *)ly.wg), G, 1.0f, 1);
        for (size_t i = 0; i < mm.size(); ++i)
            mm[i] = f2h(h2f(u[i]) * h2f(g[i]));
        View MM = contiguous(2, 1, 1, S, F, mm.data()), DN = contiguous(2, 1, 1, S, D, dn.data());
        matmul(MM, contiguous(2, 1, 1, D, F, (void *)ly.wd), DN, 1.0f, 0);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] = f2h(h2f(x[i]) + h2f(dn[i]));
    }
    rmsnorm(X, m->out_norm, N, m->eps);
    View LG = contiguous(2, 1, 1, S, V, lg.data());
    matmul(N, contiguous(2, 1, 1, V, D, (void *)m->wout), LG, 1.0f, 0);
    uint32_t ostride[4] = {S, S, 1, 1};
    arg_max(LG, tokens_out, ostride);
    if (logits_out)
        memcpy(logits_out, lg.data(), lg.size() * 2);
    return 0;
}

} // extern "C"
