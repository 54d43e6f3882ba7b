// Fused LLaMA-2 decode kernels (S = 1). One decode step is
//   embed -> L x [qkv, attn_scores, attn_pv, wo, upgate, down] -> logits(+argmax)
// with every kernel reading the step position/token from a device-resident StepState, so one
// captured CUDA Graph replays every step. Rounding points follow the reference graph
// (src/models/vkllm_llama2_layers.c:13-340): every node output is materialised as fp16, all
// arithmetic is fp32.
#pragma once

#include <cfloat>
#include <cstdint>

#include "../kernels/common.cuh"
#include "gemv_stream.cuh"

namespace vkb
{

struct StepState
{
    uint32_t token; // input token of the next step
    uint32_t pos;   // its position
    uint32_t step;  // steps taken since the last set_state
    uint32_t error; // non-zero: a kernel refused to run (position past the cache)
};

struct LayerW
{
    const __half *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *attn_norm, *ffn_norm;
    __half *kcache, *vcache; // [H, ctx, hd]
};

struct DecodeDims
{
    uint32_t D, H, hd, F, V, ctx, nsplit;
    float eps, rope_base, scale;
};

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kAttnThreads = 128;

__device__ __forceinline__ float block_sum(float v, float *red)
{
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0)
        red[w] = v;
    __syncthreads();
    if (w == 0)
    {
        float t = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
        t = warp_sum(t);
        if (l == 0)
            red[0] = t;
    }
    __syncthreads();
    float r = red[0];
    __syncthreads();
    return r;
}

// Stages the RMSNORM node's output fp16((x * g) * rsqrt(mean(x^2) + eps))
// (src/shaders/vkllm_rmsnorm.comp:48-81) into shared memory as fp32 times kHalfBitsScale (the
// streaming GEMV's activation format). K % 8 == 0.
__device__ __forceinline__ void stage_rmsnorm(const __half *__restrict__ x, const float *__restrict__ g, uint32_t K,
                                              float eps, float *xs, float *red)
{
    const uint32_t nchunk = K / 8;
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < nchunk; i += blockDim.x)
    {
        uint4 v = __ldcg(x4 + i); // L2: x may have been written by other CTAs of a persistent kernel
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            float2 f = __half22float2(h[j]);
            s = fmaf(f.x, f.x, s);
            s = fmaf(f.y, f.y, s);
        }
    }
    float tot = block_sum(s, red);
    float alpha = rsqrtf(tot / (float)K + eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    float4 *xs4 = reinterpret_cast<float4 *>(xs);
    for (uint32_t i = threadIdx.x; i < nchunk; i += blockDim.x)
    {
        uint4 v = __ldcg(x4 + i);
        float4 ga = g4[2 * i], gb = g4[2 * i + 1];
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        float o[8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            float2 f = __half22float2(h[j]);
            o[2 * j] = round_f16((f.x * gg[2 * j]) * alpha) * kHalfBitsScale;
            o[2 * j + 1] = round_f16((f.y * gg[2 * j + 1]) * alpha) * kHalfBitsScale;
        }
        xs4[2 * i] = make_float4(o[0], o[1], o[2], o[3]);
        xs4[2 * i + 1] = make_float4(o[4], o[5], o[6], o[7]);
    }
    __syncthreads();
}

// Stages an fp16 activation vector as fp32 times kHalfBitsScale.
__device__ __forceinline__ void stage_copy(const __half *__restrict__ x, uint32_t K, float *xs)
{
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    float4 *xs4 = reinterpret_cast<float4 *>(xs);
    for (uint32_t i = threadIdx.x; i < K / 8; i += blockDim.x)
    {
        uint4 v = __ldcg(x4 + i);
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]), d = __half22float2(h[3]);
        xs4[2 * i] = make_float4(a.x * kHalfBitsScale, a.y * kHalfBitsScale, b.x * kHalfBitsScale, b.y * kHalfBitsScale);
        xs4[2 * i + 1] =
            make_float4(c.x * kHalfBitsScale, c.y * kHalfBitsScale, d.x * kHalfBitsScale, d.y * kHalfBitsScale);
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------------------------
__global__ void k_dec_embed(const __half *__restrict__ table, uint32_t V, uint32_t D, uint32_t unk,
                            const StepState *__restrict__ st, __half *__restrict__ x)
{
    pdl_launch_dependents();
    pdl_wait();
    uint32_t tok = st->token;
    if (tok >= V)
        tok = unk; // src/shaders/vkllm_embedding.comp:57-60
    const uint4 *src = reinterpret_cast<const uint4 *>(table + (uint64_t)tok * D);
    uint4 *dst = reinterpret_cast<uint4 *>(x);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < D / 8; i += gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// Scores of one (head, key-split): s_j = fp16(scale * q.k_j) for keys j of this split (the scores
// node), written to `scores` [H, ctx]; plus the split's max m and sum l = sum_j exp(s_j - m).
__global__ void __launch_bounds__(kAttnThreads) k_dec_attn_scores(LayerW lw, DecodeDims dd,
                                                                  const __half *__restrict__ q,
                                                                  __half *__restrict__ scores, float2 *__restrict__ part,
                                                                  const StepState *__restrict__ st)
{
    __shared__ float qs[256];
    __shared__ float red[32];
    __shared__ float smax[kAttnThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t pos = st->pos;
    if (pos >= dd.ctx)
        return;
    const uint32_t h = blockIdx.x, split = blockIdx.y, Lk = pos + 1;
    const uint32_t chunk = (Lk + dd.nsplit - 1) / dd.nsplit;
    const uint32_t j0 = split * chunk, j1 = min(Lk, j0 + chunk);
    for (uint32_t d = threadIdx.x; d < dd.hd; d += blockDim.x)
        qs[d] = __half2float(q[h * dd.hd + d]);
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const __half *kb = lw.kcache + (uint64_t)h * dd.ctx * dd.hd;
    const uint32_t nq = dd.hd / 4; // lanes holding 4 halves each (hd % 4 == 0, hd <= 128 per pass)
    float wmax = -FLT_MAX;
    for (uint32_t j = j0 + warp; j < j1; j += nw)
    {
        const __half *kr = kb + (uint64_t)j * dd.hd;
        float a = 0.f;
        for (uint32_t c = lane; c < nq; c += 32)
        {
            uint2 raw = *reinterpret_cast<const uint2 *>(kr + 4 * c);
            const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
            float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
            a = fmaf(qs[4 * c], f0.x, a);
            a = fmaf(qs[4 * c + 1], f0.y, a);
            a = fmaf(qs[4 * c + 2], f1.x, a);
            a = fmaf(qs[4 * c + 3], f1.y, a);
        }
        a = warp_sum(a);
        float s = round_f16(a * dd.scale);
        if (lane == 0)
            scores[(uint64_t)h * dd.ctx + j] = __float2half_rn(s);
        wmax = fmaxf(wmax, s);
    }
    if (lane == 0)
        smax[warp] = wmax;
    __syncthreads();
    float m = -FLT_MAX;
    for (uint32_t w = 0; w < nw; ++w)
        m = fmaxf(m, smax[w]);
    __syncthreads(); // scores of this split are visible to the block
    float l = 0.f;
    for (uint32_t j = j0 + threadIdx.x; j < j1; j += blockDim.x)
        l += expf(__half2float(scores[(uint64_t)h * dd.ctx + j]) - m);
    l = block_sum(l, red);
    if (threadIdx.x == 0)
        part[h * dd.nsplit + split] = make_float2(j1 > j0 ? m : -FLT_MAX, j1 > j0 ? l : 0.f);
}

// probs . V of one (head, key-split): p_j = fp16(exp(s_j - M) / L) with M, L combined over all
// splits (the attn_weights node: max over all keys, src/shaders/vkllm_softmax.comp:54-85), partial
// o[d] = sum_j p_j v_j[d] in fp32. The last split to finish for a head sums the partials and
// stores fp16 attn[h*hd + d] (the attention-output node). When Lk == hd the reference's shape-only
// predicate reads V as [hd, Lk] (src/core/vkllm_op_matmul.c:14-30); that product
// o[w] = sum_k p_k V[w][k] is reproduced by split 0.
__global__ void __launch_bounds__(kAttnThreads) k_dec_attn_pv(LayerW lw, DecodeDims dd,
                                                              const __half *__restrict__ scores,
                                                              const float2 *__restrict__ part,
                                                              float *__restrict__ opart, uint32_t *__restrict__ counters,
                                                              __half *__restrict__ attn,
                                                              const StepState *__restrict__ st)
{
    __shared__ float acc_s[kAttnThreads / 32][256];
    __shared__ float ps[kAttnThreads];
    __shared__ uint32_t last;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t pos = st->pos;
    if (pos >= dd.ctx)
        return;
    const uint32_t h = blockIdx.x, split = blockIdx.y, Lk = pos + 1, hd = dd.hd;
    float M = -FLT_MAX;
    for (uint32_t c = 0; c < dd.nsplit; ++c)
        M = fmaxf(M, part[h * dd.nsplit + c].x);
    float L = 0.f;
    for (uint32_t c = 0; c < dd.nsplit; ++c)
    {
        float2 pl = part[h * dd.nsplit + c];
        if (pl.y > 0.f)
            L += pl.y * expf(pl.x - M);
    }
    const __half *sc = scores + (uint64_t)h * dd.ctx;
    const __half *vb = lw.vcache + (uint64_t)h * dd.ctx * hd;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float *op = opart + ((uint64_t)h * dd.nsplit + split) * hd;
    if (Lk == hd)
    {
        // Reference quirk: V slice read as the transposed operand.
        if (split == 0)
        {
            for (uint32_t w = threadIdx.x; w < hd; w += blockDim.x)
            {
                const __half *vr = vb + (uint64_t)w * hd;
                float o = 0.f;
                for (uint32_t k = 0; k < Lk; ++k)
                {
                    float p = round_f16(expf(__half2float(sc[k]) - M) / L);
                    o = fmaf(p, __half2float(vr[k]), o);
                }
                op[w] = o;
            }
        }
        else
            for (uint32_t w = threadIdx.x; w < hd; w += blockDim.x)
                op[w] = 0.f;
    }
    else
    {
        const uint32_t chunk = (Lk + dd.nsplit - 1) / dd.nsplit;
        const uint32_t j0 = split * chunk, j1 = min(Lk, j0 + chunk);
        const uint32_t nq = hd / 4;
        float a[4][4] = {}; // up to 4 column groups of 4 per lane (hd <= 512)
        for (uint32_t jb = j0; jb < j1; jb += blockDim.x)
        {
            uint32_t j = jb + threadIdx.x;
            ps[threadIdx.x] = j < j1 ? round_f16(expf(__half2float(sc[j]) - M) / L) : 0.f;
            __syncthreads();
            uint32_t jn = min((uint32_t)blockDim.x, j1 - jb);
            for (uint32_t t = warp; t < jn; t += nw)
            {
                float p = ps[t];
                const __half *vr = vb + (uint64_t)(jb + t) * hd;
#pragma unroll
                for (int g = 0; g < 4; ++g)
                {
                    uint32_t c = lane + 32 * g;
                    if (c < nq)
                    {
                        uint2 raw = *reinterpret_cast<const uint2 *>(vr + 4 * c);
                        const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
                        float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                        a[g][0] = fmaf(p, f0.x, a[g][0]);
                        a[g][1] = fmaf(p, f0.y, a[g][1]);
                        a[g][2] = fmaf(p, f1.x, a[g][2]);
                        a[g][3] = fmaf(p, f1.y, a[g][3]);
                    }
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int g = 0; g < 4; ++g)
        {
            uint32_t c = lane + 32 * g;
            if (c < nq && 4 * c + 3 < 256)
            {
                acc_s[warp][4 * c] = a[g][0];
                acc_s[warp][4 * c + 1] = a[g][1];
                acc_s[warp][4 * c + 2] = a[g][2];
                acc_s[warp][4 * c + 3] = a[g][3];
            }
        }
        __syncthreads();
        for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x)
        {
            float o = 0.f;
            for (uint32_t w = 0; w < nw; ++w)
                o += acc_s[w][d];
            op[d] = o;
        }
    }
    // Last split of this head combines the partials.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0)
        last = atomicAdd(&counters[h], 1u) == dd.nsplit - 1 ? 1u : 0u;
    __syncthreads();
    if (!last)
        return;
    __threadfence();
    const float *ob = opart + (uint64_t)h * dd.nsplit * hd;
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x)
    {
        float o = 0.f;
        for (uint32_t c = 0; c < dd.nsplit; ++c)
            o += __ldcg(ob + (uint64_t)c * hd + d);
        attn[h * hd + d] = __float2half_rn(o);
    }
    if (threadIdx.x == 0)
        counters[h] = 0;
}


// ------------------------------------------------------------------------------------------------
// Epilogue ops of the weight-streaming GEMV (gemv_stream.cuh), one per projection of the step.

// attn.norm + Q/K/V projections + RoPE on Q and K + KV-cache row write at `pos`. A unit is the row
// pair (2i, 2i+1) of the stacked [Wq; Wk; Wv], so each (even, odd) pair is rotated in registers:
// Q = fp16(acc), RQ = fp16(rot(Q)), as the Q -> ROPE nodes round (src/shaders/vkllm_rope.comp:68-78).
struct QkvOp
{
    static constexpr int NM = 2;
    LayerW lw;
    DecodeDims dd;
    const __half *x;
    __half *q_out;
    StepState *st;
    __device__ const __half *row_ptr(uint32_t u, uint32_t m) const
    {
        const uint32_t HD = dd.H * dd.hd, row = 2 * u + m, which = row / HD, r = row % HD;
        const __half *base = which == 0 ? lw.wq : (which == 1 ? lw.wk : lw.wv);
        return base + (uint64_t)r * dd.D;
    }
    __device__ void prologue(float *xs, float *red) const
    {
        stage_rmsnorm(x, lw.attn_norm, dd.D, dd.eps, xs, red);
    }
    __device__ void epilogue(uint32_t u, const float *s) const
    {
        const uint32_t pos = st->pos;
        if (pos >= dd.ctx)
        {
            st->error = 1;
            return;
        }
        const uint32_t HD = dd.H * dd.hd, row = 2 * u, which = row / HD, r = row % HD;
        float v0 = round_f16(s[0]), v1 = round_f16(s[1]);
        const uint32_t head = r / dd.hd, d = r % dd.hd;
        if (which < 2)
        {
            const uint32_t w = d / 2;
            const float theta = (float)pos / powf(dd.rope_base, (float)(2 * w) / (float)dd.hd);
            const float c = cosf(theta), sn = sinf(theta);
            const float o0 = c * v0 - sn * v1, o1 = sn * v0 + c * v1;
            v0 = o0;
            v1 = o1;
        }
        const __half2 hv = __floats2half2_rn(v0, v1);
        if (which == 0)
            *reinterpret_cast<__half2 *>(q_out + r) = hv;
        else
        {
            __half *cache = which == 1 ? lw.kcache : lw.vcache;
            *reinterpret_cast<__half2 *>(cache + ((uint64_t)head * dd.ctx + pos) * dd.hd + d) = hv;
        }
    }
    __device__ void finish() const
    {
    }
};

// Wo projection + residual: x = fp16(x + fp16(attn . Wo^T)) (final_output and final_output_add nodes).
struct WoOp
{
    static constexpr int NM = 1;
    LayerW lw;
    DecodeDims dd;
    const __half *attn;
    __half *x;
    float *part = nullptr; // tensor parallel: this rank's fp32 partial rows (summed over the ranks later)
    __device__ const __half *row_ptr(uint32_t u, uint32_t) const
    {
        return lw.wo + (uint64_t)u * dd.H * dd.hd;
    }
    __device__ void prologue(float *xs, float *) const
    {
        stage_copy(attn, dd.H * dd.hd, xs);
    }
    __device__ void epilogue(uint32_t u, const float *s) const
    {
        if (part)
            part[u] = s[0];
        else
            x[u] = __float2half_rn(__half2float(x[u]) + round_f16(s[0]));
    }
    __device__ void finish() const
    {
    }
};

// ffn.norm + up / gate projections + SiLU gating: m = fp16(fp16(u) * fp16(silu(g))) (up, gate(act=1)
// and mul nodes, src/models/vkllm_llama2_layers.c:36-60). A unit is one FFN column: its up row and
// its gate row.
struct UpGateOp
{
    static constexpr int NM = 2;
    LayerW lw;
    DecodeDims dd;
    const __half *x;
    __half *m;
    __device__ const __half *row_ptr(uint32_t u, uint32_t k) const
    {
        return (k == 0 ? lw.wu : lw.wg) + (uint64_t)u * dd.D;
    }
    __device__ void prologue(float *xs, float *red) const
    {
        stage_rmsnorm(x, lw.ffn_norm, dd.D, dd.eps, xs, red);
    }
    __device__ void epilogue(uint32_t u, const float *s) const
    {
        m[u] = __float2half_rn(round_f16(s[0]) * round_f16(silu_f32(s[1])));
    }
    __device__ void finish() const
    {
    }
};

// Down projection + residual: x = fp16(x + fp16(m . Wd^T)) (down and add nodes).
struct DownOp
{
    static constexpr int NM = 1;
    LayerW lw;
    DecodeDims dd;
    const __half *m;
    __half *x;
    float *part = nullptr; // tensor parallel: this rank's fp32 partial rows (summed over the ranks later)
    __device__ const __half *row_ptr(uint32_t u, uint32_t) const
    {
        return lw.wd + (uint64_t)u * dd.F;
    }
    __device__ void prologue(float *xs, float *) const
    {
        stage_copy(m, dd.F, xs);
    }
    __device__ void epilogue(uint32_t u, const float *s) const
    {
        if (part)
            part[u] = s[0];
        else
            x[u] = __float2half_rn(__half2float(x[u]) + round_f16(s[0]));
    }
    __device__ void finish() const
    {
    }
};

// The end of the reference argmax (src/shaders/vkllm_arg_max.comp:77-90) for one warp holding the
// 32 class winners (lane = class; idx 0xffffffff for an empty class): the 16/8/4/2/1 tree keeps the
// left operand unless the right one is strictly greater; lane 0 then records the token in the step
// state and the token ring and advances the position.
__device__ __forceinline__ void argmax_tree_finish(float v, uint32_t idx, uint32_t lane, StepState *st,
                                                   uint32_t *ring, uint32_t ring_len)
{
    if (idx == 0xffffffffu)
    {
        v = -FLT_MAX; // empty class (V < 32): the reference lane keeps -FLT_MAX and its own index
        idx = lane;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const float ov = __shfl_down_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, idx, o);
        if ((int)lane < o && ov > v)
        {
            v = ov;
            idx = oi;
        }
    }
    if (lane == 0)
    {
        st->token = idx;
        if (st->step < ring_len)
            ring[st->step] = idx;
        st->step += 1;
        st->pos += 1;
    }
}

// output_norm + logits + ARG_MAX. Every CTA stores its fp16 logits; the last CTA to finish computes
// the argmax over all of them with the reference tie rule (src/shaders/vkllm_arg_max.comp:54-90):
// index i competes in class i mod 32 where the first (smallest-index) strict maximum wins; classes
// are then reduced by the 16/8/4/2/1 tree that keeps the left operand unless the right one is
// strictly greater. It then writes the token into the step state and advances it.
struct LogitsOp
{
    static constexpr int NM = 1;
    const __half *wout;
    const float *gnorm;
    DecodeDims dd;
    const __half *x;
    __half *logits;
    uint32_t *counter;
    StepState *st;
    uint32_t *ring;
    uint32_t ring_len;
    // Tensor parallel: this rank's rows are vocabulary entries v0 .., and instead of finishing the
    // argmax it writes its 32 class candidates to tp_cls ([32] values, then [32] indices) for the
    // exchange (k_tp_argmax finishes).
    uint32_t v0 = 0;
    uint32_t *tp_cls = nullptr;
    __device__ const __half *row_ptr(uint32_t u, uint32_t) const
    {
        return wout + (uint64_t)u * dd.D;
    }
    __device__ void prologue(float *xs, float *red) const
    {
        stage_rmsnorm(x, gnorm, dd.D, dd.eps, xs, red);
    }
    __device__ void epilogue(uint32_t u, const float *s) const
    {
        logits[u] = __float2half_rn(s[0]);
    }
    __device__ void finish() const
    {
        __shared__ uint32_t last;
        __shared__ float cls_v[kStreamMaxWarps][32];
        __shared__ uint32_t cls_i[kStreamMaxWarps][32];
        const uint32_t nw = blockDim.x >> 5;
        const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0)
            last = atomicAdd(counter, 1u) == gridDim.x - 1 ? 1u : 0u;
        __syncthreads();
        if (!last)
            return;
        __threadfence();
        const uint32_t V = dd.V;
        float bv = -FLT_MAX;
        uint32_t bi = 0xffffffffu;
        // class of a row = its vocabulary index (v0 + i) mod 32
        for (uint32_t i = ((lane + 32 - (v0 & 31)) & 31) + 32 * warp; i < V; i += 32 * nw)
        {
            const float v = __half2float(__ldcg(logits + i));
            if (bi == 0xffffffffu || v > bv)
            {
                bv = v;
                bi = v0 + i;
            }
        }
        cls_v[warp][lane] = bv;
        cls_i[warp][lane] = bi;
        __syncthreads();
        if (warp == 0)
        {
            float v = -FLT_MAX;
            uint32_t idx = 0xffffffffu;
            for (uint32_t w = 0; w < nw; ++w)
            {
                const float cv = cls_v[w][lane];
                const uint32_t ci = cls_i[w][lane];
                if (ci == 0xffffffffu)
                    continue;
                if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))
                {
                    v = cv;
                    idx = ci;
                }
            }
            if (tp_cls)
            {
                tp_cls[lane] = __float_as_uint(v);
                tp_cls[32 + lane] = idx;
                if (lane == 0)
                    *counter = 0;
                return;
            }
            argmax_tree_finish(v, idx, lane, st, ring, ring_len);
            if (lane == 0)
                *counter = 0;
        }
    }
};

// Tensor parallel: x = fp16(x + fp16(sum)), sum = the ranks' Wo / down partial rows after the
// allreduce (the projection node's rounding, then the residual add).
__global__ void k_tp_residual(__half *__restrict__ x, const float *__restrict__ sum, uint32_t n)
{
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < n; u += gridDim.x * blockDim.x)
        x[u] = __float2half_rn(__half2float(x[u]) + round_f16(sum[u]));
}

// Tensor parallel: the argmax over the ranks' class candidates (cls: [world][64] words as LogitsOp
// writes them, ranks in vocabulary order). Class c takes the largest value over the ranks, ties to
// the smallest index (the lower rank, whose indices are smaller), as the reference's in-order scan
// of one class does; then the tree. One warp.
__global__ void k_tp_argmax(const uint32_t *__restrict__ cls, uint32_t world, StepState *st, uint32_t *ring,
                            uint32_t ring_len)
{
    const uint32_t lane = threadIdx.x & 31;
    float v = -FLT_MAX;
    uint32_t idx = 0xffffffffu;
    for (uint32_t q = 0; q < world; ++q)
    {
        const float cv = __uint_as_float(cls[q * 64 + lane]);
        const uint32_t ci = cls[q * 64 + 32 + lane];
        if (ci == 0xffffffffu)
            continue;
        if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))
        {
            v = cv;
            idx = ci;
        }
    }
    argmax_tree_finish(v, idx, lane, st, ring, ring_len);
}

__global__ void k_set_state(StepState *st, const uint32_t *tok_src, uint32_t token, uint32_t pos)
{
    st->token = tok_src ? *tok_src : token;
    st->pos = pos;
    st->step = 0;
    st->error = 0;
}

__global__ void k_emit_token(const StepState *st, uint32_t *out)
{
    *out = st->token;
}

} // namespace vkb
