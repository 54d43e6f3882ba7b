// Batched greedy decode of independent sequences that share one model's weights (
// 64 sequences, each with its own prompt and KV cache). One decode step of all sequences is the
// reference graph of vkllm_llama2_layers.c with S = 1 per sequence, evaluated for B sequences at
// once: the projections become GEMMs with M = B on the tensor cores (tcgen05, split-K when M is
// small), the weights stream once per step for all sequences, and the per-sequence parts (RoPE at
// each sequence's own position, KV rows, attention over its own cache, argmax) run as small kernels.
// Every node output is rounded to fp16 where the reference materialises it; arithmetic is fp32.
//
// Sequences are prefilled through the drop-in graph API (the model's own KV cache) and their rows
// copied into the batch (vkllm_b200_batch_load_sequence). One step is captured as a CUDA graph.
#include <cfloat>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <initializer_list>
#include <vector>

#include "../kernels/kernels.h"
#include "gemv_stream.cuh"
#include "../runtime/internal.h"
#include "vkllm_b200.h"
#include "vkllm_kvcache.h"
#include "vkllm_models_llama2.h"

namespace vkb
{
struct BatchDims
{
    uint32_t D, H, hd, F, V, ctx;
    float eps, rope_base, scale;
};

struct BatchLayer
{
    const __half *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *attn_norm, *ffn_norm;
    // The GEMM operands: [Wq; Wk; Wv] as [3 HD, D] and [Wup; Wgate] as [2 F, D], so that each is one
    // GEMM with M = sequences (fewer, larger GEMMs fill the SMs without splitting K). With the tiled
    // layout (the default) these and wo_g / wd_g are the batch's gemm_tile_b copies, whose B loads
    // stream contiguous 16 KB tiles. In place (tiled = 2) they are the model's own matrices, read as
    // grouped B operands (wqkv, wqkv1, wqkv2 and wug, wug1, each group_* rows): no copy is made.
    // Otherwise (tiled = 0) wqkv / wug are row-major concatenated copies and wo_g / wd_g the model's.
    const __half *wqkv, *wug, *wo_g, *wd_g;
    const __half *wqkv1 = nullptr, *wqkv2 = nullptr, *wug1 = nullptr;
    uint32_t group_qkv = 0, group_ug = 0;
};
} // namespace vkb

struct vkllm_b200_batch
{
    vkllm_context *ctx = nullptr;
    vkllm_models_llama2 *model = nullptr;
    uint32_t B = 0, cap = 0, L = 0, HD = 0, unk = 0;
    vkb::BatchDims dd{};
    std::vector<vkb::BatchLayer> layers;
    const __half *embed = nullptr, *wout = nullptr, *wout_g = nullptr; // wout_g: the logits GEMM operand
    uint32_t tiled = 1;                                                  // GEMM operands in tile order
    uint32_t att_staged = 256; // threads of k_b_attention_staged (0: k_b_attention)
    uint32_t att_chunk = 64, att_ring = 3; // its rows per chunk and chunk buffers
    uint32_t att_tc = 128;                 // threads of k_b_attention_tc (tensor-core attention; 0: off)
    // K splits and tiles (0: 128 x 128, 1: 128 x 256) of the QKV, up/gate and Wo / down GEMMs
    uint32_t qkv_splits = 3, ug_splits = 3, proj_splits = 4, qkv_tile = 1, ug_tile = 1, proj_tile = 0;
    const float *out_norm = nullptr;
    void *ws = nullptr;
    __half *kv = nullptr; // [L][2][B][H][cap][hd]
    __half *x = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *t0 = nullptr, *ug = nullptr,
           *m = nullptr, *logits = nullptr; // qkv [B][3 HD], ug [B][2 F] (up, then SiLU(gate)), m [B][F]
    __half *wcat = nullptr;                  // the GEMM operand copies of every layer (and wout_g when tiled)
    float *part = nullptr; // fp32 split-K partials of the GEMMs ([splits][B][N], summed by their consumers)
    uint32_t *tok = nullptr, *pos = nullptr, *ring = nullptr, *err = nullptr;
    uint32_t ring_steps = 0, last_steps = 0;
    std::vector<uint32_t> host_pos; // positions as the host knows them (load + steps)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace vkb
{
namespace
{

constexpr int kBT = 256;

// Lets the next kernel in the stream, when it was launched as this one's programmatic dependent (the
// batch's GEMMs), start its CTAs now; it still waits for this grid's completion before reading.
__device__ __forceinline__ void pdl_trigger()
{
    asm volatile("griddepcontrol.launch_dependents;");
}

constexpr uint32_t kMaxPartSplits = 4; // most split-K partials a consumer kernel sums


// t[e] = sum over the splits (in split order, from 0) of the 8 fp32 partials at src + s * plane.
// Every split's loads are issued before the first add, so the reads overlap (the partials were just
// written and sit in L2).
__device__ __forceinline__ void sum_splits8(const float *src, uint64_t plane, uint32_t splits, float (&t)[8])
{
    float4 a[kMaxPartSplits], c[kMaxPartSplits];
#pragma unroll
    for (uint32_t sp = 0; sp < kMaxPartSplits; ++sp)
        if (sp < splits)
        {
            a[sp] = __ldcs(reinterpret_cast<const float4 *>(src + sp * plane));
            c[sp] = __ldcs(reinterpret_cast<const float4 *>(src + sp * plane) + 1);
        }
#pragma unroll
    for (int e = 0; e < 8; ++e)
        t[e] = 0.f;
#pragma unroll
    for (uint32_t sp = 0; sp < kMaxPartSplits; ++sp)
        if (sp < splits)
        {
            t[0] += a[sp].x, t[1] += a[sp].y, t[2] += a[sp].z, t[3] += a[sp].w;
            t[4] += c[sp].x, t[5] += c[sp].y, t[6] += c[sp].z, t[7] += c[sp].w;
        }
}

__device__ __forceinline__ float bsum(float v, float *red)
{
    v = warp_sum(v);
    const uint32_t w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0)
        red[w] = v;
    __syncthreads();
    if (w == 0)
    {
        float t = l < (blockDim.x >> 5) ? red[l] : 0.f;
        t = warp_sum(t);
        if (l == 0)
            red[0] = t;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

__global__ void k_b_embed(const __half *__restrict__ table, uint32_t V, uint32_t D, uint32_t unk,
                          const uint32_t *__restrict__ tok, __half *__restrict__ x)
{
    uint32_t t = tok[blockIdx.x];
    if (t >= V)
        t = unk; // src/shaders/vkllm_embedding.comp:57-60
    const uint4 *src = reinterpret_cast<const uint4 *>(table + (uint64_t)t * D);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (uint64_t)blockIdx.x * D);
    for (uint32_t i = threadIdx.x; i < D / 8; i += blockDim.x)
        dst[i] = src[i];
}

// RMSNORM node per row: fp16((x * g) * rsqrt(mean(x^2) + eps)); 8 halves per load and store
// (D % 8 == 0).
__global__ void k_b_rmsnorm(const __half *__restrict__ x, const float *__restrict__ g, uint32_t D, float eps,
                            __half *__restrict__ y)
{
    pdl_trigger();
    __shared__ float red[32];
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + (uint64_t)blockIdx.x * D);
    const uint32_t n8 = D / 8;
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < n8; i += blockDim.x)
    {
        const uint4 v = xr[i];
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 f = __half22float2(h[e]);
            s = fmaf(f.x, f.x, s);
            s = fmaf(f.y, f.y, s);
        }
    }
    const float alpha = rsqrtf(bsum(s, red) / (float)D + eps);
    uint4 *yr = reinterpret_cast<uint4 *>(y + (uint64_t)blockIdx.x * D);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    for (uint32_t i = threadIdx.x; i < n8; i += blockDim.x)
    {
        const uint4 v = xr[i];
        const float4 ga = g4[2 * i], gb = g4[2 * i + 1];
        const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 f = __half22float2(h[e]);
            oh[e] = __floats2half2_rn((f.x * gg[2 * e]) * alpha, (f.y * gg[2 * e + 1]) * alpha);
        }
        yr[i] = o;
    }
}

// ROPE of q and k at each sequence's position (theta = pos / base^(2w / hd)), then the k and v rows
// written at that position of the sequence's caches (the UPDATE_ROWS nodes). q is rotated in place.
// Block (head, sequence), one thread per rotation pair w of the head.
__global__ void k_b_rope_kv(__half *__restrict__ q, const __half *__restrict__ k, const __half *__restrict__ v,
                            uint32_t stride, const uint32_t *__restrict__ pos, uint32_t H, uint32_t hd, uint32_t cap,
                            float base, __half *__restrict__ kc, __half *__restrict__ vc, uint32_t B)
{
    const uint32_t h = blockIdx.x, b = blockIdx.y, p = pos[b];
    if (p >= cap)
        return; // flagged by k_b_check_pos; no write outside the sequence's rows
    const uint64_t src = (uint64_t)b * stride + (uint64_t)h * hd, row = (((uint64_t)b * H + h) * cap + p) * hd;
    for (uint32_t w = threadIdx.x; w < hd / 2; w += blockDim.x)
    {
        const float theta = (float)p / powf(base, (float)(2 * w) / (float)hd);
        const float c = cosf(theta), sn = sinf(theta);
        __half2 *qp = reinterpret_cast<__half2 *>(q + src) + w;
        const float2 qf = __half22float2(*qp), kf = __half22float2(reinterpret_cast<const __half2 *>(k + src)[w]);
        *qp = __floats2half2_rn(c * qf.x - sn * qf.y, sn * qf.x + c * qf.y);
        reinterpret_cast<__half2 *>(kc + row)[w] = __floats2half2_rn(c * kf.x - sn * kf.y, sn * kf.x + c * kf.y);
        reinterpret_cast<__half2 *>(vc + row)[w] = reinterpret_cast<const __half2 *>(v + src)[w];
    }
}

// k_b_rope_kv reading the QKV GEMM's fp32 split-K partials ([splits][B][3 HD]) instead of its
// output: q, k, v = fp16(sum of the splits in split order), the rounding of the GEMM's own reduction,
// then the same rotation. The rotated q goes to q (row stride 3 HD) for the attention kernel.
__global__ void k_b_rope_kv_part(const float *__restrict__ part, uint32_t splits, __half *__restrict__ q, uint32_t HD,
                                 const uint32_t *__restrict__ pos, uint32_t H, uint32_t hd, uint32_t cap, float base,
                                 __half *__restrict__ kc, __half *__restrict__ vc, uint32_t B)
{
    const uint32_t h = blockIdx.x, b = blockIdx.y, p = pos[b];
    if (p >= cap)
        return; // flagged by k_b_check_pos; no write outside the sequence's rows
    const uint64_t plane = (uint64_t)B * 3 * HD;
    const uint64_t src = (uint64_t)b * 3 * HD + (uint64_t)h * hd, row = (((uint64_t)b * H + h) * cap + p) * hd;
    for (uint32_t w = threadIdx.x; w < hd / 2; w += blockDim.x)
    {
        // every split's loads first, then the sums in split order
        float2 pa[kMaxPartSplits], pk[kMaxPartSplits], pv[kMaxPartSplits];
#pragma unroll
        for (uint32_t sp = 0; sp < kMaxPartSplits; ++sp)
            if (sp < splits)
            {
                const float *pp = part + sp * plane + src + 2 * w;
                pa[sp] = __ldcs(reinterpret_cast<const float2 *>(pp));
                pk[sp] = __ldcs(reinterpret_cast<const float2 *>(pp + HD));
                pv[sp] = __ldcs(reinterpret_cast<const float2 *>(pp + 2 * HD));
            }
        float2 qs = make_float2(0.f, 0.f), ks = qs, vs = qs;
#pragma unroll
        for (uint32_t sp = 0; sp < kMaxPartSplits; ++sp)
            if (sp < splits)
                qs.x += pa[sp].x, qs.y += pa[sp].y, ks.x += pk[sp].x, ks.y += pk[sp].y, vs.x += pv[sp].x, vs.y += pv[sp].y;
        const float theta = (float)p / powf(base, (float)(2 * w) / (float)hd);
        const float c = cosf(theta), sn = sinf(theta);
        const float2 qf = make_float2(round_f16(qs.x), round_f16(qs.y)), kf = make_float2(round_f16(ks.x), round_f16(ks.y));
        reinterpret_cast<__half2 *>(q + src)[w] = __floats2half2_rn(c * qf.x - sn * qf.y, sn * qf.x + c * qf.y);
        reinterpret_cast<__half2 *>(kc + row)[w] = __floats2half2_rn(c * kf.x - sn * kf.y, sn * kf.x + c * kf.y);
        reinterpret_cast<__half2 *>(vc + row)[w] = __floats2half2_rn(vs.x, vs.y);
    }
}

constexpr uint32_t kAttChunk = 64;    // key rows per staged chunk (staged attention), default
constexpr uint32_t kAttTcChunk = 48;   // key rows per chunk of the tensor-core attention, default
constexpr uint32_t kAttTcThreads = 128; // threads per CTA of the tensor-core attention, default
// chunk buffers in flight per CTA, default (7B, 64 sequences: 2 / 3 buffers of 64 rows 4.877 / 4.966 ms
// per step; 4 / 6 of 32 rows 5.038 / 5.156)
constexpr uint32_t kAttStages = 2;
constexpr uint32_t kAttMaxStages = 8; // most chunk buffers
constexpr uint32_t kAttThreads = 512; // most threads of the staged attention kernel
constexpr uint32_t kErrAttTimeout = 2u; // batch error bit: a staged-attention copy wait expired

// Dynamic shared memory of k_b_attention_staged for head size hd and cap KV rows.
__host__ __device__ constexpr size_t att_staged_smem(uint32_t hd, uint32_t cap, uint32_t threads, uint32_t chunk,
                                                     uint32_t stages)
{
    return (size_t)stages * chunk * hd * 2 + 8 * stages +
           4 * ((size_t)((hd + 3) & ~3u) + ((cap + 3) & ~3u) + (size_t)(threads / 32) * hd);
}

// Attention of one (head, sequence) as k_b_attention computes it, with the sequence's key rows and
// then its value rows streamed through shared memory: `chunk`-row chunks (Lk x hd fp16 rows are
// contiguous in the batch's cache) are fetched by cp.async.bulk into a ring of `stages` buffers,
// so the copies of later chunks (the first value chunks included) are in flight while the scores,
// the softmax statistics and the probabilities of earlier ones are computed. Scores: `lpk` lanes
// per key row (8 fp16 each) and a shuffle sum; probabilities: the same rounding points as
// k_b_attention. Each mbarrier wait is bounded; on expiry the CTA sets kErrAttTimeout in *err,
// waits (bounded) for its copies in flight and returns.
__global__ void __launch_bounds__(kAttThreads) k_b_attention_staged(const __half *__restrict__ q, uint32_t q_stride,
                                                                  const __half *__restrict__ kc,
                                                                  const __half *__restrict__ vc,
                                                                  const uint32_t *__restrict__ pos, uint32_t H,
                                                                  uint32_t hd, uint32_t cap, float scale,
                                                                  __half *__restrict__ out, uint32_t *err,
                                                                  uint32_t chunk, uint32_t stages)
{
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char att_sm[];
    const uint32_t chunk_elems = chunk * hd; // chunk: rows per chunk (multiple of 8), stages <= kAttMaxStages
    __half *ring = reinterpret_cast<__half *>(att_sm);
    uint64_t *bars = reinterpret_cast<uint64_t *>(att_sm + (size_t)stages * chunk_elems * 2);
    float *qs = reinterpret_cast<float *>(bars + stages);
    float *sc = qs + ((hd + 3) & ~3u);
    float *acc = sc + ((cap + 3) & ~3u); // [warps][hd]
    __shared__ float red[32];
    const uint32_t h = blockIdx.x, b = blockIdx.y, HD = H * hd, tid = threadIdx.x;
    if (pos[b] >= cap)
        return; // flagged by k_b_check_pos
    const uint32_t Lk = pos[b] + 1, nk = (Lk + chunk - 1) / chunk, total = 2 * nk;
    const uint32_t warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const __half *kb = kc + ((uint64_t)b * H + h) * cap * hd;
    const __half *vb = vc + ((uint64_t)b * H + h) * cap * hd;
    // chunk c < nk: key rows [chunk c, ...); c >= nk: value rows [chunk (c - nk), ...); buffer c % stages
    auto issue = [&](uint32_t c) {
        const uint32_t r0 = (c < nk ? c : c - nk) * chunk, rows = min(chunk, Lk - r0);
        const uint32_t st = c % stages;
        mbar_arrive_expect_tx(&bars[st], rows * hd * 2);
        bulk_g2s(ring + (size_t)st * chunk_elems, (c < nk ? kb : vb) + (uint64_t)r0 * hd, rows * hd * 2, &bars[st]);
    };
    if (tid == 0)
    {
        for (uint32_t st = 0; st < stages; ++st)
            mbar_init(&bars[st], 1);
        fence_barrier_init();
    }
    for (uint32_t d = tid; d < hd; d += blockDim.x)
        qs[d] = __half2float(q[(uint64_t)b * q_stride + h * hd + d]);
    __syncthreads();
    if (tid == 0)
        for (uint32_t c = 0; c < stages && c < total; ++c)
            issue(c);
    const uint32_t pieces = hd / 8;
    uint32_t lpk = 1;
    while (lpk < pieces)
        lpk <<= 1;
    const uint32_t G = blockDim.x / lpk, gi = tid / lpk, pc = tid % lpk;
    const bool lane_on = pc < pieces;
    float qr[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
        qr[e] = lane_on ? qs[8 * pc + e] : 0.f;
    float mx = -FLT_MAX;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const bool quirk = Lk == hd; // V read as [hd, Lk] (src/core/vkllm_op_matmul.c:14-30)
    __half *o = out + (uint64_t)b * HD + h * hd;
    for (uint32_t c = 0; c < total; ++c)
    {
        const uint32_t st = c % stages;
        const bool timed_out = !mbar_wait_bounded(&bars[st], (c / stages) & 1u, kWaitLimitNs);
        if (__syncthreads_or(timed_out))
        {
            if (tid == 0)
            {
                atomicOr(err, kErrAttTimeout);
                // the copies issued and not yet consumed must land before the CTA exits
                for (uint32_t k = c; k < total && k < c + stages; ++k)
                    (void)mbar_wait_bounded(&bars[k % stages], (k / stages) & 1u, kWaitLimitNs / 4);
            }
            return;
        }
        const __half *buf = ring + (size_t)st * chunk_elems;
        const uint32_t r0 = (c < nk ? c : c - nk) * chunk, rows = min(chunk, Lk - r0);
        if (c < nk)
        {
            // scores of this chunk's keys: group gi takes rows gi, gi + G, ...
            for (uint32_t rb = 0; rb < rows; rb += G)
            {
                const uint32_t r = rb + gi;
                const bool valid = lane_on && r < rows;
                float d = 0.f;
                if (valid)
                {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(buf + (size_t)r * hd + 8 * pc);
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                    {
                        const float2 f = __half22float2(hh[e]);
                        d = fmaf(qr[2 * e], f.x, d);
                        d = fmaf(qr[2 * e + 1], f.y, d);
                    }
                }
                for (uint32_t sh = lpk / 2; sh > 0; sh >>= 1)
                    d += __shfl_xor_sync(0xffffffffu, d, sh);
                if (r < rows)
                {
                    const float sv = round_f16(d * scale);
                    if (pc == 0)
                        sc[r0 + r] = sv;
                    mx = fmaxf(mx, sv);
                }
            }
            if (c + 1 == nk)
            {
                // softmax over the whole row: max, sum of exp, p_j = fp16(exp(s_j - max) / sum)
                mx = warp_max(mx);
                if (lane == 0)
                    red[warp] = mx;
                __syncthreads();
                float m = -FLT_MAX;
                for (uint32_t w = 0; w < nw; ++w)
                    m = fmaxf(m, red[w]);
                __syncthreads();
                float l = 0.f;
                for (uint32_t j = tid; j < Lk; j += blockDim.x)
                    l += expf(sc[j] - m);
                l = bsum(l, red);
                for (uint32_t j = tid; j < Lk; j += blockDim.x)
                    sc[j] = round_f16(expf(sc[j] - m) / l);
            }
        }
        else if (quirk)
        {
            // o[w] = sum_k p_k V[w][k] for the value rows w of this chunk
            for (uint32_t r = tid; r < rows; r += blockDim.x)
            {
                float v = 0.f;
                for (uint32_t k = 0; k < Lk; ++k)
                    v = fmaf(sc[k], __half2float(buf[(size_t)r * hd + k]), v);
                o[r0 + r] = __float2half_rn(v);
            }
        }
        else if (lane_on)
        {
            for (uint32_t r = gi; r < rows; r += G)
            {
                const float pj = sc[r0 + r];
                const uint4 raw = *reinterpret_cast<const uint4 *>(buf + (size_t)r * hd + 8 * pc);
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                {
                    const float2 f = __half22float2(hh[e]);
                    a[2 * e] = fmaf(pj, f.x, a[2 * e]);
                    a[2 * e + 1] = fmaf(pj, f.y, a[2 * e + 1]);
                }
            }
        }
        __syncthreads(); // buffer st is free (and, after the last key chunk, the probabilities are set)
        if (tid == 0 && c + stages < total)
        {
            fence_proxy_async();
            issue(c + stages);
        }
    }
    if (quirk)
        return;
    // the key groups of a warp are summed with shuffles, then the warps' sums in warp order
#pragma unroll
    for (int e = 0; e < 8; ++e)
        for (uint32_t sh = lpk; sh < 32; sh <<= 1)
            a[e] += __shfl_xor_sync(0xffffffffu, a[e], sh);
    if (lane < lpk && lane_on)
#pragma unroll
        for (int e = 0; e < 8; ++e)
            acc[warp * hd + 8 * pc + e] = a[e];
    __syncthreads();
    for (uint32_t d = tid; d < hd; d += blockDim.x)
    {
        float v = 0.f;
        for (uint32_t w = 0; w < nw; ++w)
            v += acc[w * hd + d];
        o[d] = __float2half_rn(v);
    }
}


// Dynamic shared memory of k_b_attention_tc: 1 KB of alignment slack, the chunk ring (each buffer
// hd / 64 swizzled boxes of chunk x 128 bytes), the mbarriers, the fp16 scores and probabilities
// over the cap rounded up to whole chunks, the second key half's output slices (hd < 128) and q.
__host__ __device__ constexpr size_t att_tc_smem(uint32_t hd, uint32_t cap, uint32_t chunk, uint32_t stages)
{
    return 1024 + (size_t)stages * chunk * hd * 2 + 8 * stages + 2 * 2 * ((size_t)(cap + chunk - 1) / chunk * chunk + 16) +
           4 * (size_t)hd + 2 * (size_t)hd;
}

__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1, int32_t c2,
                                              int32_t c3, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
                 "%4, %5}], [%6];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void att_ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void att_ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// d += A (16 x 16, fp16, row-major fragment) . B (16 x 8, fp16, column fragment), fp32 accumulation
__device__ __forceinline__ void att_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory address of 16-byte piece `dc` (0 .. hd / 8 - 1) of row r of a chunk buffer: piece dc
// lies in box dc / 8 (64 fp16 columns each, chunk x 128 bytes), swizzled by the TMA's 128-byte
// pattern (piece c of a box row r at c ^ (r & 7)).
__device__ __forceinline__ uint32_t att_piece(uint32_t buf, uint32_t chunk, uint32_t r, uint32_t dc)
{
    return buf + (dc >> 3) * chunk * 128 + r * 128 + (((dc & 7) ^ (r & 7)) << 4);
}

// Attention of one (head, sequence) on the tensor cores: the same nodes as k_b_attention_staged
// (scores s_j = fp16(scale * q.k_j), p_j = fp16(exp(s_j - max) / sum), output fp16(sum_j p_j v_j)),
// with the sums of products on mma.sync m16n8k16 (fp16 operands, whose products are exact, fp32
// accumulation) instead of per-lane FMAs and shuffles. The sequence's key rows, then its value rows,
// arrive as `chunk`-row chunks of 16-row TMA boxes (128-byte swizzle) in a ring of `stages` buffers.
//  * Scores: warp w takes 16-key blocks w, w + 8, ... of a chunk; A = the block's key rows (ldmatrix),
//    B = q in all 8 columns, so every column of D holds the block's 16 scores.
//  * Output: the hd / 16 slices of 16 output columns are dealt to the warps (several per warp when
//    they outnumber the warps; with more warps than slices, the key blocks are split in two parts
//    summed at the end); A = the probabilities in all 16 rows, B = the value rows
//    (ldmatrix.trans), so every row of D holds p . V for 16 columns. Key rows past Lk in the last
//    value chunk are zeroed before use (their probabilities are 0, and 0 times a stale value must stay 0).
// At Lk == hd the reference reads V as [hd, Lk] (src/core/vkllm_op_matmul.c:14-30); that step runs a
// scalar path from global memory. Each mbarrier wait is bounded; on expiry the CTA sets kErrAttTimeout
// in *err, waits (bounded) for its copies in flight and returns.
template <uint32_t HD, uint32_t NT>
__global__ void __launch_bounds__(NT, NT == 256 ? 5 : 10) k_b_attention_tc(const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap,
                                                                const __half *__restrict__ q, uint32_t q_stride,
                                                                const __half *__restrict__ kc,
                                                                const __half *__restrict__ vc,
                                                                const uint32_t *__restrict__ pos, uint32_t H,
                                                                uint32_t cap, float scale, __half *__restrict__ out,
                                                                uint32_t *err, uint32_t chunk, uint32_t stages)
{
    static_assert(HD % 64 == 0 && HD <= 128 && (NT == 128 || NT == 256), "head size, threads");
    // output slices of 16 columns: G groups of warps own kSPW slices each (slices g, g + G, ...);
    // with more warps than slices the key blocks are split into kParts parts
    constexpr uint32_t kWarps = NT / 32, kSlices = HD / 16, kG = kSlices < kWarps ? kSlices : kWarps;
    constexpr uint32_t kSPW = kSlices / kG, kParts = kWarps / kG;
    static_assert(kParts <= 2, "key parts");
    pdl_trigger();
    extern __shared__ unsigned char att_tc_sm[];
    __shared__ float red[32];
    const uint32_t h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (pos[b] >= cap)
        return; // flagged by k_b_check_pos
    const uint32_t Lk = pos[b] + 1;
    const __half *qv = q + (uint64_t)b * q_stride + h * HD;
    __half *o_out = out + (uint64_t)b * H * HD + h * HD;
    const uint32_t capr = (cap + chunk - 1) / chunk * chunk + 16;
    const uint32_t base = (smem_u32(att_tc_sm) + 1023u) & ~1023u; // swizzled boxes need 1 KB alignment
    unsigned char *sm = att_tc_sm + (base - smem_u32(att_tc_sm));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + (size_t)stages * chunk * HD * 2);
    __half *sc = reinterpret_cast<__half *>(bars + stages); // [capr] scores
    __half *ph = sc + capr;                                  // [capr] probabilities, 0 past Lk
    float *acc = reinterpret_cast<float *>(ph + capr);       // [HD] the second key part's output, then q
    if (Lk == HD)
    {
        // quirk Q1, scalar from global memory: o[w] = sum_k p_k V[w][k] with V read as [hd, Lk]
        const __half *kb = kc + ((uint64_t)b * H + h) * cap * HD;
        const __half *vb = vc + ((uint64_t)b * H + h) * cap * HD;
        float mx = -FLT_MAX;
        for (uint32_t j = tid; j < Lk; j += blockDim.x)
        {
            float a = 0.f;
#pragma unroll 4
            for (uint32_t d = 0; d < HD; ++d)
                a = fmaf(__half2float(qv[d]), __half2float(kb[(uint64_t)j * HD + d]), a);
            const float s = round_f16(a * scale);
            sc[j] = __float2half_rn(s);
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        if (lane == 0)
            red[warp] = mx;
        __syncthreads();
        float m = -FLT_MAX;
        for (uint32_t w = 0; w < (blockDim.x >> 5); ++w)
            m = fmaxf(m, red[w]);
        __syncthreads();
        float l = 0.f;
        for (uint32_t j = tid; j < Lk; j += blockDim.x)
            l += expf(__half2float(sc[j]) - m);
        l = bsum(l, red);
        for (uint32_t j = tid; j < Lk; j += blockDim.x)
            ph[j] = __float2half_rn(expf(__half2float(sc[j]) - m) / l);
        __syncthreads();
        for (uint32_t w = tid; w < HD; w += blockDim.x)
        {
            float v = 0.f;
            for (uint32_t k = 0; k < Lk; ++k)
                v = fmaf(__half2float(ph[k]), __half2float(vb[(uint64_t)w * Lk + k]), v);
            o_out[w] = __float2half_rn(v);
        }
        return;
    }
    const uint32_t nk = (Lk + chunk - 1) / chunk, total = 2 * nk, buf_bytes = chunk * HD * 2;
    // chunk c < nk: key rows [chunk c, ...); c >= nk: value rows [chunk (c - nk), ...); buffer c % stages.
    // The maps' boxes are 16 rows, so a chunk fetches only the 16-key blocks that hold keys below Lk;
    // each lands at its row offset (a multiple of 8) of the chunk's boxes, in the same swizzled layout.
    auto issue = [&](uint32_t c) {
        const uint32_t st = c % stages, r0 = (c < nk ? c : c - nk) * chunk;
        const uint32_t nb = (min(chunk, Lk - r0) + 15) / 16;
        mbar_arrive_expect_tx(&bars[st], nb * 16 * HD * 2);
        for (uint32_t i = 0; i < nb; ++i)
#pragma unroll
            for (uint32_t bx = 0; bx < HD / 64; ++bx)
                tma_load_rows(base + st * buf_bytes + bx * chunk * 128 + i * 16 * 128, c < nk ? &kmap : &vmap,
                              (int32_t)(bx * 64), (int32_t)(r0 + 16 * i), (int32_t)h, (int32_t)b, &bars[st]);
    };
    if (tid == 0)
    {
        for (uint32_t st = 0; st < stages; ++st)
            mbar_init(&bars[st], 1);
        fence_barrier_init();
        for (uint32_t c = 0; c < stages && c < total; ++c)
            issue(c);
    }
    // q as fp16 pairs in shared memory: the scores' B fragments (every column) are the pairs
    // k = 16 ks + 2 (lane & 3) + {0, 1} and the same + 8
    uint32_t *qs2 = reinterpret_cast<uint32_t *>(acc + HD);
    for (uint32_t i = tid; i < HD / 2; i += NT)
        qs2[i] = reinterpret_cast<const uint32_t *>(qv)[i];
    __syncthreads(); // mbarrier initialisation and q visible to every thread
    const uint32_t mi = lane >> 3, lrow = (lane & 7) + 8 * (mi & 1); // this lane's ldmatrix row and piece
    const uint32_t grp = warp % kG, part = warp / kG;
    float mx = -FLT_MAX;
    float o[kSPW][2][4] = {};
    for (uint32_t c = 0; c < total; ++c)
    {
        const uint32_t st = c % stages;
        const bool timed_out = !mbar_wait_bounded(&bars[st], (c / stages) & 1u, kWaitLimitNs);
        if (__syncthreads_or(timed_out))
        {
            if (tid == 0)
            {
                atomicOr(err, kErrAttTimeout);
                for (uint32_t k = c; k < total && k < c + stages; ++k)
                    (void)mbar_wait_bounded(&bars[k % stages], (k / stages) & 1u, kWaitLimitNs / 4);
            }
            return;
        }
        const uint32_t buf = base + st * buf_bytes;
        const uint32_t r0 = (c < nk ? c : c - nk) * chunk, rows = min(chunk, Lk - r0), nkb = (rows + 15) / 16;
        if (c < nk)
        {
            for (uint32_t kb = warp; kb < nkb; kb += kWarps)
            {
                float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
                for (uint32_t ks = 0; ks < HD / 16; ++ks)
                {
                    uint32_t a0, a1, a2, a3;
                    att_ldsm_x4(att_piece(buf, chunk, kb * 16 + lrow, 2 * ks + (mi >> 1)), a0, a1, a2, a3);
                    att_mma(d, a0, a1, a2, a3, qs2[8 * ks + (lane & 3)], qs2[8 * ks + 4 + (lane & 3)]);
                }
                if ((lane & 3) == 0) // d[0]: key 16 kb + lane / 4, d[2]: that + 8
#pragma unroll
                    for (uint32_t e = 0; e < 2; ++e)
                    {
                        const uint32_t r = kb * 16 + (lane >> 2) + 8 * e;
                        if (r < rows)
                        {
                            const float s = round_f16(d[2 * e] * scale);
                            sc[r0 + r] = __float2half_rn(s);
                            mx = fmaxf(mx, s);
                        }
                    }
            }
            if (c + 1 == nk)
            {
                // softmax over the whole row: max, sum of exp, p_j = fp16(exp(s_j - max) / sum), 0 past Lk
                mx = warp_max(mx);
                if (lane == 0)
                    red[warp] = mx;
                __syncthreads();
                float m = -FLT_MAX;
                for (uint32_t w = 0; w < kWarps; ++w)
                    m = fmaxf(m, red[w]);
                __syncthreads();
                float l = 0.f;
                for (uint32_t j = tid; j < Lk; j += NT)
                    l += expf(__half2float(sc[j]) - m);
                l = bsum(l, red);
                for (uint32_t j = tid; j < nk * chunk; j += NT)
                    ph[j] = j < Lk ? __float2half_rn(expf(__half2float(sc[j]) - m) / l) : __float2half_rn(0.f);
            }
        }
        else
        {
            const uint32_t padded = nkb * 16;
            if (rows < padded) // the last value chunk: zero its rows past Lk that the key blocks read
            {
                const uint32_t per_row = HD / 8, n = (padded - rows) * per_row;
                for (uint32_t i = tid; i < n; i += NT)
                {
                    const uint32_t r = rows + i / per_row, dc = i % per_row;
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(att_piece(buf, chunk, r, dc)), "r"(0u)
                                 : "memory");
                }
                __syncthreads();
            }
            for (uint32_t kb = part; kb < nkb; kb += kParts)
            {
                const uint32_t k0 = r0 + kb * 16 + 2 * (lane & 3);
                const uint32_t pa = *reinterpret_cast<const uint32_t *>(ph + k0);
                const uint32_t pb = *reinterpret_cast<const uint32_t *>(ph + k0 + 8);
#pragma unroll
                for (uint32_t j = 0; j < kSPW; ++j)
                {
                    uint32_t b00, b01, b10, b11;
                    att_ldsm_x4_t(att_piece(buf, chunk, kb * 16 + lrow, 2 * (grp + kG * j) + (mi >> 1)), b00, b01, b10,
                                  b11);
                    att_mma(o[j][0], pa, pa, pb, pb, b00, b01);
                    att_mma(o[j][1], pa, pa, pb, pb, b10, b11);
                }
            }
        }
        __syncthreads(); // buffer st is free (and, after the last key chunk, the probabilities are set)
        if (tid == 0 && c + stages < total)
        {
            fence_proxy_async();
            issue(c + stages);
        }
    }
    // o[j][0] / o[j][1]: columns 16 (grp + kG j) + 2 (lane & 3) + {0, 1} and the same + 8 (every row of
    // D is equal); with two key parts, part 1 hands its sums to part 0 through shared memory
#pragma unroll
    for (uint32_t j = 0; j < kSPW; ++j)
    {
        const uint32_t col = 16 * (grp + kG * j) + 2 * (lane & 3);
        if (kParts > 1 && part == 1 && lane < 4)
        {
            acc[col] = o[j][0][0], acc[col + 1] = o[j][0][1], acc[col + 8] = o[j][1][0], acc[col + 9] = o[j][1][1];
        }
    }
    if (kParts > 1)
        __syncthreads();
    if (part == 0 && lane < 4)
#pragma unroll
        for (uint32_t j = 0; j < kSPW; ++j)
        {
            const uint32_t col = 16 * (grp + kG * j) + 2 * (lane & 3);
            float v[4] = {o[j][0][0], o[j][0][1], o[j][1][0], o[j][1][1]};
            if (kParts > 1)
                v[0] += acc[col], v[1] += acc[col + 1], v[2] += acc[col + 8], v[3] += acc[col + 9];
            *reinterpret_cast<__half2 *>(o_out + col) = __floats2half2_rn(v[0], v[1]);
            *reinterpret_cast<__half2 *>(o_out + col + 8) = __floats2half2_rn(v[2], v[3]);
        }
}

using AttTcKernel = void (*)(CUtensorMap, CUtensorMap, const __half *, uint32_t, const __half *, const __half *,
                            const uint32_t *, uint32_t, uint32_t, float, __half *, uint32_t *, uint32_t, uint32_t);

// The instantiation for head size hd (64 or 128) and `threads` per CTA (128 or 256).
AttTcKernel att_tc_kernel(uint32_t hd, uint32_t threads)
{
    if (hd == 128)
        return threads == 128 ? k_b_attention_tc<128, 128> : k_b_attention_tc<128, 256>;
    return threads == 128 ? k_b_attention_tc<64, 128> : k_b_attention_tc<64, 256>;
}

// Attention of one (head, sequence): scores s_j = fp16(scale * q.k_j) over the sequence's Lk = pos + 1
// keys, softmax p_j = fp16(exp(s_j - max) / sum) (max over all entries, vkllm_softmax.comp), output
// fp16(sum_j p_j v_j). For Lk == hd the reference reads V as [hd, Lk] (src/core/vkllm_op_matmul.c:14-30):
// o[w] = sum_k p_k V[w][k]. Keys are read `lpk` lanes per key row (8 fp16 per lane, 16-byte loads);
// the CTA's kBT / lpk key groups each sum their keys, then the groups are summed in order.
__global__ void __launch_bounds__(kBT) k_b_attention(const __half *__restrict__ q, uint32_t q_stride,
                                                     const __half *__restrict__ kc, const __half *__restrict__ vc,
                                                     const uint32_t *__restrict__ pos, uint32_t H, uint32_t hd,
                                                     uint32_t cap, float scale, __half *__restrict__ out)
{
    pdl_trigger();
    extern __shared__ float sm[];
    float *qs = sm;           // [hd]
    float *sc = sm + 256;     // [Lk]
    __shared__ float red[32];
    const uint32_t h = blockIdx.x, b = blockIdx.y, HD = H * hd;
    if (pos[b] >= cap)
        return; // flagged by k_b_check_pos
    const uint32_t Lk = pos[b] + 1;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x)
        qs[d] = __half2float(q[(uint64_t)b * q_stride + h * hd + d]);
    __syncthreads();
    const __half *kb = kc + ((uint64_t)b * H + h) * cap * hd;
    const __half *vb = vc + ((uint64_t)b * H + h) * cap * hd;
    const uint32_t pieces = hd / 8;
    uint32_t lpk = 1;
    while (lpk < pieces)
        lpk <<= 1;
    const uint32_t G = blockDim.x / lpk, gi = threadIdx.x / lpk, pc = threadIdx.x % lpk;
    const bool lane_on = pc < pieces;
    float qr[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
        qr[e] = lane_on ? qs[8 * pc + e] : 0.f;
    float mx = -FLT_MAX;
    // four rounds of key rows in flight per lane, then their dot products in order
    for (uint32_t j0 = 0; j0 < Lk; j0 += 4 * G)
    {
        uint4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
        {
            const uint32_t j = j0 + u * G + gi;
            raw[u] = (lane_on && j < Lk) ? reinterpret_cast<const uint4 *>(kb + (uint64_t)j * hd)[pc]
                                         : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
        {
            const uint32_t j = j0 + u * G + gi;
            float a = 0.f;
            if (lane_on && j < Lk)
            {
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                {
                    const float2 f = __half22float2(hh[e]);
                    a = fmaf(qr[2 * e], f.x, a);
                    a = fmaf(qr[2 * e + 1], f.y, a);
                }
            }
            for (uint32_t o = lpk / 2; o > 0; o >>= 1)
                a += __shfl_xor_sync(0xffffffffu, a, o);
            if (j < Lk)
            {
                const float s = round_f16(a * scale);
                if (pc == 0)
                    sc[j] = s;
                mx = fmaxf(mx, s);
            }
        }
    }
    mx = warp_max(mx);
    if (lane == 0)
        red[warp] = mx;
    __syncthreads();
    float m = -FLT_MAX;
    for (uint32_t w = 0; w < nw; ++w)
        m = fmaxf(m, red[w]);
    __syncthreads();
    float l = 0.f;
    for (uint32_t j = threadIdx.x; j < Lk; j += blockDim.x)
        l += expf(sc[j] - m);
    l = bsum(l, red);
    for (uint32_t j = threadIdx.x; j < Lk; j += blockDim.x)
        sc[j] = round_f16(expf(sc[j] - m) / l);
    __syncthreads();
    __half *o = out + (uint64_t)b * HD + h * hd;
    if (Lk == hd)
    {
        for (uint32_t w = threadIdx.x; w < hd; w += blockDim.x)
        {
            float a = 0.f;
            for (uint32_t kk = 0; kk < Lk; ++kk)
                a = fmaf(sc[kk], __half2float(vb[(uint64_t)w * hd + kk]), a);
            o[w] = __float2half_rn(a);
        }
        return;
    }
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (lane_on)
        for (uint32_t j0 = gi; j0 < Lk; j0 += 4 * G) // four value rows in flight, summed in key order
        {
            uint4 raw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
            {
                const uint32_t j = j0 + u * G;
                raw[u] = j < Lk ? reinterpret_cast<const uint4 *>(vb + (uint64_t)j * hd)[pc] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
            {
                const uint32_t j = j0 + u * G;
                if (j >= Lk)
                    break;
                const float pj = sc[j];
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                {
                    const float2 f = __half22float2(hh[e]);
                    a[2 * e] = fmaf(pj, f.x, a[2 * e]);
                    a[2 * e + 1] = fmaf(pj, f.y, a[2 * e + 1]);
                }
            }
        }
    float *acc = sc + ((Lk + 31) & ~31u); // [G][hd]
    if (lane_on)
#pragma unroll
        for (int e = 0; e < 8; ++e)
            acc[gi * hd + 8 * pc + e] = a[e];
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x)
    {
        float t = 0.f;
        for (uint32_t g2 = 0; g2 < G; ++g2)
            t += acc[g2 * hd + d];
        o[d] = __float2half_rn(t);
    }
}

// The gate BIN mul from the concatenated up/gate GEMM output: m[b][f] = fp16(ug[b][f] * ug[b][F + f])
// (the gate half already SiLU'd by the GEMM epilogue), 8 halves per thread (F % 8 == 0).
// k_b_gate reading the up/gate GEMM's fp32 split-K partials ([splits][B][2 F]): up = fp16(sum),
// gate = fp16(SiLU(sum)) as the GEMM's reduction rounds them, m = fp16(up * gate).
__global__ void k_b_gate_part(__half *__restrict__ m, const float *__restrict__ part, uint32_t splits, uint32_t F,
                              uint32_t B)
{
    pdl_trigger();
    const uint32_t f8 = F / 8;
    const uint64_t plane = (uint64_t)B * 2 * F;
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < (uint64_t)B * f8;
         t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t b = (uint32_t)(t / f8), c = (uint32_t)(t % f8);
        float u[8], g[8];
        sum_splits8(part + (uint64_t)b * 2 * F + 8ull * c, plane, splits, u);
        sum_splits8(part + (uint64_t)b * 2 * F + F + 8ull * c, plane, splits, g);
        uint4 o;
        __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e)
        {
            const float gs = g[e] / (1.0f + expf(-g[e])); // SiLU as the GEMM epilogue evaluates it
            oh[e] = __float2half_rn(round_f16(u[e]) * round_f16(gs));
        }
        reinterpret_cast<uint4 *>(m + (uint64_t)b * F)[c] = o;
    }
}

__global__ void k_b_gate(__half *__restrict__ m, const __half *__restrict__ ug, uint32_t F, uint32_t B)
{
    pdl_trigger();
    const uint32_t f8 = F / 8;
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < (uint64_t)B * f8;
         t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t b = (uint32_t)(t / f8), c = (uint32_t)(t % f8);
        const uint4 u = reinterpret_cast<const uint4 *>(ug + (uint64_t)b * 2 * F)[c];
        const uint4 gt = reinterpret_cast<const uint4 *>(ug + (uint64_t)b * 2 * F + F)[c];
        const __half2 *uh = reinterpret_cast<const __half2 *>(&u), *gh = reinterpret_cast<const __half2 *>(&gt);
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 a = __half22float2(uh[e]), g = __half22float2(gh[e]);
            oh[e] = __floats2half2_rn(a.x * g.x, a.y * g.y);
        }
        reinterpret_cast<uint4 *>(m + (uint64_t)b * F)[c] = o;
    }
}

// Three graph nodes in one pass over each sequence's row: the projection's output from its split-K
// partials, t = fp16(sum of the partials in split order) (the GEMM node, scale 1); the residual BIN
// add x = fp16(x + t); and the next RMSNORM node xn = fp16((x * g) * rsqrt(mean(x^2) + eps)) over the
// new fp16 row. Block per sequence with kBT threads, 8 halves per chunk in k_b_rmsnorm's thread
// mapping (so the norm reduces in the same order).
__global__ void k_b_proj_residual_norm(const float *__restrict__ part, uint32_t splits, __half *__restrict__ x,
                                       const float *__restrict__ g, uint32_t D, float eps, __half *__restrict__ xn,
                                       uint32_t B)
{
    pdl_trigger();
    __shared__ float red[32];
    const uint32_t b = blockIdx.x, n8 = D / 8;
    const uint64_t plane = (uint64_t)B * D;
    uint4 *xr = reinterpret_cast<uint4 *>(x + (uint64_t)b * D);
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < n8; i += blockDim.x)
    {
        float t[8];
        sum_splits8(part + (uint64_t)b * D + 8ull * i, plane, splits, t);
        const uint4 xv = xr[i];
        const __half *xh = reinterpret_cast<const __half *>(&xv);
        uint4 o;
        __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e)
        {
            oh[e] = __float2half_rn(__half2float(xh[e]) + round_f16(t[e]));
            const float f = __half2float(oh[e]);
            s = fmaf(f, f, s);
        }
        xr[i] = o;
    }
    const float alpha = rsqrtf(bsum(s, red) / (float)D + eps);
    uint4 *yr = reinterpret_cast<uint4 *>(xn + (uint64_t)b * D);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    for (uint32_t i = threadIdx.x; i < n8; i += blockDim.x)
    {
        const uint4 v = xr[i]; // this thread's own chunk, written above
        const float4 ga = g4[2 * i], gb = g4[2 * i + 1];
        const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e)
        {
            const float2 f = __half22float2(h[e]);
            oh[e] = __floats2half2_rn((f.x * gg[2 * e]) * alpha, (f.y * gg[2 * e + 1]) * alpha);
        }
        yr[i] = o;
    }
}

// x = fp16(x + t) (the residual BIN add) or m = fp16(a * b) (the gate BIN mul), 8 halves per thread.
__global__ void k_b_bin8(__half *__restrict__ out, const __half *__restrict__ a, const __half *__restrict__ b,
                         uint64_t n8, int mul)
{
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n8; t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint4 va = reinterpret_cast<const uint4 *>(a)[t], vb = reinterpret_cast<const uint4 *>(b)[t];
        const __half *ha = reinterpret_cast<const __half *>(&va), *hb = reinterpret_cast<const __half *>(&vb);
        uint4 o;
        __half *ho = reinterpret_cast<__half *>(&o);
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float x = __half2float(ha[i]), y = __half2float(hb[i]);
            ho[i] = __float2half_rn(mul ? x * y : x + y);
        }
        reinterpret_cast<uint4 *>(out)[t] = o;
    }
}

// ARG_MAX per sequence with the reference rule (src/shaders/vkllm_arg_max.comp:54-90): lane l keeps
// the first strict maximum of i = l, l + 32, ...; a 16/8/4/2/1 tree keeps the left operand unless the
// right one is strictly greater. Then the token feeds back and the position advances.
__global__ void k_b_argmax(const __half *__restrict__ logits, uint32_t V, uint32_t *__restrict__ tok,
                           uint32_t *__restrict__ pos, uint32_t *__restrict__ ring, uint32_t ring_steps,
                           uint32_t *__restrict__ step_ctr, uint32_t B)
{
    // The reference's rule (src/shaders/vkllm_arg_max.comp:40-97): lane l scans class l (i = l, l + 32,
    // ...) from its first element and replaces on a strict maximum; then 16/8/4/2/1 keeps the left
    // value unless the right one is strictly greater. The block's warps split each class: a class's
    // result is (its first element, index l) when that element is NaN, else its largest non-NaN value
    // at its smallest index.
    __shared__ float cv[32][32];
    __shared__ uint32_t ci[32][32];
    const uint32_t b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const __half *row = logits + (uint64_t)b * V;
    float v = -FLT_MAX;
    uint32_t idx = 0xffffffffu;
    // this thread's elements i = lane + 32 warp + k * 32 nw, eight loads in flight at a time, compared
    // in increasing k
    const uint32_t stride = 32 * nw;
    for (uint32_t base = lane + 32 * warp; base < V; base += 8 * stride)
    {
        float c[8];
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = base + u * stride;
            c[u] = i < V ? __half2float(row[i]) : 0.f;
        }
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u)
        {
            const uint32_t i = base + u * stride;
            if (i < V && c[u] == c[u] && (idx == 0xffffffffu || c[u] > v))
            {
                v = c[u];
                idx = i;
            }
        }
    }
    cv[warp][lane] = v;
    ci[warp][lane] = idx;
    __syncthreads();
    if (warp != 0)
        return;
    v = -FLT_MAX;
    idx = 0xffffffffu;
    for (uint32_t w = 0; w < nw; ++w) // interleaved indices: ties go to the smaller one
        if (ci[w][lane] != 0xffffffffu && (idx == 0xffffffffu || cv[w][lane] > v || (cv[w][lane] == v && ci[w][lane] < idx)))
        {
            v = cv[w][lane];
            idx = ci[w][lane];
        }
    if (lane < V)
    {
        const float first = __half2float(row[lane]);
        if (first != first || idx == 0xffffffffu)
        {
            v = first;
            idx = lane;
        }
    }
    else
    {
        v = -FLT_MAX;
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
        tok[b] = idx;
        const uint32_t st = *step_ctr;
        if (st < ring_steps)
            ring[(uint64_t)st * B + b] = idx;
        pos[b] += 1;
    }
}

__global__ void k_b_step_done(uint32_t *step_ctr)
{
    *step_ctr += 1;
}

__global__ void k_b_check_pos(const uint32_t *pos, uint32_t cap, uint32_t B, uint32_t *err)
{
    for (uint32_t b = threadIdx.x; b < B; b += blockDim.x)
        if (pos[b] >= cap)
            atomicOr(err, 1u);
}

// B operand of a batch GEMM: W (tile-order copy when tiled == 1), or rows in `group` blocks from
// W, W1, W2 (row-major, the model's matrices) when group > 0.
struct BOp
{
    const __half *W, *W1, *W2;
    uint32_t group;
};

inline BOp bop(const __half *W, const __half *W1 = nullptr, const __half *W2 = nullptr, uint32_t group = 0)
{
    return BOp{W, W1, W2, group};
}

void set_b(GemmArgs &g, const BOp &b, uint32_t tiled)
{
    g.B = b.W;
    g.B1 = b.W1;
    g.B2 = b.W2;
    g.b_group_n = b.group;
    g.b_tiled = b.group ? 0u : (tiled == 1 ? 1u : 0u);
}

bool gemm(const __half *A, const BOp &W, uint32_t tiled, __half *C, uint32_t M, uint32_t N, uint32_t K, int act,
          cudaStream_t s, uint32_t act_from = 0)
{
    GemmArgs g{};
    g.act_from = act_from;
    set_b(g, W, tiled);
    g.pdl = 1;
    g.A = A;
    g.C = C;
    g.M = M;
    g.N = N;
    g.K = K;
    g.lda = K;
    g.ldb = K;
    g.ldc = N;
    g.batch = 1;
    g.batch_c = 1;
    g.scale = 1.0f;
    g.act = act;
    return gemm_tcgen05_launch(g, s);
}

// C = A . W^T as fp32 split-K partials in `part` (no reduction); false when the GEMM cannot split.
bool gemm_partials(const __half *A, const BOp &W, uint32_t tiled, float *part, uint32_t M, uint32_t N, uint32_t K,
                   uint32_t splits, uint32_t *used, cudaStream_t s, uint32_t tile = 0)
{
    GemmArgs g{};
    set_b(g, W, tiled);
    g.pdl = 1;
    g.A = A;
    g.C = nullptr;
    g.M = M;
    g.N = N;
    g.K = K;
    g.lda = K;
    g.ldb = K;
    g.ldc = N;
    g.batch = 1;
    g.batch_c = 1;
    g.scale = 1.0f;
    g.act = 0;
    return gemm_tcgen05_partials(g, s, splits, part, used, tile);
}

// The Wo / down projection with its residual add and the following RMSNORM (gains g) in one pass
// over the rows when the GEMM can split K (bt->proj_splits ways) into bt->part, else the three nodes
// separately.
vkllm_err_t proj_residual_norm(vkllm_b200_batch *bt, const __half *in, const __half *w, uint32_t K, const float *g,
                               cudaStream_t s)
{
    const BatchDims &dd = bt->dd;
    const uint32_t B = bt->B, D = dd.D;
    uint32_t used = 0;
    if (bt->proj_splits > 1 && gemm_partials(in, bop(w), bt->tiled, bt->part, B, D, K, bt->proj_splits, &used, s,
                                             bt->proj_tile))
    {
        // a thread per 8 columns (up to 1024), so each thread's partial loads are issued at once
        const uint32_t threads = std::min(1024u, std::max(64u, (D / 8 + 31) & ~31u));
        k_b_proj_residual_norm<<<B, threads, 0, s>>>(bt->part, used, bt->x, g, D, dd.eps, bt->xn, B);
        return VKLLM_ERR_OK;
    }
    (void)cudaGetLastError();
    if (!gemm(in, bop(w), bt->tiled, bt->t0, B, D, K, 0, s))
        return VKLLM_ERR_VULKAN;
    k_b_bin8<<<grid_1d((uint64_t)B * D / 8, kBT), kBT, 0, s>>>(bt->x, bt->x, bt->t0, (uint64_t)B * D / 8, 0);
    k_b_rmsnorm<<<B, kBT, 0, s>>>(bt->x, g, D, dd.eps, bt->xn);
    return VKLLM_ERR_OK;
}

vkllm_err_t enqueue_batch_step(vkllm_b200_batch *bt, cudaStream_t s)
{
    const BatchDims &dd = bt->dd;
    const uint32_t B = bt->B, D = dd.D, HD = bt->HD, F = dd.F, H = dd.H, hd = dd.hd;
    k_b_check_pos<<<1, 64, 0, s>>>(bt->pos, bt->cap, B, bt->err);
    k_b_embed<<<B, kBT, 0, s>>>(bt->embed, dd.V, D, bt->unk, bt->tok, bt->x);
    uint32_t lpk = 1;
    while (lpk < hd / 8)
        lpk <<= 1;
    const size_t att_smem = (256 + ((bt->cap + 31) & ~31u) + (size_t)(kBT / lpk) * hd) * 4;
    for (uint32_t l = 0; l < bt->L; ++l)
    {
        const BatchLayer &w = bt->layers[l];
        __half *kc = bt->kv + ((uint64_t)l * 2 + 0) * B * H * bt->cap * hd;
        __half *vc = bt->kv + ((uint64_t)l * 2 + 1) * B * H * bt->cap * hd;
        if (l == 0) // later layers get xn from the previous layer's down projection pass
            k_b_rmsnorm<<<B, kBT, 0, s>>>(bt->x, w.attn_norm, D, dd.eps, bt->xn);
        // QKV as split-K partials summed by the RoPE / KV-row kernel (else the GEMM's own reduction)
        uint32_t used = 0;
        const BOp b_qkv = bop(w.wqkv, w.wqkv1, w.wqkv2, w.group_qkv), b_ug = bop(w.wug, w.wug1, nullptr, w.group_ug);
        if (bt->qkv_splits > 1 &&
            gemm_partials(bt->xn, b_qkv, bt->tiled, bt->part, B, 3 * HD, D, bt->qkv_splits, &used, s, bt->qkv_tile))
            k_b_rope_kv_part<<<dim3(H, B), (hd / 2 + 31) / 32 * 32, 0, s>>>(bt->part, used, bt->qkv, HD, bt->pos, H, hd,
                                                                              bt->cap, dd.rope_base, kc, vc, B);
        else
        {
            (void)cudaGetLastError();
            if (!gemm(bt->xn, b_qkv, bt->tiled, bt->qkv, B, 3 * HD, D, 0, s))
                return VKLLM_ERR_VULKAN;
            k_b_rope_kv<<<dim3(H, B), (hd / 2 + 31) / 32 * 32, 0, s>>>(
                bt->qkv, bt->qkv + HD, bt->qkv + 2 * HD, 3 * HD, bt->pos, H, hd, bt->cap, dd.rope_base, kc, vc, B);
        }
        CUtensorMap km, vm;
        if (bt->att_tc && encode_kv_rows_map(&km, kc, hd, bt->cap, H, B, 16) &&
            encode_kv_rows_map(&vm, vc, hd, bt->cap, H, B, 16))
        {
            const size_t smem = att_tc_smem(hd, bt->cap, bt->att_chunk, bt->att_ring);
            auto kern = att_tc_kernel(hd, bt->att_tc);
            kern<<<dim3(H, B), bt->att_tc, smem, s>>>(km, vm, bt->qkv, 3 * HD, kc, vc, bt->pos, H, bt->cap, dd.scale,
                                                      bt->attn, bt->err, bt->att_chunk, bt->att_ring);
        }
        else if (bt->att_staged)
            k_b_attention_staged<<<dim3(H, B), bt->att_staged,
                                   att_staged_smem(hd, bt->cap, bt->att_staged, bt->att_chunk, bt->att_ring), s>>>(
                bt->qkv, 3 * HD, kc, vc, bt->pos, H, hd, bt->cap, dd.scale, bt->attn, bt->err, bt->att_chunk,
                bt->att_ring);
        else
            k_b_attention<<<dim3(H, B), kBT, att_smem, s>>>(bt->qkv, 3 * HD, kc, vc, bt->pos, H, hd, bt->cap, dd.scale,
                                                             bt->attn);
        _CHECK(proj_residual_norm(bt, bt->attn, w.wo_g, HD, w.ffn_norm, s));
        // up/gate as split-K partials summed by the gate kernel (else the GEMM's own reduction, with
        // SiLU on the gate half only)
        if (bt->ug_splits > 1 &&
            gemm_partials(bt->xn, b_ug, bt->tiled, bt->part, B, 2 * F, D, bt->ug_splits, &used, s, bt->ug_tile))
            k_b_gate_part<<<grid_1d((uint64_t)B * F / 8, kBT), kBT, 0, s>>>(bt->m, bt->part, used, F, B);
        else
        {
            (void)cudaGetLastError();
            if (!gemm(bt->xn, b_ug, bt->tiled, bt->ug, B, 2 * F, D, 1, s, F))
                return VKLLM_ERR_VULKAN;
            k_b_gate<<<grid_1d((uint64_t)B * F / 8, kBT), kBT, 0, s>>>(bt->m, bt->ug, F, B);
        }
        // the down projection's pass also norms for the next layer (or the output norm after the last)
        _CHECK(
            proj_residual_norm(bt, bt->m, w.wd_g, F, l + 1 < bt->L ? bt->layers[l + 1].attn_norm : bt->out_norm, s));
    }
    if (!gemm(bt->xn, bop(bt->wout_g), bt->tiled, bt->logits, B, dd.V, D, 0, s))
        return VKLLM_ERR_VULKAN;
    k_b_argmax<<<B, 1024, 0, s>>>(bt->logits, dd.V, bt->tok, bt->pos, bt->ring, bt->ring_steps, bt->err + 1, B);
    k_b_step_done<<<1, 1, 0, s>>>(bt->err + 1);
    return cudaGetLastError() == cudaSuccess ? VKLLM_ERR_OK : VKLLM_ERR_VULKAN;
}

} // namespace
} // namespace vkb

using namespace vkb;

extern "C" vkllm_err_t vkllm_b200_batch_new(struct vkllm_context *ctx, struct vkllm_models_llama2 *model,
                                            uint32_t n_seqs, uint32_t kv_rows, struct vkllm_b200_batch **out)
{
    _CHECK_ARGS(ctx && model && out && n_seqs > 0 && kv_rows > 0);
    _CHECK_ARGS(model->weights.blocks && model->weights.tok_embed_weights && model->weights.output_weight);
    block_weights *b0 = model->weights.blocks->data[0];
    auto *bt = new vkllm_b200_batch();
    bt->ctx = ctx;
    bt->model = model;
    BatchDims &dd = bt->dd;
    dd.D = model->meta.embedding_length;
    dd.H = model->meta.head_count;
    dd.V = model->meta.vocab_size;
    dd.ctx = model->meta.context_length;
    dd.eps = model->meta.layer_norm_rms_epsilon;
    dd.rope_base = model->meta.rope_freq_base;
    bt->HD = b0->WQ->shapes[2];
    dd.hd = bt->HD / dd.H;
    dd.F = b0->WU->shapes[2];
    dd.scale = 1.0f / sqrtf((float)dd.hd);
    bt->B = n_seqs;
    bt->cap = kv_rows < dd.ctx ? kv_rows : dd.ctx;
    bt->L = model->meta.block_count;
    bt->unk = model->meta.padding_token_id;
    bt->host_pos.assign(n_seqs, 0);
    if (dd.D % 8 || dd.F % 8 || bt->HD % 8 || dd.hd > 256 || dd.hd % 8 || bt->cap > 8192 - 256)
    {
        delete bt;
        return VKLLM_ERR_ARGS;
    }
    for (uint32_t l = 0; l < bt->L; ++l)
    {
        block_weights *bw = model->weights.blocks->data[l];
        BatchLayer w{};
        w.wq = (const __half *)dev_ptr(ctx, bw->WQ);
        w.wk = (const __half *)dev_ptr(ctx, bw->WK);
        w.wv = (const __half *)dev_ptr(ctx, bw->WV);
        w.wo = (const __half *)dev_ptr(ctx, bw->WO);
        w.wu = (const __half *)dev_ptr(ctx, bw->WU);
        w.wg = (const __half *)dev_ptr(ctx, bw->WG);
        w.wd = (const __half *)dev_ptr(ctx, bw->WD);
        w.attn_norm = (const float *)dev_ptr(ctx, bw->attn_norm_weight);
        w.ffn_norm = (const float *)dev_ptr(ctx, bw->ffn_norm_weight);
        bt->layers.push_back(w);
    }
    bt->embed = (const __half *)dev_ptr(ctx, model->weights.tok_embed_weights);
    bt->wout = (const __half *)dev_ptr(ctx, model->weights.output_weight);
    bt->out_norm = (const float *)dev_ptr(ctx, model->weights.output_norm_weight);
    const uint32_t B = n_seqs, D = dd.D, HD = bt->HD, F = dd.F;
    bt->ring_steps = 1024;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t kv_bytes = al((size_t)bt->L * 2 * B * dd.H * bt->cap * dd.hd * 2);
    const size_t part_elems = (size_t)B * kMaxPartSplits * std::max({(size_t)D, (size_t)3 * HD, (size_t)2 * F});
    const size_t act = al((size_t)B * D * 2) * 3 + al((size_t)B * 3 * HD * 2) + al((size_t)B * HD * 2) +
                       al((size_t)B * 2 * F * 2) + al((size_t)B * F * 2) + al((size_t)B * dd.V * 2) +
                       al(part_elems * 4);
    const size_t small = al((size_t)B * 4) * 2 + al((size_t)bt->ring_steps * B * 4) + al(16);
    if (cudaMalloc(&bt->ws, kv_bytes + act + small) != cudaSuccess)
    {
        (void)cudaGetLastError();
        delete bt;
        return VKLLM_ERR_ALLOC;
    }
    char *p = (char *)bt->ws;
    auto take = [&](size_t b) {
        char *r = p;
        p += al(b);
        return r;
    };
    bt->kv = (__half *)take(kv_bytes);
    bt->x = (__half *)take((size_t)B * D * 2);
    bt->xn = (__half *)take((size_t)B * D * 2);
    bt->t0 = (__half *)take((size_t)B * D * 2);
    bt->qkv = (__half *)take((size_t)B * 3 * HD * 2);
    bt->attn = (__half *)take((size_t)B * HD * 2);
    bt->ug = (__half *)take((size_t)B * 2 * F * 2);
    bt->m = (__half *)take((size_t)B * F * 2);
    bt->logits = (__half *)take((size_t)B * dd.V * 2);
    bt->part = (float *)take(part_elems * 4);
    bt->tok = (uint32_t *)take((size_t)B * 4);
    bt->pos = (uint32_t *)take((size_t)B * 4);
    bt->ring = (uint32_t *)take((size_t)bt->ring_steps * B * 4);
    bt->err = (uint32_t *)take(16); // [0] error bits, [1] step counter
    cudaStream_t s = ctx->runtime->stream;
    // GEMM operand copies, per layer [Wq; Wk; Wv] then [Wup; Wgate] (then Wo and Wdown when tiled)
    const char *att_env = getenv("VKLLM_B200_BATCH_ATT_STAGED");
    bt->att_staged = att_env ? (uint32_t)atoi(att_env) : 256u;
    // VKLLM_B200_BATCH_ATT_TC = 0 selects the FMA kernels below instead of the tensor-core attention
    // (which needs hd 64 or 128 and whole 16-row key blocks per chunk), 128 / 256 its threads per CTA.
    // 7B, 64 sequences, one box (chunk / ring / threads): 48/2/128 4.733, 64/2/128 4.810, 32/3/128
    // 4.818, 64/2/256 4.849-4.865 ms per step; the FMA kernel 64/2/256 4.862.
    const char *tc_env = getenv("VKLLM_B200_BATCH_ATT_TC");
    bt->att_tc = tc_env ? (uint32_t)atoi(tc_env) : kAttTcThreads;
    if (bt->att_tc != 128 && bt->att_tc != 256)
        bt->att_tc = 0;
    const bool tc_shape = dd.hd == 64 || dd.hd == 128;
    const uint32_t chunk_default = bt->att_tc && tc_shape ? kAttTcChunk : kAttChunk;
    const char *chunk_env = getenv("VKLLM_B200_BATCH_ATT_CHUNK"), *ring_env = getenv("VKLLM_B200_BATCH_ATT_RING");
    bt->att_chunk = chunk_env ? (uint32_t)atoi(chunk_env) : chunk_default;
    bt->att_ring = ring_env ? (uint32_t)atoi(ring_env) : kAttStages;
    if (bt->att_chunk < 8 || bt->att_chunk > 256 || bt->att_chunk % 8 || bt->att_ring < 2 || bt->att_ring > kAttMaxStages)
    {
        bt->att_chunk = chunk_default;
        bt->att_ring = kAttStages;
    }
    if (!(bt->att_staged == 128 || bt->att_staged == 256 || bt->att_staged == 512) || dd.hd % 8 || dd.hd > 128 ||
        att_staged_smem(dd.hd, bt->cap, bt->att_staged, bt->att_chunk, bt->att_ring) > 200 * 1024)
        bt->att_staged = 0;
    if (!tc_shape || bt->att_chunk % 16 ||
        att_tc_smem(dd.hd, bt->cap, bt->att_chunk, bt->att_ring) > 200 * 1024)
        bt->att_tc = 0;
    // VKLLM_B200_BATCH_GEMM="qs,us,ps,qt,ut,pt": K splits (1..4) and tiles (0: 128 x 128, 1: 128 x 256;
    // 2, 3: the same loading 64 rows of A per stage, for up to 64 sequences) of the QKV, up/gate
    // and Wo / down GEMMs (defaults 3,3,4,1,1,0; 7B, 64 sequences: 2,3,4 / 3,3,4 / 4,3,4 / 3,2,4 splits
    // 4.966 / 4.936 / 5.223 / 5.108 ms per step). Up to 8 sequences the tiles that stage 64 rows of A
    // keep one more weight stage in flight: 8 sequences 3.52 against 3.74 ms per step (16: 3.66
    // against 3.63, 64: 4.93 against 4.87, so not there).
    if (B <= 8)
        bt->qkv_tile = 3, bt->ug_tile = 3, bt->proj_tile = 2;
    if (const char *ge = getenv("VKLLM_B200_BATCH_GEMM"))
    {
        unsigned v[6];
        if (sscanf(ge, "%u,%u,%u,%u,%u,%u", &v[0], &v[1], &v[2], &v[3], &v[4], &v[5]) == 6 && v[0] >= 1 &&
            v[0] <= kMaxPartSplits && v[1] >= 1 && v[1] <= kMaxPartSplits && v[2] >= 1 && v[2] <= kMaxPartSplits &&
            v[3] <= 3 && v[4] <= 3 && v[5] <= 3)
        {
            bt->qkv_splits = v[0], bt->ug_splits = v[1], bt->proj_splits = v[2];
            bt->qkv_tile = v[3], bt->ug_tile = v[4], bt->proj_tile = v[5];
        }
    }
    // VKLLM_B200_BATCH_TILED: 1 (default) tile-order copies, 2 the model's matrices in place (grouped
    // B operands; HD and F multiples of 32), 0 row-major concatenated copies.
    const char *tiled_env = getenv("VKLLM_B200_BATCH_TILED");
    bt->tiled = tiled_env ? (uint32_t)atoi(tiled_env) : 1u;
    if (bt->tiled > 2 || (bt->tiled == 2 && (HD % 32 != 0 || F % 32 != 0)))
        bt->tiled = 1;
    const size_t t_qkv = gemm_tiled_b_elems(3 * HD, D), t_ug = gemm_tiled_b_elems(2 * F, D),
                 t_wo = gemm_tiled_b_elems(D, HD), t_wd = gemm_tiled_b_elems(D, F);
    const size_t per_layer = bt->tiled == 1   ? t_qkv + t_ug + t_wo + t_wd
                             : bt->tiled == 0 ? ((size_t)3 * HD + (size_t)2 * F) * D
                                              : 0;
    const size_t extra = bt->tiled == 1 ? gemm_tiled_b_elems(dd.V, D) : 0;
    if (per_layer + extra > 0 && cudaMalloc(&bt->wcat, (per_layer * bt->L + extra) * sizeof(__half)) != cudaSuccess)
    {
        (void)cudaGetLastError();
        cudaFree(bt->ws);
        delete bt;
        return VKLLM_ERR_ALLOC;
    }
    bool copied = true;
    for (uint32_t l = 0; l < bt->L && copied; ++l)
    {
        BatchLayer &w = bt->layers[l];
        if (bt->tiled == 2)
        {
            w.wqkv = w.wq;
            w.wqkv1 = w.wk;
            w.wqkv2 = w.wv;
            w.group_qkv = HD;
            w.wug = w.wu;
            w.wug1 = w.wg;
            w.group_ug = F;
            w.wo_g = w.wo;
            w.wd_g = w.wd;
            continue;
        }
        __half *qkv = bt->wcat + per_layer * l;
        if (bt->tiled == 1)
        {
            __half *ug = qkv + t_qkv, *wo = ug + t_ug, *wd = wo + t_wo;
            copied = gemm_tile_b(TileSrcs{{w.wq, w.wk, w.wv}, {HD, HD, HD}, 3}, D, qkv, s) &&
                     gemm_tile_b(TileSrcs{{w.wu, w.wg}, {F, F}, 2}, D, ug, s) &&
                     gemm_tile_b(TileSrcs{{w.wo}, {D}, 1}, HD, wo, s) && gemm_tile_b(TileSrcs{{w.wd}, {D}, 1}, F, wd, s);
            w.wqkv = qkv;
            w.wug = ug;
            w.wo_g = wo;
            w.wd_g = wd;
            continue;
        }
        __half *ug = qkv + (size_t)3 * HD * D;
        const size_t mat = (size_t)HD * D * sizeof(__half), fm = (size_t)F * D * sizeof(__half);
        copied = cudaMemcpyAsync(qkv, w.wq, mat, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(qkv + (size_t)HD * D, w.wk, mat, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(qkv + (size_t)2 * HD * D, w.wv, mat, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(ug, w.wu, fm, cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(ug + (size_t)F * D, w.wg, fm, cudaMemcpyDeviceToDevice, s) == cudaSuccess;
        w.wqkv = qkv;
        w.wug = ug;
        w.wo_g = w.wo;
        w.wd_g = w.wd;
    }
    if (bt->tiled == 1)
    {
        __half *wo = bt->wcat + per_layer * bt->L;
        copied = copied && gemm_tile_b(TileSrcs{{bt->wout}, {dd.V}, 1}, D, wo, s);
        bt->wout_g = wo;
    }
    else
        bt->wout_g = bt->wout;
    if (!copied || cudaMemsetAsync(bt->ws, 0, kv_bytes + act + small, s) != cudaSuccess ||
        cudaFuncSetAttribute(k_b_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024) != cudaSuccess ||
        (bt->att_tc && cudaFuncSetAttribute(att_tc_kernel(dd.hd, bt->att_tc),
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)att_tc_smem(dd.hd, bt->cap, bt->att_chunk, bt->att_ring)) != cudaSuccess) ||
        (bt->att_staged && cudaFuncSetAttribute(k_b_attention_staged, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)att_staged_smem(dd.hd, bt->cap, bt->att_staged, bt->att_chunk,
                                                                     bt->att_ring)) != cudaSuccess) ||
        cudaStreamSynchronize(s) != cudaSuccess)
    {
        (void)cudaGetLastError();
        cudaFree(bt->ws);
        cudaFree(bt->wcat);
        delete bt;
        return VKLLM_ERR_VULKAN;
    }
    *out = bt;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_batch_load_sequence(struct vkllm_context *ctx, struct vkllm_b200_batch *bt,
                                                      uint32_t seq, uint32_t next_token, uint32_t n_rows)
{
    _CHECK_ARGS(ctx && bt && seq < bt->B && n_rows < bt->cap && n_rows <= bt->dd.ctx);
    vkllm_kvcache *kv = bt->model->weights.kvcache;
    _CHECK_ARGS(kv && kv->kcaches && kv->vcaches);
    cudaStream_t s = ctx->runtime->stream;
    const BatchDims &dd = bt->dd;
    const size_t row = (size_t)dd.hd * 2;
    for (uint32_t l = 0; l < bt->L; ++l)
        for (int which = 0; which < 2; ++which)
        {
            const __half *src = (const __half *)dev_ptr(ctx, which == 0 ? kv->kcaches->data[l] : kv->vcaches->data[l]);
            __half *dst = bt->kv + (((uint64_t)l * 2 + which) * bt->B + seq) * dd.H * bt->cap * dd.hd;
            if (n_rows > 0)
                VKB_CUDA(cudaMemcpy2DAsync(dst, bt->cap * row, src, (size_t)dd.ctx * row, n_rows * row, dd.H,
                                           cudaMemcpyDeviceToDevice, s));
        }
    VKB_CUDA(cudaMemcpyAsync(bt->tok + seq, &next_token, 4, cudaMemcpyHostToDevice, s));
    VKB_CUDA(cudaMemcpyAsync(bt->pos + seq, &n_rows, 4, cudaMemcpyHostToDevice, s));
    VKB_CUDA(cudaStreamSynchronize(s));
    bt->host_pos[seq] = n_rows;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_batch_decode_steps(struct vkllm_context *ctx, struct vkllm_b200_batch *bt,
                                                     uint32_t n_steps)
{
    _CHECK_ARGS(ctx && bt && n_steps <= bt->ring_steps);
    for (uint32_t b = 0; b < bt->B; ++b)
        if (bt->host_pos[b] + n_steps > bt->cap)
        {
            log_error("batched decode: sequence %u would pass its %u KV rows", b, bt->cap);
            return VKLLM_ERR_ARGS;
        }
    cudaStream_t s = ctx->runtime->stream;
    const uint32_t total = n_steps;
    VKB_CUDA(cudaMemsetAsync(bt->err, 0, 8, s));
    if (!bt->exec && n_steps > 0)
    {
        // First step eagerly (first-use allocations of the GEMM: kernel attributes, split-K workspace),
        // then capture one step as a graph for the rest.
        _CHECK(enqueue_batch_step(bt, s));
        n_steps -= 1;
        cudaStream_t cs;
        VKB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
        VKB_CUDA(cudaStreamSynchronize(s));
        vkllm_err_t err = VKLLM_ERR_OK;
        if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            err = VKLLM_ERR_VULKAN;
        if (err == VKLLM_ERR_OK)
        {
            vkllm_err_t le = enqueue_batch_step(bt, cs);
            if (cudaStreamEndCapture(cs, &bt->graph) != cudaSuccess || le != VKLLM_ERR_OK)
                err = VKLLM_ERR_VULKAN;
        }
        if (err == VKLLM_ERR_OK && cudaGraphInstantiate(&bt->exec, bt->graph, 0) != cudaSuccess)
            err = VKLLM_ERR_VULKAN;
        cudaStreamDestroy(cs);
        if (err != VKLLM_ERR_OK)
        {
            (void)cudaGetLastError();
            return err;
        }
    }
    for (uint32_t i = 0; i < n_steps; ++i)
        VKB_CUDA(cudaGraphLaunch(bt->exec, s));
    bt->last_steps = total;
    for (uint32_t b = 0; b < bt->B; ++b)
        bt->host_pos[b] += total;
    uint32_t e[2] = {0, 0};
    VKB_CUDA(cudaMemcpyAsync(e, bt->err, 8, cudaMemcpyDeviceToHost, s));
    VKB_CUDA(cudaStreamSynchronize(s));
    if (e[0] != 0 || gemm_tcgen05_error(ctx->device->ordinal) != 0)
    {
        log_error("batched decode: %s", (e[0] & 1u)                ? "a sequence reached its KV capacity"
                                        : (e[0] & kErrAttTimeout) ? "an attention copy wait expired"
                                                                  : "tensor-core GEMM wait expired");
        return VKLLM_ERR_ARGS;
    }
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_batch_read_tokens(struct vkllm_context *ctx, struct vkllm_b200_batch *bt,
                                                    uint32_t *out, uint32_t n_steps)
{
    _CHECK_ARGS(ctx && bt && out && n_steps <= bt->ring_steps);
    VKB_CUDA(cudaMemcpy(out, bt->ring, (size_t)n_steps * bt->B * 4, cudaMemcpyDeviceToHost));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_batch_read_logits(struct vkllm_context *ctx, struct vkllm_b200_batch *bt,
                                                    uint16_t *out)
{
    _CHECK_ARGS(ctx && bt && out);
    VKB_CUDA(cudaMemcpy(out, bt->logits, (size_t)bt->B * bt->dd.V * 2, cudaMemcpyDeviceToHost));
    return VKLLM_ERR_OK;
}

extern "C" void vkllm_b200_batch_free(struct vkllm_context *ctx, struct vkllm_b200_batch *bt)
{
    (void)ctx;
    if (!bt)
        return;
    if (bt->exec)
        cudaGraphExecDestroy(bt->exec);
    if (bt->graph)
        cudaGraphDestroy(bt->graph);
    if (bt->ws)
    {
        cudaDeviceSynchronize();
        cudaFree(bt->ws);
    }
    if (bt->wcat)
        cudaFree(bt->wcat);
    delete bt;
}
