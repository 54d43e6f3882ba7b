// Kernels of the fused prefill step (a llama2 graph with S > 1 tokens; the host side is
// prefill_run in engine.cu). They compute the nodes of src/models/vkllm_llama2_layers.c:98-340 for
// a block of S tokens at positions p0 .. p0 + S - 1, rounding to fp16 where the reference graph
// materialises a node:
//   k_pf_embed       EMBEDDING (src/shaders/vkllm_embedding.comp:41-70, ids >= V -> unk)
//   k_pf_rope_kv     ROPE of Q and K (src/shaders/vkllm_rope.comp:39-79, normal style) and the two
//                    UPDATE_ROWS of the KV cache (src/models/vkllm_kvcache.c:65-102)
//   k_pf_attention   scores MATMUL (scale 1/sqrt(hd)), SOFTMAX with the causal mask and the max over
//                    every entry of the row, masked ones included (src/shaders/vkllm_softmax.comp:
//                    42-96), probs . V MATMUL, and the COPY that lays heads side by side
//                    (src/models/vkllm_llama2_layers.c:223-281), in one pass over the cache with
//                    tensor-core tiles (mma.sync m16n8k16: fp16 operands, fp32 accumulation).
#pragma once

#include <cfloat>
#include <cuda_fp16.h>
#include <cstdint>

namespace vkb
{

// x[s][:] = table[id_s][:] (id >= V -> unk), 16 bytes per thread.
__global__ void k_pf_embed(const uint32_t *__restrict__ ids, const __half *__restrict__ table, uint32_t V,
                           uint32_t D, uint32_t unk, __half *__restrict__ x)
{
    const uint32_t s = blockIdx.x;
    uint32_t id = ids[s];
    if (id >= V)
        id = unk < V ? unk : 0; // an unk id outside the table would read past it; row 0 instead
    const uint4 *src = reinterpret_cast<const uint4 *>(table + (uint64_t)id * D);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (uint64_t)s * D);
    for (uint32_t i = threadIdx.x; i < D / 8; i += blockDim.x)
        dst[i] = src[i];
}

// RoPE of Q and K and the KV-cache rows. q, k, v: [S][H * hd] rows `ld` elements apart (the
// projection nodes, side by side when one grouped GEMM produced them). Writes
// rq [H][S][hd] (the rotated-Q node, contiguous as the reference's ROPE output), the rotated K rows
// to kcache[h][p0 + s] and the V rows to vcache[h][p0 + s]. Pair w of a row rotates by
// theta = (p0 + s) / base^(2w / hd) in fp32. One thread per 8 elements (4 pairs).
__global__ void k_pf_rope_kv(const __half *__restrict__ q, const __half *__restrict__ k, const __half *__restrict__ v,
                             uint32_t ld, uint32_t S, uint32_t H, uint32_t hd, uint32_t p0, uint32_t ctx, float base,
                             __half *__restrict__ rq, __half *__restrict__ kcache, __half *__restrict__ vcache)
{
    const uint32_t per_row = H * hd / 8;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)S * per_row)
        return;
    const uint32_t s = (uint32_t)(t / per_row), c8 = (uint32_t)(t % per_row);
    const uint32_t col = 8 * c8, h = col / hd, d = col % hd;
    const uint64_t src = (uint64_t)s * ld + col;
    const uint4 qv = *reinterpret_cast<const uint4 *>(q + src);
    const uint4 kv = *reinterpret_cast<const uint4 *>(k + src);
    const __half2 *qh = reinterpret_cast<const __half2 *>(&qv);
    const __half2 *kh = reinterpret_cast<const __half2 *>(&kv);
    uint4 qo, ko;
    __half2 *qoh = reinterpret_cast<__half2 *>(&qo);
    __half2 *koh = reinterpret_cast<__half2 *>(&ko);
    const float pos = (float)(p0 + s);
#pragma unroll
    for (int e = 0; e < 4; ++e)
    {
        const uint32_t w = d / 2 + (uint32_t)e;
        const float theta = pos / powf(base, (float)(2 * w) / (float)hd);
        const float cs = cosf(theta), sn = sinf(theta);
        const float2 a = __half22float2(qh[e]), b = __half22float2(kh[e]);
        qoh[e] = __floats2half2_rn(cs * a.x - sn * a.y, sn * a.x + cs * a.y);
        koh[e] = __floats2half2_rn(cs * b.x - sn * b.y, sn * b.x + cs * b.y);
    }
    *reinterpret_cast<uint4 *>(rq + ((uint64_t)h * S + s) * hd + d) = qo;
    const uint64_t row = ((uint64_t)h * ctx + p0 + s) * hd + d;
    *reinterpret_cast<uint4 *>(kcache + row) = ko;
    *reinterpret_cast<uint4 *>(vcache + row) = *reinterpret_cast<const uint4 *>(v + src);
}

// m[s][f] = fp16(up[s][f] * gate[s][f]) (the FFN's BIN mul node); up and gate rows `ld` elements
// apart, m dense [S][F]. 8 elements per thread.
__global__ void k_pf_gate_mul(const __half *__restrict__ up, const __half *__restrict__ gate, uint32_t ld, uint32_t S,
                              uint32_t F, __half *__restrict__ m)
{
    const uint32_t per_row = F / 8;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)S * per_row)
        return;
    const uint32_t s = (uint32_t)(t / per_row), c = 8 * (uint32_t)(t % per_row);
    const uint4 a = *reinterpret_cast<const uint4 *>(up + (uint64_t)s * ld + c);
    const uint4 b = *reinterpret_cast<const uint4 *>(gate + (uint64_t)s * ld + c);
    const __half2 *ah = reinterpret_cast<const __half2 *>(&a), *bh = reinterpret_cast<const __half2 *>(&b);
    uint4 o;
    __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e)
    {
        const float2 x = __half22float2(ah[e]), y = __half22float2(bh[e]);
        oh[e] = __floats2half2_rn(x.x * y.x, x.y * y.y);
    }
    *reinterpret_cast<uint4 *>(m + (uint64_t)s * F + c) = o;
}

__device__ __forceinline__ uint32_t pf_smem(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void pf_ldsm4(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void pf_ldsm4_t(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

// c += A (16 x 16, row) . B (16 x 8, col), fp16 operands, fp32 accumulation.
__device__ __forceinline__ void pf_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pf_pack(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float pf_round16(float x)
{
    return __half2float(__float2half_rn(x));
}

constexpr int kPfBQ = 64;      // query rows per CTA (16 per warp)
constexpr int kPfBK = 64;      // keys per block
constexpr int kPfThreads = 128;

template <int HD> struct PfSmem
{
    static constexpr int LD = HD + 8;        // halves per Q/K/V smem row (16-byte pad: conflict-free ldmatrix)
    static constexpr int LDT = kPfBK + 8;    // halves per row of the transposed-V tile (quirk Q1)
    static constexpr int kQ = kPfBQ * LD, kK = kPfBK * LD;
    static constexpr int kV = (kPfBK * LD > HD * LDT) ? kPfBK * LD : HD * LDT;
    // [Q tile, later value buffer 1 | key buffer 0 | key buffer 1 | value buffer 0]: the Q tile is read
    // into registers before the first value tile is issued, so its space serves as value buffer 1
    // (three CTAs per SM fit at HD = 128)
    static constexpr int kQV = kQ > kV ? kQ : kV;
    static constexpr int kBytes = (kQV + 2 * kK + kV) * 2;
};

// Loads rows [r0, r0 + rows) (of `n_valid` existing rows) of a [*, HD] fp16 matrix with row pitch
// `pitch` into smem rows of LD halves; missing rows are zero.
template <int HD, int LD>
__device__ __forceinline__ void pf_load_rows(__half *dst, const __half *src, uint64_t pitch, uint32_t r0,
                                             uint32_t rows, uint32_t n_valid)
{
    constexpr uint32_t C8 = HD / 8;
    for (uint32_t i = threadIdx.x; i < rows * C8; i += kPfThreads)
    {
        const uint32_t r = i / C8, c = i % C8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r0 + r < n_valid)
            v = *reinterpret_cast<const uint4 *>(src + (uint64_t)(r0 + r) * pitch + 8 * c);
        *reinterpret_cast<uint4 *>(dst + r * LD + 8 * c) = v;
    }
}

// 16-byte asynchronous copy global -> shared; `valid` false writes zeros (src is then not read).
__device__ __forceinline__ void pf_cp16(__half *dst, const __half *src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(pf_smem(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void pf_cp_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N> __device__ __forceinline__ void pf_cp_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// pf_load_rows as asynchronous copies (committed by the caller).
template <int HD, int LD>
__device__ __forceinline__ void pf_async_rows(__half *dst, const __half *src, uint64_t pitch, uint32_t r0,
                                              uint32_t rows, uint32_t n_valid)
{
    constexpr uint32_t C8 = HD / 8;
    for (uint32_t i = threadIdx.x; i < rows * C8; i += kPfThreads)
    {
        const uint32_t r = i / C8, c = i % C8;
        const bool valid = r0 + r < n_valid;
        pf_cp16(dst + r * LD + 8 * c, valid ? src + (uint64_t)(r0 + r) * pitch + 8 * c : src, valid);
    }
}

// Quirk Q1 V tile: dst[w][jj] = V row w (w < HD), column j0 + jj (< HD), rows LDT halves apart.
template <int HD, int LDT>
__device__ __forceinline__ void pf_async_vt(__half *dst, const __half *vb, uint32_t j0)
{
    for (uint32_t t = threadIdx.x; t < (uint32_t)HD * (kPfBK / 8); t += kPfThreads)
    {
        const uint32_t w = t / (kPfBK / 8), c8 = t % (kPfBK / 8), col = j0 + 8 * c8;
        const bool valid = col < (uint32_t)HD;
        pf_cp16(dst + w * LDT + 8 * c8, valid ? vb + (uint64_t)w * HD + col : vb, valid);
    }
}

// Scores of this warp's 16 query rows against the 64 keys of the block in `sk`:
// s[nt][e] for rows g (e = 0, 1) and g + 8 (e = 2, 3), keys nt * 8 + 2c + (e & 1), where g = lane / 4
// and c = lane % 4; each score rounded to fp16 after the scale (the scores node).
template <int HD, int LD>
__device__ __forceinline__ void pf_scores(const uint32_t (&qa)[HD / 16][4], const __half *sk, float scale,
                                          float (&s)[kPfBK / 8][4])
{
    const uint32_t lane = threadIdx.x & 31;
#pragma unroll
    for (int nt = 0; nt < kPfBK / 8; ++nt)
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    // ldmatrix x4 of K rows (keys) n0 .. n0 + 15 at d k0 .. k0 + 15: b0, b1 of key tiles n0 and n0 + 8
    const uint32_t krow = (lane & 7) + ((lane >> 4) << 3), kcol = ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks)
    {
#pragma unroll
        for (int np = 0; np < kPfBK / 16; ++np)
        {
            uint32_t b[4];
            pf_ldsm4(pf_smem(sk + (np * 16 + krow) * LD + ks * 16 + kcol), b);
            pf_mma(s[2 * np], qa[ks], b[0], b[1]);
            pf_mma(s[2 * np + 1], qa[ks], b[2], b[3]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < kPfBK / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            s[nt][e] = pf_round16(s[nt][e] * scale);
}

// Cluster helpers of the CTA-pair form of k_pf_attention: this CTA's rank in its cluster, a barrier
// over the cluster (release / acquire), and a float load from the peer CTA's shared memory.
__device__ __forceinline__ uint32_t pf_cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void pf_cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float pf_peer_ld(const float *local, uint32_t peer)
{
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(pf_smem(local)), "r"(peer));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// Attention of one head over keys 0 .. Lk - 1 (Lk = p0 + S) for query rows q0 .. q0 + 63 of the S new
// tokens, in two passes over the cache: (1) scores of every key block to get each row's max over
// all Lk entries (masked ones included, as the reference shader) and its sum of exp(s - max) over
// the unmasked ones (keys j <= p0 + i), (2) the same scores again, p = fp16(exp(s - max) / sum) (0
// where masked), and p . V summed in fp32; the result rounded to fp16 into out[s][h * HD + d].
// When Lk == HD the reference's shape-only predicate reads the V slice as [HD, Lk]
// (src/core/vkllm_op_matmul.c:14-30): the product is then out[i][w] = sum_j p_ij V[w][j].
// PAIR: a cluster of two CTAs shares the query tile, CTA r taking the key blocks b with b % 2 == r in
// both passes; they combine their row statistics (max, then the sums rescaled to it) and then their
// fp32 partial outputs through distributed shared memory, and CTA 0 stores the rows. Twice the CTAs
// (and half the serial key blocks per CTA) for the same work; only fp32 summation orders change.
template <int HD, bool PAIR>
__global__ void __launch_bounds__(kPfThreads, HD == 128 ? 3 : 2) k_pf_attention(const __half *__restrict__ rq, const __half *__restrict__ kc,
                                                             const __half *__restrict__ vc, uint32_t ctx, uint32_t S,
                                                             uint32_t p0, uint32_t H, float scale,
                                                             __half *__restrict__ out)
{
    using SM = PfSmem<HD>;
    constexpr int LD = SM::LD, LDT = SM::LDT;
    constexpr uint32_t step = PAIR ? 2u : 1u;
    extern __shared__ __align__(16) unsigned char pf_sm[];
    __shared__ float st_m[kPfBQ], st_l[kPfBQ]; // PAIR: this CTA's row statistics for the peer
    __half *sq = reinterpret_cast<__half *>(pf_sm);
    // key buffer b at sk0 + b * kK; value buffer 0 at sv0, value buffer 1 where the Q tile was
    __half *const sk0 = sq + SM::kQV, *const sv0 = sq + SM::kQV + 2 * SM::kK;
    const uint32_t r = PAIR ? pf_cluster_rank() : 0u;
    // heaviest query tiles (most unmasked key blocks) first: with twice the CTAs the grid exceeds one
    // wave, and the tail should hold the light ones
    const uint32_t h = blockIdx.y,
                   q0 = (PAIR ? (gridDim.x >> 1) - 1 - (blockIdx.x >> 1) : blockIdx.x) * kPfBQ;
    const uint32_t Lk = p0 + S;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const bool q1 = Lk == (uint32_t)HD;
    const __half *kb = kc + (uint64_t)h * ctx * HD, *vb = vc + (uint64_t)h * ctx * HD;

    pf_load_rows<HD, LD>(sq, rq + (uint64_t)h * S * HD, HD, q0, kPfBQ, S);
    __syncthreads();
    uint32_t qa[HD / 16][4];
    {
        const uint32_t arow = 16 * warp + (lane & 15), acol = (lane >> 4) * 8;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
            pf_ldsm4(pf_smem(sq + arow * LD + ks * 16 + acol), qa[ks]);
    }
    // rows of this thread (of the S new tokens): i0 = q0 + 16 warp + g, i1 = i0 + 8
    const uint32_t i0 = q0 + 16 * warp + g, i1 = i0 + 8;
    float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;
    const uint32_t nkb = (Lk + kPfBK - 1) / kPfBK;
    // this CTA's key blocks: r, r + step, ...
    const uint32_t nb1 = nkb > r ? (nkb - r + step - 1) / step : 0u;
    float s[kPfBK / 8][4];

    // ---- pass 1: row max over every key, row sum over the unmasked keys (rescaled online). Key
    // tiles are double-buffered: the next block is in flight while one is scored.
    if (nb1 > 0)
    {
        pf_async_rows<HD, LD>(sk0, kb, HD, r * kPfBK, kPfBK, Lk);
        pf_cp_commit();
    }
    for (uint32_t it = 0; it < nb1; ++it)
    {
        const uint32_t j0 = (r + it * step) * kPfBK;
        if (it + 1 < nb1)
        {
            pf_async_rows<HD, LD>(sk0 + ((it + 1) & 1) * SM::kK, kb, HD, j0 + step * kPfBK, kPfBK, Lk);
            pf_cp_commit();
            pf_cp_wait<1>();
        }
        else
            pf_cp_wait<0>();
        __syncthreads();
        pf_scores<HD, LD>(qa, sk0 + (it & 1) * SM::kK, scale, s);
        float bm0 = -FLT_MAX, bm1 = -FLT_MAX;
#pragma unroll
        for (int nt = 0; nt < kPfBK / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
            {
                const uint32_t j = j0 + nt * 8 + 2 * c + e;
                if (j < Lk)
                {
                    bm0 = fmaxf(bm0, s[nt][e]);
                    bm1 = fmaxf(bm1, s[nt][2 + e]);
                }
            }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1)
        {
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, o));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, o));
        }
        const float n0 = fmaxf(m0, bm0), n1 = fmaxf(m1, bm1);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < kPfBK / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
            {
                const uint32_t j = j0 + nt * 8 + 2 * c + e;
                if (j <= p0 + i0)
                    a0 += expf(s[nt][e] - n0);
                if (j <= p0 + i1)
                    a1 += expf(s[nt][2 + e] - n1);
            }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1)
        {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        }
        l0 = l0 * expf(m0 - n0) + a0;
        l1 = l1 * expf(m1 - n1) + a1;
        m0 = n0;
        m1 = n1;
        __syncthreads(); // every warp is done with this buffer before it is refilled
    }

    if constexpr (PAIR)
    {
        // the pair's row statistics: max of the two, sums rescaled to it (the same bits in both CTAs:
        // fp32 addition commutes)
        if (c == 0)
        {
            st_m[16 * warp + g] = m0;
            st_l[16 * warp + g] = l0;
            st_m[16 * warp + g + 8] = m1;
            st_l[16 * warp + g + 8] = l1;
        }
        pf_cluster_sync();
        const float pm0 = pf_peer_ld(&st_m[16 * warp + g], r ^ 1u), pl0 = pf_peer_ld(&st_l[16 * warp + g], r ^ 1u);
        const float pm1 = pf_peer_ld(&st_m[16 * warp + g + 8], r ^ 1u),
                    pl1 = pf_peer_ld(&st_l[16 * warp + g + 8], r ^ 1u);
        const float M0 = fmaxf(m0, pm0), M1 = fmaxf(m1, pm1);
        l0 = l0 * expf(m0 - M0) + pl0 * expf(pm0 - M0);
        l1 = l1 * expf(m1 - M1) + pl1 * expf(pm1 - M1);
        m0 = M0;
        m1 = M1;
    }

    // ---- pass 2: probabilities and p . V over this CTA's key blocks that hold an unmasked key
    float o[HD / 8][4];
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt)
        o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    const uint32_t last_row = min(q0 + kPfBQ, S) - 1;
    const uint32_t nkb2 = min(nkb, (p0 + last_row) / kPfBK + 1);
    const uint32_t nb2 = nkb2 > r ? (nkb2 - r + step - 1) / step : 0u;
    // K and V tiles of the next block are in flight while one is used (buffer = iteration parity)
    auto issue_kv = [&](uint32_t blk, uint32_t buf) {
        const uint32_t jb = blk * kPfBK;
        pf_async_rows<HD, LD>(sk0 + buf * SM::kK, kb, HD, jb, kPfBK, Lk);
        if (!q1)
            pf_async_rows<HD, LD>((buf ? sq : sv0), vb, HD, jb, kPfBK, Lk);
        else
            pf_async_vt<HD, LDT>((buf ? sq : sv0), vb, jb);
        pf_cp_commit();
    };
    if (nb2 > 0)
        issue_kv(r, 0);
    for (uint32_t it = 0; it < nb2; ++it)
    {
        const uint32_t j0 = (r + it * step) * kPfBK;
        if (it + 1 < nb2)
        {
            issue_kv(r + (it + 1) * step, (it + 1) & 1);
            pf_cp_wait<1>();
        }
        else
            pf_cp_wait<0>();
        __syncthreads();
        const __half *sk = sk0 + (it & 1) * SM::kK, *sv = ((it & 1) ? sq : sv0);
        pf_scores<HD, LD>(qa, sk, scale, s);
        // p = fp16(exp(s - max) / sum) where unmasked, else 0 (the softmax node)
#pragma unroll
        for (int nt = 0; nt < kPfBK / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
            {
                const uint32_t j = j0 + nt * 8 + 2 * c + e;
                s[nt][e] = j <= p0 + i0 ? pf_round16(expf(s[nt][e] - m0) / l0) : 0.f;
                s[nt][2 + e] = j <= p0 + i1 ? pf_round16(expf(s[nt][2 + e] - m1) / l1) : 0.f;
            }
        // p as the A operand: key tiles 2t and 2t + 1 form k-step t
#pragma unroll
        for (int t = 0; t < kPfBK / 16; ++t)
        {
            uint32_t pa[4];
            pa[0] = pf_pack(s[2 * t][0], s[2 * t][1]);
            pa[1] = pf_pack(s[2 * t][2], s[2 * t][3]);
            pa[2] = pf_pack(s[2 * t + 1][0], s[2 * t + 1][1]);
            pa[3] = pf_pack(s[2 * t + 1][2], s[2 * t + 1][3]);
#pragma unroll
            for (int np = 0; np < HD / 16; ++np)
            {
                uint32_t b[4];
                if (!q1)
                {
                    // V rows (keys) 16t .. 16t + 15 at d 16np .. 16np + 15, transposed: b0, b1 of d tiles
                    const uint32_t vrow = 16 * t + (lane & 7) + ((lane >> 3) & 1) * 8, vcol = 16 * np + (lane >> 4) * 8;
                    pf_ldsm4_t(pf_smem(sv + vrow * LD + vcol), b);
                }
                else
                {
                    // rows w = 16np .. 16np + 15 of sv, keys 16t .. 16t + 15 (already K-contiguous)
                    const uint32_t wrow = 16 * np + (lane & 7) + ((lane >> 4) << 3), kcol = 16 * t + ((lane >> 3) & 1) * 8;
                    pf_ldsm4(pf_smem(sv + wrow * LDT + kcol), b);
                }
                pf_mma(o[2 * np], pa, b[0], b[1]);
                pf_mma(o[2 * np + 1], pa, b[2], b[3]);
            }
        }
        __syncthreads(); // every warp is done with these buffers before they are refilled
    }
    if constexpr (PAIR)
    {
        // CTA 1 publishes its fp32 partial rows (in the K buffers, free after the loop's last barrier);
        // CTA 0 adds them to its own and stores; the last barrier keeps CTA 1's shared memory alive
        // until CTA 0 has read it
        float *so = reinterpret_cast<float *>(sk0); // [64][HD]
        if (r == 1)
        {
#pragma unroll
            for (int nt = 0; nt < HD / 8; ++nt)
            {
                const uint32_t d = nt * 8 + 2 * c;
                so[(16 * warp + g) * HD + d] = o[nt][0];
                so[(16 * warp + g) * HD + d + 1] = o[nt][1];
                so[(16 * warp + g + 8) * HD + d] = o[nt][2];
                so[(16 * warp + g + 8) * HD + d + 1] = o[nt][3];
            }
        }
        pf_cluster_sync();
        if (r == 0)
        {
#pragma unroll
            for (int nt = 0; nt < HD / 8; ++nt)
            {
                const uint32_t d = nt * 8 + 2 * c;
                o[nt][0] += pf_peer_ld(&so[(16 * warp + g) * HD + d], 1);
                o[nt][1] += pf_peer_ld(&so[(16 * warp + g) * HD + d + 1], 1);
                o[nt][2] += pf_peer_ld(&so[(16 * warp + g + 8) * HD + d], 1);
                o[nt][3] += pf_peer_ld(&so[(16 * warp + g + 8) * HD + d + 1], 1);
            }
        }
        pf_cluster_sync();
        if (r != 0)
            return;
    }
    // ---- store: out[i][h * HD + d] = fp16(o)
    const uint64_t row_pitch = (uint64_t)H * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt)
    {
        const uint32_t d = nt * 8 + 2 * c;
        if (i0 < S)
            *reinterpret_cast<__half2 *>(out + (uint64_t)i0 * row_pitch + (uint64_t)h * HD + d) =
                __floats2half2_rn(o[nt][0], o[nt][1]);
        if (i1 < S)
            *reinterpret_cast<__half2 *>(out + (uint64_t)i1 * row_pitch + (uint64_t)h * HD + d) =
                __floats2half2_rn(o[nt][2], o[nt][3]);
    }
}

} // namespace vkb
