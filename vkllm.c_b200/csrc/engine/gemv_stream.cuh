// Bulk-async weight-streaming GEMV for sm_100a.
//
// Each CTA owns a contiguous range of output "units" (a unit is one output row, or a group of
// weight rows that one epilogue consumes together, e.g. the up and gate rows of one FFN column).
// Each of the eight warps of a CTA is an independent streaming pipeline: it owns `spw` private
// shared-memory stages, lane 0 fills them with cp.async.bulk (the 1-D TMA engine) completing on
// the stage's mbarrier, and the warp refills a stage itself right after consuming it. The warp
// computes fp32 dot products against the input vector staged in shared memory and runs the
// epilogue of its own units, so the main loop has no block-wide barrier, no warp waits for
// another, and every SM keeps 8 * spw chunks of weights in flight. Because a stage is only ever
// used by one warp, in order, its barrier phases cannot be overtaken.
//
// Chunks: when a unit is small, a chunk packs `upc` whole units; when it is large, each weight row
// of a unit is split into `segs` equal segments and a chunk is one segment (the warp accumulates
// the row across its segments and runs the epilogue after the unit's last one). The kernel participates in Programmatic Dependent Launch: it
// issues its first weight chunks before griddepcontrol.wait, i.e. while the previous kernel of the
// step is still finishing, and only then reads the activation vector that kernel produced.
//
// Every mbarrier wait is bounded (about 2 s on %globaltimer); on expiry the kernel records an error
// code in *err, drains its own copies still in flight (bounded again) and returns.
#pragma once

#include <cstdint>

#include "../kernels/common.cuh"

namespace vkb
{

// One CTA per SM with many warps (up to 32), each with its own stage(s): measured on B200, the
// read rate follows the number of independent warp pipelines per SM (one warp computing holds only
// its own stage while every other warp's copy stays in flight).
constexpr int kStreamMaxWarps = 32;
constexpr uint32_t kStreamMaxSpw = 4; // stages per warp
constexpr uint32_t kStreamBarBytes = 8 * kStreamMaxWarps * kStreamMaxSpw;

struct StreamGeom
{
    uint32_t units;       // total units
    uint32_t nm;          // weight rows per unit (1 or 2)
    uint32_t K;           // halves per weight row (multiple of 8)
    uint32_t upc;         // packed mode: units per chunk (segs == 0)
    uint32_t segs;        // split mode: segments per row (> 0), K / segs a multiple of 8
    uint32_t spw;         // stages per warp
    uint32_t warps;       // warps per CTA (block = 32 * warps threads)
    uint32_t chunk_bytes; // bytes of the largest chunk (stage size)
    uint32_t xs_bytes;    // input staging bytes (fp32, multiple of 128)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Bounded wait on phase `parity` of `bar`: false after ~limit_ns.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait(bar, parity))
        return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
    {
        if (global_ns() - t0 > limit_ns)
            return false;
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Prefetches [src, src + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 policy that marks lines first in line for eviction (weights are read once per step).
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void bulk_g2s_hint(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
                 "[%3], %4;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

constexpr uint64_t kWaitLimitNs = 2000000000ull; // 2 s
constexpr uint32_t kErrMbarTimeout = 0x100;

// Issues chunk k of warp w into stage buffer `dst`. Packed mode: units [(w + 8k) * upc, ...) of the
// CTA's range, coalescing rows adjacent in memory. Split mode: segment (k % segs) of row
// (k / segs) % nm of the warp's unit (w + 8 * (k / (nm * segs))). One lane calls it.
template <class Op>
__device__ __forceinline__ void stream_issue(const Op &op, const StreamGeom &g, uint32_t u0, uint32_t count,
                                             uint32_t w, uint32_t k, unsigned char *dst, uint64_t *bar)
{
    const uint32_t row_bytes = g.K * 2;
    if (g.segs == 0)
    {
        const uint32_t ub = (w + g.warps * k) * g.upc;
        const uint32_t n = min(g.upc, count - ub);
        mbar_arrive_expect_tx(bar, n * g.nm * row_bytes);
        const char *seg = nullptr;
        uint32_t seg_bytes = 0;
        unsigned char *seg_dst = dst;
        for (uint32_t i = 0; i < n; ++i)
            for (uint32_t m = 0; m < g.nm; ++m)
            {
                const char *p = reinterpret_cast<const char *>(op.row_ptr(u0 + ub + i, m));
                if (seg && p == seg + seg_bytes)
                    seg_bytes += row_bytes;
                else
                {
                    if (seg)
                        bulk_g2s(seg_dst, seg, seg_bytes, bar);
                    seg_dst = dst + (size_t)(i * g.nm + m) * row_bytes;
                    seg = p;
                    seg_bytes = row_bytes;
                }
            }
        if (seg)
            bulk_g2s(seg_dst, seg, seg_bytes, bar);
    }
    else
    {
        const uint32_t per_unit = g.nm * g.segs;
        const uint32_t u = w + g.warps * (k / per_unit), r = k % per_unit, m = r / g.segs, sg = r % g.segs;
        const uint32_t bytes = row_bytes / g.segs;
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(dst, reinterpret_cast<const char *>(op.row_ptr(u0 + u, m)) + (size_t)sg * bytes, bytes, bar);
    }
}

// Number of chunks warp w streams.
__device__ __forceinline__ uint32_t warp_chunks(const StreamGeom &g, uint32_t count, uint32_t w)
{
    if (g.segs == 0)
    {
        const uint32_t groups = (count + g.upc - 1) / g.upc;
        return groups > w ? (groups - w + g.warps - 1) / g.warps : 0;
    }
    const uint32_t units = count > w ? (count - w + g.warps - 1) / g.warps : 0;
    return units * g.nm * g.segs;
}

// Warp dot products of NM rows (stored back to back, n8 uint4 each) with the staged vector `xs`
// (fp32, pre-scaled by kHalfBitsScale, 2 float4 per uint4 of weights), fp32 accumulation in two
// independent chains per row; results summed across the warp into out[NM].
template <int NM>
__device__ __forceinline__ void warp_dot_rows(const float4 *__restrict__ xs, const uint4 *__restrict__ rows,
                                              uint32_t n8, float *out)
{
    const uint32_t lane = threadIdx.x & 31;
    float a0[NM], a1[NM];
#pragma unroll
    for (int m = 0; m < NM; ++m)
        a0[m] = a1[m] = 0.f;
    uint32_t i = lane;
    for (; i + 32 < n8; i += 64)
    {
        const float4 x0 = xs[2 * i], x1 = xs[2 * i + 1], x2 = xs[2 * (i + 32)], x3 = xs[2 * (i + 32) + 1];
#pragma unroll
        for (int m = 0; m < NM; ++m)
        {
            a0[m] = dot8_scaled(x0, x1, rows[m * n8 + i], a0[m]);
            a1[m] = dot8_scaled(x2, x3, rows[m * n8 + i + 32], a1[m]);
        }
    }
    if (i < n8)
    {
        const float4 x0 = xs[2 * i], x1 = xs[2 * i + 1];
#pragma unroll
        for (int m = 0; m < NM; ++m)
            a0[m] = dot8_scaled(x0, x1, rows[m * n8 + i], a0[m]);
    }
#pragma unroll
    for (int m = 0; m < NM; ++m)
        out[m] = warp_sum(a0[m] + a1[m]);
}

// Op interface:
//   static constexpr int NM;                                // weight rows per unit (1 or 2)
//   const __half *row_ptr(uint32_t unit, uint32_t m) const;
//   void prologue(float *xs, float *red) const;             // all threads; stage the input vector
//                                                           // as fp32 times kHalfBitsScale
//   void epilogue(uint32_t unit, const float *sums) const;  // one lane per unit, sums[NM]
//   void finish() const;                                    // all threads, after the last chunk
template <class Op>
__global__ void __launch_bounds__(kStreamMaxWarps * 32) k_gemv_stream(Op op, StreamGeom g, uint32_t *err)
{
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem); // warps * spw barriers
    float *xs = reinterpret_cast<float *>(smem + kStreamBarBytes);
    unsigned char *stages = smem + kStreamBarBytes + g.xs_bytes;
    __shared__ float sred[32];

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t base = g.units / gridDim.x, rem = g.units % gridDim.x;
    const uint32_t u0 = blockIdx.x * base + min(blockIdx.x, rem);
    const uint32_t count = base + (blockIdx.x < rem ? 1u : 0u);
    const uint32_t nk = warp_chunks(g, count, warp);
    uint64_t *mybar = bars + warp * g.spw;
    unsigned char *mystage = stages + (size_t)warp * g.spw * g.chunk_bytes;

    if (lane == 0)
    {
        for (uint32_t s = 0; s < g.spw; ++s)
            mbar_init(&mybar[s], 1);
        fence_barrier_init();
        fence_proxy_async(); // initialised barriers visible to the bulk-copy (async) proxy
        // Weights do not depend on the previous kernel: start streaming before waiting for it.
        for (uint32_t k = 0; k < nk && k < g.spw; ++k)
            stream_issue(op, g, u0, count, warp, k, mystage + (size_t)k * g.chunk_bytes, &mybar[k]);
    }
    pdl_launch_dependents();
    pdl_wait(); // the input vector (and the residual) come from the previous kernel
    op.prologue(xs, sred);
    __syncthreads();

    const uint32_t n8 = g.K / 8;
    bool failed = false;
    uint32_t issued = min(nk, g.spw);
    if (g.segs == 0)
    {
        for (uint32_t k = 0; k < nk; ++k)
        {
            const uint32_t s = k % g.spw;
            const bool ok = mbar_wait_bounded(&mybar[s], (k / g.spw) & 1u, kWaitLimitNs);
            if (__any_sync(0xffffffffu, !ok)) // warp-uniform decision
            {
                failed = true;
                break;
            }
            const uint32_t ub = (warp + g.warps * k) * g.upc;
            const uint32_t nu = min(g.upc, count - ub);
            const uint4 *st = reinterpret_cast<const uint4 *>(mystage + (size_t)s * g.chunk_bytes);
            float mine[Op::NM];
            for (uint32_t uu = 0; uu < nu; ++uu)
            {
                float sums[Op::NM];
                warp_dot_rows<Op::NM>(reinterpret_cast<const float4 *>(xs), st + (size_t)uu * Op::NM * n8, n8, sums);
                if (lane == (uu & 31))
#pragma unroll
                    for (int m = 0; m < Op::NM; ++m)
                        mine[m] = sums[m];
                if ((uu & 31) == 31 || uu + 1 == nu)
                {
                    const uint32_t first = uu & ~31u;
                    if (lane <= (uu & 31))
                        op.epilogue(u0 + ub + first + lane, mine);
                }
            }
            __syncwarp();
            if (lane == 0 && k + g.spw < nk)
            {
                fence_proxy_async(); // this warp's reads of stage s precede the async refill
                stream_issue(op, g, u0, count, warp, k + g.spw, mystage + (size_t)s * g.chunk_bytes, &mybar[s]);
            }
            issued = min(nk, k + 1 + g.spw);
        }
    }
    else
    {
        const uint32_t sn8 = n8 / g.segs, per_unit = Op::NM * g.segs;
        float acc[Op::NM];
        for (uint32_t k = 0; k < nk; ++k)
        {
            const uint32_t s = k % g.spw;
            const bool ok = mbar_wait_bounded(&mybar[s], (k / g.spw) & 1u, kWaitLimitNs);
            if (__any_sync(0xffffffffu, !ok)) // warp-uniform decision
            {
                failed = true;
                break;
            }
            const uint32_t r = k % per_unit, m = r / g.segs, sg = r % g.segs;
            if (r == 0)
#pragma unroll
                for (int q = 0; q < Op::NM; ++q)
                    acc[q] = 0.f;
            float part;
            warp_dot_rows<1>(reinterpret_cast<const float4 *>(xs) + (size_t)sg * sn8 * 2,
                             reinterpret_cast<const uint4 *>(mystage + (size_t)s * g.chunk_bytes), sn8, &part);
#pragma unroll
            for (int q = 0; q < Op::NM; ++q)
                if ((uint32_t)q == m)
                    acc[q] += part;
            __syncwarp();
            if (lane == 0)
            {
                if (k + g.spw < nk)
                {
                    fence_proxy_async();
                    stream_issue(op, g, u0, count, warp, k + g.spw, mystage + (size_t)s * g.chunk_bytes, &mybar[s]);
                }
                if (r == per_unit - 1)
                    op.epilogue(u0 + warp + g.warps * (k / per_unit), acc);
            }
            issued = min(nk, k + 1 + g.spw);
        }
    }
    if (failed)
    {
        if (lane == 0)
        {
            atomicOr(err, kErrMbarTimeout);
            // Copies this warp issued must land before the CTA's shared memory is released.
            for (uint32_t k = issued > g.spw ? issued - g.spw : 0; k < issued; ++k)
                (void)mbar_wait_bounded(&mybar[k % g.spw], (k / g.spw) & 1u, kWaitLimitNs / 4);
        }
        __syncwarp();
    }
    __syncthreads();
    op.finish();
}

// Host-side geometry: chunks of at most `target` bytes, `spw` stages per warp, and as many warps
// (<= 32) as fit in `smem_cap` next to the fp32 input staging.
inline StreamGeom make_stream_geom(uint32_t units, uint32_t nm, uint32_t K, uint32_t xs_halves, uint32_t target,
                                   uint32_t smem_cap, uint32_t spw = 1)
{
    StreamGeom g{};
    g.units = units;
    g.nm = nm;
    g.K = K;
    const uint32_t row_bytes = K * 2, unit_bytes = nm * row_bytes;
    if (unit_bytes <= target)
    {
        g.upc = target / unit_bytes;
        g.segs = 0;
        g.chunk_bytes = g.upc * unit_bytes;
    }
    else
    {
        const uint32_t n8 = K / 8;
        uint32_t segs = (row_bytes + target - 1) / target;
        while (segs < n8 && n8 % segs != 0)
            ++segs;
        g.upc = 1;
        g.segs = segs;
        g.chunk_bytes = row_bytes / segs;
    }
    g.xs_bytes = (xs_halves * 4 + 127) / 128 * 128; // fp32 staging
    g.spw = spw < 1 ? 1 : (spw > kStreamMaxSpw ? kStreamMaxSpw : spw);
    const uint32_t fixed = kStreamBarBytes + g.xs_bytes;
    const uint32_t w = smem_cap > fixed ? (smem_cap - fixed) / (g.spw * g.chunk_bytes) : 0;
    g.warps = w > (uint32_t)kStreamMaxWarps ? (uint32_t)kStreamMaxWarps : w;
    return g;
}

inline size_t stream_smem_bytes(const StreamGeom &g)
{
    return kStreamBarBytes + g.xs_bytes + (size_t)g.warps * g.spw * g.chunk_bytes;
}

} // namespace vkb
