// Tensor-core GEMM for sm_100a: C[z] = act(scale * A[z] . B[z]^T), fp16 A [M, K] and B [N, K]
// (both K-contiguous), fp32 accumulation in tensor memory, fp16 C [M, N].
//
// One CTA computes a 128 x BN tile of C:
//   warp 4 (one lane)  TMA producer: 2-D boxes of 64 K-elements (128 B, 128-byte swizzle) x 128 rows
//                      of A and x BN rows of B into a ring of shared-memory stages (full barriers);
//   warp 5             allocates BN tensor-memory columns; one lane issues tcgen05.mma
//                      (kind::f16, M = 128, N = BN, K = 16 per instruction, 4 per stage) and
//                      tcgen05.commit frees each stage (empty barriers) and finally signals `done`;
//   warps 0-3          epilogue: tcgen05.ld of their 32 accumulator lanes (rows), scale, SiLU,
//                      fp16 stores with bounds checks.
// Rows and K beyond the operands are zero-filled by TMA, so any M, N and K (K a multiple of 8)
// work. Every wait is bounded (2 s of %globaltimer): on expiry the CTA records an error, lets the
// copies and MMAs it issued complete (bounded again), frees its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <unordered_map>
#include <mutex>
#include <tuple>

#include "kernels.h"

namespace vkb
{
namespace
{

constexpr uint32_t kBK = 64;
constexpr uint32_t kTileRows = 128; // rows of one B tile in the tiled operand layout
constexpr uint64_t kTcWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t su32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t gtime()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(su32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit)
{
    if (try_wait(bar, parity))
        return true;
    const uint64_t t0 = gtime();
    while (!try_wait(bar, parity))
        if (gtime() - t0 > limit)
            return false;
    return true;
}

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile whose 8-row groups are
// 1024 B apart (the layout TMA writes for a 64 x rows fp16 box): start address >> 4 in bits
// [0, 14), leading byte offset 1 (unused for swizzled K-major), stride byte offset 1024 >> 4 in
// bits [32, 46), descriptor version 1 in bits [46, 48), layout SWIZZLE_128B (2) in bits [61, 64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D fp32 (bits [4, 6) = 1), A and B fp16 (formats 0), both
// K-major, N >> 3 in bits [17, 23), M >> 4 in bits [24, 29).
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t M, uint32_t N)
{
    return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
                 "%4, %5}], [%6];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su32(bar))
                 : "memory");
}

// Tile BM x N: BM = 128 (one accumulator) or 256 (two M = 128 accumulators side by side in tensor
// memory, sharing each B tile, which halves the operand bytes per flop of a 128 x N tile). AR: rows
// of A loaded per stage. AR = 64 < BM = 128 serves M <= 64 (batched decode): the stage keeps 8 KB of
// A instead of 16, so one more stage of B fits in flight; the MMA still reads 128 rows, the upper 64
// from the start of the stage's B region (in bounds), and those accumulator rows are never stored.
template <int BM, int N, int AR = BM> struct TileCfg
{
    static constexpr uint32_t kAcc = BM / 128;
    static constexpr uint32_t kABytes = (uint32_t)AR * kBK * 2;
    static constexpr uint32_t kBBytes = (uint32_t)N * kBK * 2;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kStages = (200u * 1024u) / kStageBytes;
    // tensor-memory columns: a power of two >= 32 covering the accumulators
    static constexpr uint32_t kTmemCols = kAcc * N <= 128 ? 128u : (kAcc * N <= 256 ? 256u : 512u);
    static constexpr uint32_t kSmem = 1024 /* alignment slack */ + kStages * kStageBytes + 256 /* barriers */;
};

struct TcParams
{
    uint32_t M, N, K;
    uint64_t ldc;
    uint32_t batch_c;
    uint32_t a_bc, a_cc, b_bc, b_cc; // 1 where the operand's b / c index is broadcast (use 0)
    uint64_t c_sb, c_sc;
    float scale;
    int act;
    uint32_t act_from; // act applies to output columns >= act_from
    uint32_t b_tiled;  // B in 128-row x 64-column tiles (gemm_tile_b); its map is (64, 128, k-block, n-tile)
    uint32_t b_group_n; // > 0: B rows come from up to three matrices of b_group_n rows each (tmB, tmB1, tmB2)
    uint32_t b_groups;  // their count
    uint32_t b_piece;   // > 0: grouped B tiles load as pieces of this many rows (b_group_n % BN != 0)
    __half *C;
    uint32_t *err;
    // Split-K: `splits` CTAs share a tile, each over kb_per k-blocks, writing fp32 partials to
    // `ws` [split][z][M][N]; k_splitk_reduce sums them in split order and applies the epilogue.
    uint32_t splits, kb_per;
    float *ws;
};

// Split-K epilogue part: 32 fp32 partial columns of one row to the workspace.
__device__ __forceinline__ void store_part32(float *wrow, uint32_t nb, const uint32_t (&r)[32], const TcParams &p)
{
    if (nb + 32 <= p.N && (p.N % 4) == 0)
    {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            reinterpret_cast<float4 *>(wrow + nb)[j] =
                make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                            __uint_as_float(r[4 * j + 3]));
    }
    else
    {
        for (uint32_t j = 0; j < 32 && nb + j < p.N; ++j)
            wrow[nb + j] = __uint_as_float(r[j]);
    }
}

// Epilogue of 32 consecutive accumulator columns of one row: scale, SiLU when act, fp16.
__device__ __forceinline__ void store_row32(__half *crow, uint32_t nb, const uint32_t (&r)[32], const TcParams &p)
{
    __half h[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
    {
        float v = __uint_as_float(r[j]) * p.scale;
        if (p.act && nb + j >= p.act_from)
            v = v / (1.0f + expf(-v)); // SiLU as the reference evaluates it
        h[j] = __float2half_rn(v);
    }
    if (nb + 32 <= p.N && (p.ldc % 8) == 0 && ((reinterpret_cast<uintptr_t>(crow) & 15) == 0))
    {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4 *>(crow + nb)[j] = reinterpret_cast<const uint4 *>(h)[j];
    }
    else
    {
        for (uint32_t j = 0; j < 32 && nb + j < p.N; ++j)
            crow[nb + j] = h[j];
    }
}

template <int BM, int BN, int AR = BM>
__global__ void __launch_bounds__(192, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmA,
                                                     const __grid_constant__ CUtensorMap tmB,
                                                     const __grid_constant__ CUtensorMap tmB1,
                                                     const __grid_constant__ CUtensorMap tmB2, TcParams p)
{
    static_assert(AR == BM || (BM == 128 && AR == 64), "A rows per stage: the tile's, or 64 of a 128-row tile");
    using Cfg = TileCfg<BM, BN, AR>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t base = (su32(smem_raw) + 1023u) & ~1023u; // 1024-B aligned stages (swizzle atoms)
    unsigned char *smem = smem_raw + (base - su32(smem_raw));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Cfg::kStages * Cfg::kStageBytes);
    uint64_t *empty = full + Cfg::kStages;
    uint64_t *done = empty + Cfg::kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    __shared__ uint32_t fail_s;

    // a kernel launched as this one's programmatic dependent may start its CTAs now (its own wait
    // still orders it after this grid's completion)
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, z = blockIdx.z / p.splits, split = blockIdx.z % p.splits;
    const uint32_t zb = z / p.batch_c, zc = z % p.batch_c;
    const uint32_t kb_all = (p.K + kBK - 1) / kBK;
    const uint32_t kb_lo = split * p.kb_per, kb_n = min(kb_all, kb_lo + p.kb_per) - kb_lo; // >= 1 (host)

    if (threadIdx.x == 0)
    {
        for (uint32_t s = 0; s < Cfg::kStages; ++s)
        {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(done)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fail_s = 0;
    }
    if (warp == 5)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(Cfg::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4 && lane == 0)
    {
        // Producer.
        const int32_t ca = p.a_cc ? 0 : (int32_t)zc, ba = p.a_bc ? 0 : (int32_t)zb;
        const int32_t cb = p.b_cc ? 0 : (int32_t)zc, bb = p.b_bc ? 0 : (int32_t)zb;
        // grouped B, whole tiles: the tile's rows n0 .. n0 + BN - 1 lie in one group (b_group_n % BN == 0)
        const uint32_t grp = p.b_group_n && !p.b_piece ? n0 / p.b_group_n : 0u;
        const CUtensorMap *mapB = grp == 0 ? &tmB : (grp == 1 ? &tmB1 : &tmB2);
        const uint32_t nb0 = n0 - grp * p.b_group_n;
        auto load_b = [&](uint32_t kb, uint32_t sb, uint64_t *bar) {
            if (p.b_tiled) // BN / 128 consecutive tiles of the k-block: the same smem image as BN rows
                tma_load_4d(sb, mapB, 0, 0, (int32_t)(kb_lo + kb), (int32_t)(nb0 / kTileRows), bar);
            else if (p.b_piece)
            {
                // pieces of b_piece rows (128 B each in the swizzled image), each from its group's map;
                // rows past N read the last group's map out of range (zero fill, same byte count)
                for (uint32_t r = 0; r < (uint32_t)BN; r += p.b_piece)
                {
                    const uint32_t row = n0 + r, gi = min(row / p.b_group_n, p.b_groups - 1);
                    tma_load_4d(sb + r * 128, gi == 0 ? &tmB : (gi == 1 ? &tmB1 : &tmB2), (int32_t)((kb_lo + kb) * kBK),
                                (int32_t)(row - gi * p.b_group_n), 0, 0, bar);
                }
            }
            else
                tma_load_4d(sb, mapB, (int32_t)((kb_lo + kb) * kBK), (int32_t)nb0, cb, bb, bar);
        };
        // The first stages' B tiles (weights, never written by the kernels this one may overlap) load
        // before the wait for the previous kernel in the stream (a no-op unless launched as its
        // programmatic dependent); A, its output, loads after it.
        const uint32_t pre = kb_n < Cfg::kStages ? kb_n : Cfg::kStages;
        for (uint32_t kb = 0; kb < pre; ++kb)
        {
            const uint32_t sa = base + kb * Cfg::kStageBytes;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[kb])),
                         "r"(Cfg::kStageBytes)
                         : "memory");
            load_b(kb, sa + Cfg::kABytes, &full[kb]);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (uint32_t kb = 0; kb < pre; ++kb)
            tma_load_4d(base + kb * Cfg::kStageBytes, &tmA, (int32_t)((kb_lo + kb) * kBK), (int32_t)m0, ca, ba,
                        &full[kb]);
        uint32_t issued = pre;
        bool ok = true;
        for (uint32_t kb = pre; kb < kb_n; ++kb)
        {
            const uint32_t s = kb % Cfg::kStages, n = kb / Cfg::kStages;
            if (n > 0 && !wait_bounded(&empty[s], (n - 1) & 1u, kTcWaitNs))
            {
                ok = false;
                break;
            }
            const uint32_t sa = base + s * Cfg::kStageBytes, sb = sa + Cfg::kABytes;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[s])),
                         "r"(Cfg::kStageBytes)
                         : "memory");
            tma_load_4d(sa, &tmA, (int32_t)((kb_lo + kb) * kBK), (int32_t)m0, ca, ba, &full[s]); // BM rows
            load_b(kb, sb, &full[s]);
            ++issued;
        }
        if (!ok)
        {
            atomicOr(p.err, 1u);
            fail_s = 1;
            // the stages issued and not yet consumed must land before the CTA exits
            for (uint32_t kb = issued > Cfg::kStages ? issued - Cfg::kStages : 0; kb < issued; ++kb)
                (void)wait_bounded(&full[kb % Cfg::kStages], (kb / Cfg::kStages) & 1u, kTcWaitNs / 4);
        }
    }
    else if (warp == 5 && lane == 0)
    {
        // MMA issuer.
        constexpr uint32_t idesc = f16_idesc(128, BN);
        bool ok = true;
        for (uint32_t kb = 0; kb < kb_n; ++kb)
        {
            const uint32_t s = kb % Cfg::kStages;
            if (!wait_bounded(&full[s], (kb / Cfg::kStages) & 1u, kTcWaitNs))
            {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = base + s * Cfg::kStageBytes, sb = sa + Cfg::kABytes;
#pragma unroll
            for (uint32_t k = 0; k < kBK / 16; ++k)
            {
                const uint64_t db = sw128_desc(sb + 32 * k);
                const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
                for (uint32_t h = 0; h < Cfg::kAcc; ++h)
                {
                    // rows 128 h .. 128 h + 127 of the A tile (16 KB further per half) -> accumulator h
                    const uint64_t da = sw128_desc(sa + h * (128 * 128) + 32 * k);
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem + h * BN),
                                 "l"(da), "l"(db), "r"(idesc), "r"(acc));
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             su32(&empty[s]))
                         : "memory");
        }
        if (!ok)
        {
            atomicOr(p.err, 1u);
            fail_s = 1;
        }
        // Signals the epilogue once every MMA issued above has completed (also on the error path,
        // so that the tensor memory is idle before it is freed).
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(done))
                     : "memory");
    }
    else if (warp < 4)
    {
        // Epilogue: row m0 + 32 * warp + lane of the tile, 32 accumulator columns per load.
        const bool ok = wait_bounded(done, 0, 2 * kTcWaitNs);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__all_sync(0xffffffffu, ok) && !fail_s)
#pragma unroll 1
            for (uint32_t h = 0; h < Cfg::kAcc; ++h)
        {
            const uint32_t row = m0 + 128 * h + 32 * warp + lane;
            __half *crow = p.C + zb * p.c_sb + zc * p.c_sc + (uint64_t)row * p.ldc;
            const uint32_t taddr = tmem + ((32 * warp) << 16) + h * BN;
#pragma unroll 1
            for (uint32_t c = 0; c < (uint32_t)BN; c += 32)
            {
                uint32_t r[32];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
                             "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
                             "%28, %29, %30, %31}, [%32];"
                             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                               "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                               "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
                               "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
                               "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                             : "r"(taddr + c));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const uint32_t nb = n0 + c;
                if (row < p.M && nb < p.N)
                {
                    if (p.splits > 1)
                        store_part32(p.ws + (((uint64_t)split * gridDim.z / p.splits + z) * p.M + row) * p.N, nb, r,
                                     p);
                    else
                        store_row32(crow, nb, r, p);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 5)
    {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols));
    }
}

// Sums the split-K partials in split order, then scale, SiLU and fp16 store (the epilogue of the
// unsplit kernel). One thread per 4 columns.
__global__ void k_splitk_reduce(const float *__restrict__ ws, TcParams p, uint32_t batch)
{
    // 8 consecutive columns per thread: two 16-byte loads per split, one 16-byte fp16 store when the
    // rows of C allow it (the sum runs in split order either way, so both paths give the same bits)
    const uint32_t n8 = (p.N + 7) / 8;
    const uint64_t total = (uint64_t)batch * p.M * n8;
    const uint64_t plane = (uint64_t)batch * p.M * p.N;
    const bool vec = (p.N % 8) == 0 && (p.ldc % 8) == 0 && (p.c_sb % 8) == 0 && (p.c_sc % 8) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.C) & 15) == 0;
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t c8 = (uint32_t)(t % n8);
        const uint64_t rz = t / n8;
        const uint32_t row = (uint32_t)(rz % p.M), z = (uint32_t)(rz / p.M);
        const uint32_t zb = z / p.batch_c, zc = z % p.batch_c;
        __half *crow = p.C + zb * p.c_sb + zc * p.c_sc + (uint64_t)row * p.ldc;
        const uint64_t off = ((uint64_t)z * p.M + row) * p.N + 8ull * c8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (vec)
        {
            for (uint32_t sidx = 0; sidx < p.splits; ++sidx)
            {
                const float4 a = __ldcs(reinterpret_cast<const float4 *>(ws + sidx * plane + off));
                const float4 b = __ldcs(reinterpret_cast<const float4 *>(ws + sidx * plane + off) + 1);
                v[0] += a.x, v[1] += a.y, v[2] += a.z, v[3] += a.w, v[4] += b.x, v[5] += b.y, v[6] += b.z, v[7] += b.w;
            }
        }
        else
        {
            for (uint32_t sidx = 0; sidx < p.splits; ++sidx)
                for (uint32_t j = 0; j < 8 && 8 * c8 + j < p.N; ++j)
                    v[j] += ws[sidx * plane + off + j];
        }
        __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            float x = v[j] * p.scale;
            if (p.act && 8 * c8 + j >= p.act_from)
                x = x / (1.0f + expf(-x));
            h[j] = __float2half_rn(x);
        }
        if (vec)
            *reinterpret_cast<uint4 *>(crow + 8 * c8) = *reinterpret_cast<const uint4 *>(h);
        else
            for (uint32_t j = 0; j < 8 && 8 * c8 + j < p.N; ++j)
                crow[8 * c8 + j] = h[j];
    }
}

// Per-device split-K workspace, grown on demand (never inside stream capture: growth fails there and
// the caller runs without splitting).
float *splitk_workspace(int dev, size_t bytes, cudaStream_t s)
{
    static float *ws[64] = {};
    static size_t cap[64] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64)
        return nullptr;
    if (cap[dev] >= bytes)
        return ws[dev];
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess || st != cudaStreamCaptureStatusNone)
    {
        (void)cudaGetLastError();
        return nullptr;
    }
    (void)cudaGetLastError();
    float *p = nullptr;
    const size_t want = bytes < ((size_t)32 << 20) ? ((size_t)32 << 20) : bytes;
    if (cudaMalloc(&p, want) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return nullptr;
    }
    if (ws[dev])
    {
        cudaDeviceSynchronize();
        cudaFree(ws[dev]);
    }
    ws[dev] = p;
    cap[dev] = want;
    return p;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            (void)cudaGetLastError();
    });
    return fn;
}

// Encoded tensor maps, keyed by everything an encoding reads (a map holds an address and a shape,
// so a key seen before gives the same map): prefill and the op path launch their GEMMs on the same
// operands every step. Per thread, bounded (cleared when full).
struct MapKey
{
    const void *ptr;
    uint64_t v[9];
    bool operator==(const MapKey &o) const
    {
        return ptr == o.ptr && memcmp(v, o.v, sizeof(v)) == 0;
    }
};
struct MapKeyHash
{
    size_t operator()(const MapKey &k) const
    {
        uint64_t h = reinterpret_cast<uintptr_t>(k.ptr) * 1099511628211ull;
        for (uint64_t x : k.v)
            h = (h ^ x) * 1099511628211ull;
        return (size_t)h;
    }
};
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> &map_cache()
{
    static thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
    if (maps.size() > 4096)
        maps.clear();
    return maps;
}

bool encode_operand_uncached(CUtensorMap *m, const void *ptr, uint32_t K, uint32_t rows, uint64_t ld,
                             uint32_t ext_c, uint64_t sc, uint32_t ext_b, uint64_t sb, uint32_t box_rows);

// 4-D map {K, rows, C, B} of an fp16 operand (K innermost), box {64, box_rows, 1, 1}, 128-byte
// swizzle, zero fill outside. Broadcast dimensions get extent 1.
bool encode_operand(CUtensorMap *m, const void *ptr, uint32_t K, uint32_t rows, uint64_t ld, uint32_t ext_c,
                    uint64_t sc, uint32_t ext_b, uint64_t sb, uint32_t box_rows)
{
    const MapKey key{ptr, {K, rows, ld, ext_c, sc, ext_b, sb, box_rows, 0}};
    auto &maps = map_cache();
    auto it = maps.find(key);
    if (it != maps.end())
    {
        *m = it->second;
        return true;
    }
    if (!encode_operand_uncached(m, ptr, K, rows, ld, ext_c, sc, ext_b, sb, box_rows))
        return false;
    maps.emplace(key, *m);
    return true;
}

bool encode_operand_uncached(CUtensorMap *m, const void *ptr, uint32_t K, uint32_t rows, uint64_t ld,
                             uint32_t ext_c, uint64_t sc, uint32_t ext_b, uint64_t sb, uint32_t box_rows)
{
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn)
        return false;
    const uint64_t row_b = ld * 2;
    const uint64_t c_b = ext_c > 1 ? sc * 2 : row_b * rows;
    const uint64_t b_b = ext_b > 1 ? sb * 2 : c_b * ext_c;
    cuuint64_t dims[4] = {K, rows, ext_c, ext_b};
    cuuint64_t strides[3] = {row_b, c_b, b_b};
    cuuint32_t box[4] = {kBK, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    if (row_b % 16 || c_b % 16 || b_b % 16 || (reinterpret_cast<uintptr_t>(ptr) & 15))
        return false;
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// B in tile order (gemm_tile_b): dims (64, 128, k-blocks, n-tiles), every box (64, 128, 1,
// box_rows / 128) a contiguous run of box_rows * 128 bytes.
bool encode_tiled_b(CUtensorMap *m, const void *ptr, uint32_t K, uint32_t N, uint32_t box_rows)
{
    const MapKey key{ptr, {K, N, box_rows, 0, 0, 0, 0, 0, 1}};
    auto &maps = map_cache();
    auto it = maps.find(key);
    if (it != maps.end())
    {
        *m = it->second;
        return true;
    }
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || box_rows % kTileRows)
        return false;
    const uint64_t kbs = (K + kBK - 1) / kBK, nts = (N + kTileRows - 1) / kTileRows;
    const uint64_t tile_b = (uint64_t)kTileRows * kBK * 2;
    cuuint64_t dims[4] = {kBK, kTileRows, kbs, nts};
    cuuint64_t strides[3] = {kBK * 2, tile_b, tile_b * kbs};
    cuuint32_t box[4] = {kBK, kTileRows, 1, box_rows / kTileRows};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    maps.emplace(key, *m);
    return true;
}

uint32_t *error_word(int dev)
{
    static uint32_t *words[64] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64)
        return nullptr;
    if (!words[dev])
    {
        if (cudaMalloc(&words[dev], sizeof(uint32_t)) != cudaSuccess || cudaMemset(words[dev], 0, 4) != cudaSuccess)
        {
            (void)cudaGetLastError();
            words[dev] = nullptr;
        }
    }
    return words[dev];
}

// ws_ext / splits_out: when given, the split-K partials go to the caller's buffer ([splits][batch][M]
// [N] fp32, splits > 1) and no reduction is launched; *splits_out receives the split count used.
template <int BM, int BN, int AR = BM>
bool launch_tc(const GemmArgs &g, cudaStream_t s, uint32_t splits = 1, float *ws_ext = nullptr,
               uint32_t *splits_out = nullptr)
{
    using Cfg = TileCfg<BM, BN, AR>;
    if (AR < BM && g.M > (uint32_t)AR)
        return false;
    int dev = 0, cc = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return false;
    cudaDeviceGetAttribute(&cc, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (cc != 10 || (uint32_t)optin < Cfg::kSmem)
        return false;
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev])
    {
        if (cudaFuncSetAttribute(k_gemm_tc<BM, BN, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Cfg::kSmem) != cudaSuccess)
        {
            (void)cudaGetLastError();
            return false;
        }
        attr_set[dev] = true;
    }
    const uint32_t batch_b = g.batch / g.batch_c;
    CUtensorMap ma, mb;
    // broadcast dimensions (stride 0) are described with extent 1 and indexed 0 by the kernel
    if (!encode_operand(&ma, g.A, g.K, g.M, g.lda, g.a_sc ? g.batch_c : 1, g.a_sc, g.a_sb ? batch_b : 1, g.a_sb, AR))
        return false;
    if (g.b_tiled)
    {
        if (g.batch != 1 || BN % kTileRows || !encode_tiled_b(&mb, g.B, g.K, g.N, BN))
            return false;
    }
    else if (!encode_operand(&mb, g.B, g.K, g.N, g.ldb, g.b_sc ? g.batch_c : 1, g.b_sc, g.b_sb ? batch_b : 1, g.b_sb,
                             BN))
        return false;
    CUtensorMap mb1 = mb, mb2 = mb;
    uint32_t group_n = 0, groups = 0, piece = 0;
    if (g.b_group_n)
    {
        // grouped B: N = groups * b_group_n rows, group i from B, B1, B2; a tile that may straddle two
        // groups (b_group_n % BN != 0) loads in 32-row pieces, which never do (b_group_n % 32 == 0)
        groups = g.N / g.b_group_n;
        piece = g.b_group_n % BN ? 32u : 0u;
        if (g.b_tiled || g.batch != 1 || (piece && g.b_group_n % piece) || groups * g.b_group_n != g.N ||
            groups < 1 || groups > 3)
            return false;
        const void *src[3] = {g.B, g.B1, g.B2};
        CUtensorMap *dst[3] = {&mb, &mb1, &mb2};
        for (uint32_t i = 0; i < groups; ++i)
            if (!src[i] || !encode_operand(dst[i], src[i], g.K, g.b_group_n, g.ldb, 1, 0, 1, 0, piece ? piece : BN))
                return false;
        group_n = g.b_group_n;
    }
    TcParams p{};
    p.b_group_n = group_n;
    p.b_groups = groups;
    p.b_piece = piece;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.ldc = g.ldc;
    p.batch_c = g.batch_c;
    p.a_bc = g.a_sb == 0;
    p.a_cc = g.a_sc == 0;
    p.b_bc = g.b_sb == 0;
    p.b_cc = g.b_sc == 0;
    p.c_sb = g.c_sb;
    p.c_sc = g.c_sc;
    p.scale = g.scale;
    p.act = g.act;
    p.act_from = g.act_from;
    p.b_tiled = g.b_tiled ? 1u : 0u;
    p.C = (__half *)g.C;
    p.err = error_word(dev);
    if (!p.err)
        return false;
    const uint32_t kb_all = (g.K + kBK - 1) / kBK;
    if (splits > kb_all)
        splits = kb_all;
    p.kb_per = (kb_all + splits - 1) / splits;
    p.splits = splits > 1 ? (kb_all + p.kb_per - 1) / p.kb_per : 1; // every split gets >= 1 k-block
    p.ws = nullptr;
    if (ws_ext)
    {
        if (p.splits < 2)
            return false;
        p.ws = ws_ext;
        *splits_out = p.splits;
    }
    else if (p.splits > 1)
    {
        p.ws = splitk_workspace(dev, (size_t)p.splits * g.batch * g.M * g.N * sizeof(float), s);
        if (!p.ws)
        {
            p.splits = 1;
            p.kb_per = kb_all;
        }
    }
    dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.batch * p.splits);
    if (g.pdl)
    {
        // programmatic dependent of the previous kernel in the stream: CTAs start (and prefetch B)
        // while it finishes; griddepcontrol.wait in the producer orders everything else after it
        cudaLaunchConfig_t lc{};
        lc.gridDim = grid;
        lc.blockDim = dim3(192);
        lc.dynamicSmemBytes = Cfg::kSmem;
        lc.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        if (cudaLaunchKernelEx(&lc, k_gemm_tc<BM, BN, AR>, ma, mb, mb1, mb2, p) != cudaSuccess)
            return false;
    }
    else
        k_gemm_tc<BM, BN, AR><<<grid, 192, Cfg::kSmem, s>>>(ma, mb, mb1, mb2, p);
    if (p.splits > 1 && !ws_ext)
    {
        const uint64_t work = (uint64_t)g.batch * g.M * ((g.N + 7) / 8);
        const unsigned blocks = (unsigned)((work + 255) / 256 < 148u * 16u ? (work + 255) / 256 : 148u * 16u);
        k_splitk_reduce<<<blocks, 256, 0, s>>>(p.ws, p, g.batch);
    }
    return cudaGetLastError() == cudaSuccess;
}

} // namespace

bool encode_kv_rows_map(CUtensorMap *m, const __half *base, uint32_t hd, uint32_t cap, uint32_t heads, uint32_t seqs,
                        uint32_t box_rows)
{
    return hd % kBK == 0 && box_rows >= 8 && box_rows <= 256 && box_rows % 8 == 0 &&
           encode_operand(m, base, hd, cap, hd, heads, (uint64_t)cap * hd, seqs, (uint64_t)heads * cap * hd, box_rows);
}

bool make_gemm_args(const Desc4 &da, const Desc4 &db, const Desc4 &dc, bool trans_b, const void *a, const void *b,
                    void *c, float scale, int act, GemmArgs *g)
{
    // A [Ba, Ca, M, K], B [Bb, Cb, N, K] (trans_b), C [B, C, M, N]; unit inner strides; row and batch
    // strides multiples of 8 elements; 16-byte aligned bases.
    if (!trans_b)
        return false;
    if (da.stride[3] != 1 || db.stride[3] != 1 || dc.stride[3] != 1)
        return false;
    const uint32_t M = dc.shape[2], N = dc.shape[3], K = da.shape[3];
    if (db.shape[3] != K || db.shape[2] != N || da.shape[2] != M || K == 0 || M == 0 || N == 0)
        return false;
    if (K % 8 || da.stride[2] % 8 || db.stride[2] % 8)
        return false;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al16(a) || !al16(b) || !al16(c))
        return false;
    const uint32_t Bc = dc.shape[0], Cc = dc.shape[1];
    for (int i = 0; i < 2; ++i)
    {
        if ((da.shape[i] != 1 && da.shape[i] != dc.shape[i]) || (db.shape[i] != 1 && db.shape[i] != dc.shape[i]))
            return false;
        if (da.stride[i] % 8 || db.stride[i] % 8)
            return false;
    }
    g->A = a;
    g->B = b;
    g->C = c;
    g->M = M;
    g->N = N;
    g->K = K;
    g->lda = da.stride[2];
    g->ldb = db.stride[2];
    g->ldc = dc.stride[2];
    g->batch_c = Cc;
    g->batch = Bc * Cc;
    g->a_sb = da.shape[0] == 1 ? 0 : da.stride[0];
    g->a_sc = da.shape[1] == 1 ? 0 : da.stride[1];
    g->b_sb = db.shape[0] == 1 ? 0 : db.stride[0];
    g->b_sc = db.shape[1] == 1 ? 0 : db.stride[1];
    g->c_sb = dc.stride[0];
    g->c_sc = dc.stride[1];
    g->scale = scale;
    g->act = act;
    return true;
}

namespace
{
// A launch configuration: tile (kTiles[tile]) and K splits. The 256-row tiles narrower than 256
// columns let a shape's tile count fill the SMs in whole waves (e.g. 512 x 12288: 128 tiles of
// 256 x 192 in one wave, against 96 of 256 x 256 or 192 of 128 x 256).
struct TcChoice
{
    uint8_t tile = 0, splits = 1;
};
// Tiles 6 and 7 are 128 x 256 and 128 x 128 loading 64 rows of A per stage (M <= 64).
constexpr uint32_t kNumTiles = 8;
constexpr uint32_t kTileBM[kNumTiles] = {128, 128, 256, 256, 256, 256, 128, 128};
constexpr uint32_t kTileBN[kNumTiles] = {128, 256, 256, 192, 160, 224, 256, 128};
constexpr uint32_t kTileAR[kNumTiles] = {128, 128, 256, 256, 256, 256, 64, 64};

bool launch_choice(const GemmArgs &g, cudaStream_t s, TcChoice c)
{
    switch (c.tile)
    {
    case 7:
        return launch_tc<128, 128, 64>(g, s, c.splits);
    case 6:
        return launch_tc<128, 256, 64>(g, s, c.splits);
    case 5:
        return launch_tc<256, 224>(g, s, c.splits);
    case 4:
        return launch_tc<256, 160>(g, s, c.splits);
    case 3:
        return launch_tc<256, 192>(g, s, c.splits);
    case 2:
        return launch_tc<256, 256>(g, s, c.splits);
    case 1:
        return launch_tc<128, 256>(g, s, c.splits);
    default:
        return launch_tc<128, 128>(g, s, c.splits);
    }
}

// Cost-model choice: the tile minimising waves x time per tile; small M (GEMM-shaped decode) splits K
// so that every SM streams.
TcChoice model_choice(const GemmArgs &g, int sms)
{
    auto tiles = [&](uint32_t bm, uint32_t bn) {
        return (uint64_t)((g.N + bn - 1) / bn) * ((g.M + bm - 1) / bm) * g.batch;
    };
    auto cost = [&](uint32_t bm, uint32_t bn, double per_tile) {
        return (double)((tiles(bm, bn) + sms - 1) / sms) * per_tile;
    };
    TcChoice c;
    const uint64_t t128 = tiles(128, 128);
    if (g.M <= 128 && t128 * 2 <= (uint64_t)sms)
    {
        const uint64_t sp = (uint64_t)sms / t128;
        c.splits = (uint8_t)(sp > 8 ? 8 : sp);
        return c;
    }
    // Per K step, a 128 x 128 tile takes ~0.85 and a 256 x 256 tile ~1.64 of the time of a 128 x 256
    // tile (L2-to-SM operand bandwidth, measured on B200).
    const double c128 = cost(128, 128, 0.85), c256 = cost(128, 256, 1.0), c2x = g.M > 128 ? cost(256, 256, 1.64) : 1e30;
    c.tile = (c2x < c256 && c2x < c128) ? 2 : (c256 < c128 ? 1 : 0);
    return c;
}

struct TuneKey
{
    int dev;
    uint32_t M, N, K, batch, tiled;
    bool operator<(const TuneKey &o) const
    {
        return std::tie(dev, M, N, K, batch, tiled) < std::tie(o.dev, o.M, o.N, o.K, o.batch, o.tiled);
    }
};

// Times each candidate (tile x splits) twice after one warm-up launch and returns the fastest; the
// model's choice is kept unless another is more than 3 % faster. Every candidate computes the same
// C (to fp32 summation order), so the trials are harmless; the caller then launches the winner.
TcChoice tune(const GemmArgs &g_in, cudaStream_t s, int sms, TcChoice model)
{
    GemmArgs g = g_in;
    g.pdl = 0; // trials run one after another, without overlapping the previous one

    cudaEvent_t e0, e1;
    if (cudaEventCreate(&e0) != cudaSuccess)
        return model;
    if (cudaEventCreate(&e1) != cudaSuccess)
    {
        cudaEventDestroy(e0);
        return model;
    }
    auto time_of = [&](TcChoice c) {
        if (!launch_choice(g, s, c))
            return 1e30f;
        float best = 1e30f;
        for (int r = 0; r < 2; ++r)
        {
            float ms = 0.f;
            if (cudaEventRecord(e0, s) != cudaSuccess || !launch_choice(g, s, c) ||
                cudaEventRecord(e1, s) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess ||
                cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess)
                return 1e30f;
            best = ms < best ? ms : best;
        }
        return best;
    };
    const uint32_t kb_all = (g.K + kBK - 1) / kBK;
    float t_model = time_of(model), t_best = t_model;
    TcChoice best = model;
    for (uint8_t t = 0; t < kNumTiles; ++t)
    {
        if ((kTileBM[t] == 256 && g.M <= 128) || g.M > kTileAR[t])
            continue;
        if (g.b_tiled && kTileBN[t] % 128)
            continue;
        const uint64_t n_tiles =
            (uint64_t)((g.N + kTileBN[t] - 1) / kTileBN[t]) * ((g.M + kTileBM[t] - 1) / kTileBM[t]) * g.batch;
        for (uint8_t sp : {1, 2, 3, 4, 6, 8})
        {
            if (sp > kb_all || (sp > 1 && n_tiles * sp > 2ull * (uint64_t)sms) || (t == model.tile && sp == model.splits))
                continue;
            const float tm = time_of(TcChoice{t, sp});
            if (tm < t_best)
            {
                t_best = tm;
                best = TcChoice{t, sp};
            }
        }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    (void)cudaGetLastError();
    return t_best < 0.97f * t_model ? best : model;
}
} // namespace

bool gemm_tcgen05_launch(const GemmArgs &g, cudaStream_t s)
{
    if (g.batch == 0 || g.batch_c == 0)
        return false;
    const char *force = getenv("VKLLM_B200_GEMM_TILE"), *force_splits = getenv("VKLLM_B200_GEMM_SPLITS");
    if (force)
    {
        const uint32_t sp = force_splits ? (uint32_t)atoi(force_splits) : 1u;
        if (!strcmp(force, "256x256"))
            return launch_tc<256, 256>(g, s, sp);
        if (!strcmp(force, "128x256a64"))
            return launch_tc<128, 256, 64>(g, s, sp);
        if (!strcmp(force, "128x128a64"))
            return launch_tc<128, 128, 64>(g, s, sp);
        if (!strcmp(force, "256x192"))
            return launch_tc<256, 192>(g, s, sp);
        if (!strcmp(force, "256x160"))
            return launch_tc<256, 160>(g, s, sp);
        if (!strcmp(force, "256x224"))
            return launch_tc<256, 224>(g, s, sp);
        if (!strcmp(force, "128x256"))
            return launch_tc<128, 256>(g, s, sp);
        if (!strcmp(force, "128x128"))
            return launch_tc<128, 128>(g, s, sp);
    }
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const TcChoice model = model_choice(g, sms);
    // Shapes worth more than ~1 GFLOP are tuned once per process (VKLLM_B200_GEMM_TUNE=0: model only);
    // never inside stream capture, where the model's choice (or an earlier tuning result) is used.
    // VKLLM_B200_GEMM_TUNE_FILE: choices are read from this file at the first call and appended to
    // it when tuned, so later processes (or a profiler run, whose timings would mislead the tuner)
    // reuse them. One line per shape: "M N K batch layout tile splits" (layout: bit 0 tiled B, bit 1
    // grouped B).
    static std::map<TuneKey, TcChoice> cache;
    static std::mutex mu;
    static bool file_loaded = false;
    const char *tune_file = getenv("VKLLM_B200_GEMM_TUNE_FILE");
    const uint32_t layout = (g.b_tiled ? 1u : 0u) | (g.b_group_n ? 2u : 0u); // operand layout of B
    const TuneKey key{dev, g.M, g.N, g.K, g.batch, layout};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (tune_file && !file_loaded)
        {
            file_loaded = true;
            if (FILE *f = fopen(tune_file, "r"))
            {
                unsigned m, n, k, b, bt, t, sp;
                while (fscanf(f, "%u %u %u %u %u %u %u", &m, &n, &k, &b, &bt, &t, &sp) == 7)
                    if (bt <= 3 && t < kNumTiles && sp >= 1 && sp <= 8)
                        for (int d = 0; d < 64; ++d) // the file carries no device: it applies to each
                            cache[TuneKey{d, m, n, k, b, bt}] = TcChoice{(uint8_t)t, (uint8_t)sp};
                fclose(f);
            }
        }
        auto it = cache.find(key);
        if (it != cache.end())
            return launch_choice(g, s, it->second);
    }
    const char *tune_env = getenv("VKLLM_B200_GEMM_TUNE");
    const bool tune_on = !(tune_env && atoi(tune_env) == 0);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (!tune_on || 2.0 * g.M * g.N * (double)g.K * g.batch < 1e9 || cudaStreamIsCapturing(s, &cap) != cudaSuccess ||
        cap != cudaStreamCaptureStatusNone)
    {
        (void)cudaGetLastError();
        return launch_choice(g, s, model);
    }
    const TcChoice best = tune(g, s, sms, model);
    {
        std::lock_guard<std::mutex> lk(mu);
        cache[key] = best;
        if (tune_file)
            if (FILE *f = fopen(tune_file, "a"))
            {
                fprintf(f, "%u %u %u %u %u %u %u\n", g.M, g.N, g.K, g.batch, layout, (unsigned)best.tile,
                        (unsigned)best.splits);
                fclose(f);
            }
    }
    return launch_choice(g, s, best);
}

bool gemm_tcgen05_partials(const GemmArgs &g, cudaStream_t s, uint32_t splits, float *ws, uint32_t *splits_used,
                           uint32_t tile)
{
    if (g.batch == 0 || g.batch_c == 0 || !ws || !splits_used || splits < 2)
        return false;
    switch (tile)
    {
    case 3:
        return launch_tc<128, 256, 64>(g, s, splits, ws, splits_used);
    case 2:
        return launch_tc<128, 128, 64>(g, s, splits, ws, splits_used);
    case 1:
        return launch_tc<128, 256>(g, s, splits, ws, splits_used);
    default:
        return launch_tc<128, 128>(g, s, splits, ws, splits_used);
    }
}

namespace
{
// One 16-byte chunk (8 fp16) of the tiled copy per thread; rows past the sources and columns past K
// are zero.
__global__ void k_tile_b(TileSrcs src, uint32_t K, uint32_t kbs, __half *__restrict__ dst, uint64_t chunks, bool vec)
{
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t c8 = (uint32_t)(i & 7), r = (uint32_t)((i >> 3) % kTileRows);
        const uint64_t tk = (i >> 3) / kTileRows;
        const uint32_t kb = (uint32_t)(tk % kbs), nt = (uint32_t)(tk / kbs);
        uint32_t n = nt * kTileRows + r;
        const uint32_t k = kb * kBK + 8 * c8;
        uint4 v = make_uint4(0, 0, 0, 0);
        uint32_t si = 0;
        while (si < src.n && n >= src.rows[si])
            n -= src.rows[si++];
        if (si < src.n && k < K)
        {
            const __half *row = src.ptr[si] + (uint64_t)n * K;
            if (vec)
                v = *reinterpret_cast<const uint4 *>(row + k);
            else
            {
                __half *h = reinterpret_cast<__half *>(&v);
                for (uint32_t e = 0; e < 8 && k + e < K; ++e)
                    h[e] = row[k + e];
            }
        }
        reinterpret_cast<uint4 *>(dst)[i] = v;
    }
}
} // namespace

uint64_t gemm_tiled_b_elems(uint32_t N, uint32_t K)
{
    return (uint64_t)((N + kTileRows - 1) / kTileRows) * kTileRows * ((K + kBK - 1) / kBK) * kBK;
}

bool gemm_tile_b(const TileSrcs &src, uint32_t K, __half *dst, cudaStream_t s)
{
    uint64_t n = 0;
    bool vec = (K % 8) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (src.n == 0 || src.n > TileSrcs::kMax || K == 0)
        return false;
    for (uint32_t i = 0; i < src.n; ++i)
    {
        if (!src.ptr[i])
            return false;
        n += src.rows[i];
        vec = vec && (reinterpret_cast<uintptr_t>(src.ptr[i]) & 15) == 0;
    }
    if (n == 0 || n > 0xffffffffull)
        return false;
    const uint64_t chunks = gemm_tiled_b_elems((uint32_t)n, K) / 8;
    const uint64_t blocks = (chunks + 255) / 256;
    k_tile_b<<<(unsigned)(blocks < 148u * 32u ? blocks : 148u * 32u), 256, 0, s>>>(src, K, (K + kBK - 1) / kBK, dst,
                                                                                chunks, vec);
    return cudaGetLastError() == cudaSuccess;
}

uint32_t gemm_tcgen05_error(int dev)
{
    uint32_t *w = error_word(dev), v = 0;
    if (!w || cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0xffffffffu;
    return v;
}

} // namespace vkb

// ------------------------------------------------------------------------------------------------
// C-ABI: the tensor-core GEMM on raw device pointers (declared in include/vkllm_b200.h).
#include "vkllm_errors.h"

extern "C" vkllm_err_t vkllm_b200_gemm_f16(const void *A, const void *B, void *C, uint32_t M, uint32_t N, uint32_t K,
                                           uint64_t lda, uint64_t ldb, uint64_t ldc, float scale, int act,
                                           void *stream)
{
    if (!A || !B || !C || M == 0 || N == 0 || K == 0 || lda < K || ldb < K || ldc < N)
        return VKLLM_ERR_ARGS;
    vkb::Desc4 da{{1, 1, M, K}, {0, 0, (uint32_t)lda, 1}};
    vkb::Desc4 db{{1, 1, N, K}, {0, 0, (uint32_t)ldb, 1}};
    vkb::Desc4 dc{{1, 1, M, N}, {0, 0, (uint32_t)ldc, 1}};
    vkb::GemmArgs g;
    if (lda > 0xffffffffull || ldb > 0xffffffffull || ldc > 0xffffffffull ||
        !vkb::make_gemm_args(da, db, dc, true, A, B, C, scale, act, &g))
        return VKLLM_ERR_ARGS;
    if (!vkb::gemm_tcgen05_launch(g, (cudaStream_t)stream))
    {
        (void)cudaGetLastError();
        return VKLLM_ERR_VULKAN;
    }
    return VKLLM_ERR_OK;
}

extern "C" uint32_t vkllm_b200_gemm_f16_error(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return 0xffffffffu;
    return vkb::gemm_tcgen05_error(dev);
}
