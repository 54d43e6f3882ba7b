// Persistent LLaMA-2 decode: one cooperative launch runs whole decode steps.
//
// One CTA per SM. Every warp of every CTA streams its share of ALL the step's weights, in step
// order (per layer: QKV, Wo, up/gate, down; then the logits matrix), through its private
// shared-memory stages with cp.async.bulk, and keeps streaming across matrix boundaries: while the
// CTA waits at a grid barrier, or computes attention, the next matrix's weights are already
// landing. Activations are exchanged through global memory between grid barriers.
//
// Weight tiles: a CTA owns a contiguous range of output rows of each matrix, cut into tiles of 16
// rows x 256 columns. The engine keeps a decode copy of the weights in which every tile is
// contiguous in HBM (tiles in the order the CTA consumes them, each CTA's tiles where its rows are
// in the row-major matrix) with the 16-byte chunks of tile row r XOR-swizzled by r & 7, so a tile is
// ONE bulk copy (the bulk-copy request rate of one SM, not HBM, limits 512 B row copies) and the
// ldmatrix reads of 8 rows hit 8 different bank groups. A warp reduces a tile against the staged
// fp16 input vector with mma.sync m16n8k16 (the vector is the B operand, replicated over the 8
// columns; products exact, fp32 accumulation): ~4 instructions per 512 B. The tile partials land
// in a per-CTA [segment][row] buffer that is summed in a fixed order after the phase.
//
// Phases:
//
//   [embed rows]  per layer: rmsnorm+QKV+RoPE+KV write | scores | probs.V | Wo+residual |
//                 rmsnorm+up/gate+SiLU | down+residual   then: rmsnorm+logits | argmax
//
// Every node output is rounded to fp16 where the reference graph materialises it
// (src/models/vkllm_llama2_layers.c:13-340), arithmetic is fp32. Every spin (mbarrier waits, grid
// barriers) is bounded (~2 s on %globaltimer); on expiry or when another CTA reported an error the
// kernel records it, drains its own bulk copies still in flight and returns.
#pragma once

#include "decode_kernels.cuh"
#include "gemv_stream.cuh"

namespace vkb
{

enum PhaseKind : uint32_t
{
    PK_QKV = 0,
    PK_WO = 1,
    PK_UPGATE = 2,
    PK_DOWN = 3,
    PK_LOGITS = 4,
    PK_COUNT = 5
};

constexpr uint32_t kErrBarrierTimeout = 0x200;
constexpr uint32_t kErrPeerTimeout = 0x400;
constexpr uint32_t kTpMax = 8;     // ranks
constexpr uint32_t kTpCtas = 256;  // flag slots per site (>= CTAs of the grid)
constexpr uint32_t kTpRows = 64;   // Wo / down output rows a CTA may own under tensor parallelism
constexpr uint32_t kErrPosition = 0x1;

#ifndef VKB_PERSIST_SEG
#define VKB_PERSIST_SEG 256
#endif
constexpr uint32_t kTileRows = 16;                        // MMA M
constexpr uint32_t kSegHalves = VKB_PERSIST_SEG;          // columns per tile (one bulk copy per row)
constexpr uint32_t kTileBytes = kTileRows * kSegHalves * 2; // one stage (a full tile)
// At most 24 warps per CTA, so that the launch bound leaves each thread 80 registers (65536 / 768);
// shared memory limits the 7B and 13B shapes to 23 and 22 warps of one 8 KB stage each anyway.
constexpr int kPersistMaxWarps = 24;
constexpr uint32_t kPersistMaxGrid = 256; // CTAs (one per SM)
constexpr uint32_t kAttWindow = 4; // attention key rounds whose K (then V) rows are loaded at once
// Trace slots after the per-warp pipeline accounting: CTA 0's attention sub-steps (SM cycles).
constexpr uint32_t kAttTraceBase = kStreamMaxWarps * PK_COUNT * 4, kAttTraceSlots = 8;
constexpr uint32_t kCtaTraceBarriers = 1024, kCtaTraceMaxCtas = 256;

// Physical 16-byte chunk of logical chunk c in row r of a tile whose rows hold nchunks chunks:
// swizzled within aligned groups of 8 (the tail of a row that is not a whole group stays in place).
__host__ __device__ __forceinline__ uint32_t tile_chunk(uint32_t c, uint32_t r, uint32_t nchunks)
{
    return ((c | 7u) < nchunks) ? (c ^ (r & 7u)) : c;
}

// Geometry of one GEMV phase kind: `units` outputs of `nm` rows each, rows of K columns cut into
// Ks segments of kSegHalves (the last one `last` wide, a multiple of 16).
struct TileGeom
{
    uint32_t units, nm, K, Ks, last;
};

struct PersistParams
{
    DecodeDims dd;
    const LayerW *layers; // device array [L]
    uint32_t L;
    const __half *embed, *wout;
    const float *out_norm;
    uint32_t unk;
    __half *x, *q, *m, *logits, *scores;
    float2 *part;
    float *opart;
    float *am_val;     // per-CTA argmax partials [grid][32]
    uint32_t *am_idx;  // [grid][32]
    StepState *st;
    uint32_t *ring;
    uint32_t ring_len;
    uint32_t *bar_count;    // grid barrier arrivals (zeroed before each launch, with the two below)
    uint32_t *head_cnt;     // [H] attention splits that published their softmax statistics
    uint32_t *head_done;    // [H] attention splits that published their partial outputs
    __half *attn;           // [H * hd] attention output (the combined splits)
    uint32_t att_groups;    // key groups of the attention phase (bounded by the scratch)
    uint32_t *err;
    TileGeom tg[PK_COUNT];
    uint32_t spw, warps;    // stages per warp (a power of two), warps per CTA
    uint32_t spw_shift;     // log2(spw): stage and phase of chunk i are i & (spw - 1), (i >> spw_shift) & 1
    uint32_t xs_bytes;      // fp16 input staging (>= 2 * max K)
    uint32_t part_bytes;    // tile partials; xs + part also serve as the attention scratch
    uint32_t n_steps;
    uint32_t att_split;     // key splits per head in the attention phases
    const __half *const *tiled; // decode copy of the weights: [layer * 4 + kind] (QKV, Wo, up/gate, down)
    const __half *tiled_logits; // decode copy of the output matrix
    const float *rope_den;      // [hd / 2] RoPE denominators base^(2w / hd)
    const uint32_t *utab;       // [kind][grid + 1]: CTA b owns units [utab[b], utab[b + 1]) of each phase
    uint64_t *trace;        // optional: CTA 0 records %globaltimer at every barrier arrival/release
    uint32_t trace_cap;     // entries available in `trace`
    unsigned long long *wtrace; // optional: CTA 0 per (warp, kind): wait, consume, chunks, compute part
    uint64_t *trace_last;       // optional: per trace entry, %globaltimer when the last CTA arrived
    uint64_t *trace_cta;        // optional: [barrier][CTA] %globaltimer of each CTA's arrival (first
                                // kCtaTraceBarriers grid barriers of a launch)
    // Fine-grained Wo and down phases (fine = 1): instead of a grid barrier after attention and after
    // up/gate, each producer publishes an epoch flag (head_flag[h] once head h's attention output is
    // combined, cta_flag[b] once CTA b's up/gate rows are written), and a Wo or down tile waits only
    // for the producers of its 256 input columns: the heads they span, or dn_seg[2 k] .. dn_seg[2 k + 1],
    // the first and last CTA whose up/gate units intersect segment k.
    uint32_t fine;
    uint32_t *cta_flag;         // [grid], zeroed before each launch (grows within a launch)
    uint32_t *head_flag;        // [H]: epoch once a head's attention output is combined (fine = 1)
    const uint32_t *dn_seg;     // [2 * segments of the down phase]
    uint32_t l2_bytes;          // per CTA: next-phase weights prefetched into L2 at each barrier
    uint32_t l2_hint;           // 1: stage loads mark their lines evict-first in L2
    // Tensor parallelism over peer memory (tp_size 1: off). Each rank owns H / N heads, F / N FFN
    // rows and V / N vocabulary rows (from v0); the Wo and down outputs are partial sums that every
    // rank writes, per output row, into every peer's receive area, then raises a flag per CTA.
    uint32_t tp_size, tp_rank, v0, Vg;
    uint64_t *tp_x[kTpMax];       // rank q's receive slots [2 sites][N ranks][kTpCtas][kTpRows]: epoch, fp32
    uint32_t *tp_flag[kTpMax];    // rank q's flags [3 sites][kTpCtas][N ranks]
    float *tp_amv[kTpMax];        // rank q's argmax class slots [N ranks][32]
    uint32_t *tp_ami[kTpMax];
    uint32_t tp_base[3];          // exchanges done per site before this launch (flags only grow)
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Barrier and trace bookkeeping of thread 0 of a CTA.
struct SyncState
{
    uint32_t n;     // trace entries so far
    uint32_t epoch; // grid barriers passed so far
};

// Grid-wide barrier for a cooperative launch (all CTAs co-resident): one release-add per CTA on a
// counter that only grows during the launch (zeroed before it); barrier n completes when the
// counter reaches n * gridDim.x. Bounded: false when it timed out or another CTA reported an error.
__device__ __forceinline__ bool grid_sync(const PersistParams &P, SyncState &tr)
{
    __shared__ uint32_t ok_s;
    __syncthreads();
    if (threadIdx.x == 0)
    {
        if (P.trace && blockIdx.x == 0 && tr.n < P.trace_cap)
            P.trace[tr.n] = global_ns();
        ++tr.n;
        bool ok = true;
        if (P.trace_cta && tr.epoch < kCtaTraceBarriers - 1)
            P.trace_cta[(uint64_t)tr.epoch * gridDim.x + blockIdx.x] = global_ns();
        const uint32_t target = (++tr.epoch) * gridDim.x;
        uint32_t prev;
        asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.bar_count) : "memory");
        if (prev + 1 == target)
        {
            if (P.trace_last && tr.n < P.trace_cap)
                P.trace_last[tr.n] = global_ns();
        }
        else
        {
            const uint64_t t0 = global_ns();
            while (ld_acquire_u32(P.bar_count) < target)
            {
                if (ld_acquire_u32(P.err) != 0)
                {
                    ok = false;
                    break;
                }
                if (global_ns() - t0 > kWaitLimitNs)
                {
                    atomicOr(P.err, kErrBarrierTimeout);
                    ok = false;
                    break;
                }
            }
        }
        if (P.trace && blockIdx.x == 0 && tr.n < P.trace_cap)
            P.trace[tr.n] = global_ns();
        ++tr.n;
        ok_s = ok ? 1u : 0u;
    }
    __syncthreads();
    return ok_s != 0;
}

// Trace point of CTA 0 (after a staging prologue); `tr` counts entries on every CTA.
__device__ __forceinline__ void trace_mark(const PersistParams &P, SyncState &tr)
{
    if (threadIdx.x == 0)
    {
        if (P.trace && blockIdx.x == 0 && tr.n < P.trace_cap)
            P.trace[tr.n] = global_ns();
        ++tr.n;
    }
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A flag store after the caller's __threadfence_system(): that one fence orders every earlier store
// of the thread (and, after __syncthreads, of its CTA) before the flags, so the flags to each peer
// need no release of their own (a system-scope release per peer costs a fence each).
__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t *p, uint32_t v)
{
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 8-byte slots of the tensor-parallel exchange: (epoch << 32) | fp32 bits, written and read as one
// aligned 64-bit access, so a reader that sees the epoch sees the value with it.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p)
{
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

struct UnitRange
{
    uint32_t u0, count;
};

// This CTA's units of each phase, loaded from P.utab when the launch starts.
__shared__ UnitRange s_units[PK_COUNT];

__device__ __forceinline__ UnitRange cta_units(uint32_t kind)
{
    return s_units[kind];
}

// This CTA's fp32 partials of its Wo / down output rows under tensor parallelism (the epilogue
// stages them here; tp_allreduce_rows pushes them to the peers as one block).
__shared__ __align__(16) float s_tp_stage[kTpRows];

// Tensor-parallel allreduce of this CTA's output rows of the Wo (site 0) or down (site 1) phase:
// each staged row partial goes to the same CTA slot of every rank as one 8-byte store carrying the
// exchange's epoch with the value (no fence and no separate flag: a slot showing the epoch holds
// the value). Then each row waits (bounded) for every rank's slot to show the epoch, sums the
// partials in rank order (fp32, so every rank computes the same bits), rounds to fp16 (the
// projection node) and adds the residual: x = fp16(x + fp16(sum)). A slot is rewritten only after
// its reader has used it: the writer's next exchange at this site needs the reader's contribution
// to the exchange in between. Returns false on a timed-out wait or a reported error.
__device__ __forceinline__ bool tp_allreduce_rows(const PersistParams &P, uint32_t site, uint32_t epoch)
{
    __syncthreads(); // the staged rows are complete
    const UnitRange r = cta_units(site == 0 ? PK_WO : PK_DOWN);
    {
        const uint64_t blk = (((uint64_t)site * P.tp_size + P.tp_rank) * kTpCtas + blockIdx.x) * kTpRows;
        const uint64_t tag = (uint64_t)epoch << 32;
        for (uint32_t t = threadIdx.x; t < r.count * P.tp_size; t += blockDim.x)
        {
            const uint32_t q = t / r.count, i = t % r.count;
            st_relaxed_sys_u64(P.tp_x[q] + blk + i, tag | __float_as_uint(s_tp_stage[i]));
        }
    }
    bool ok = true;
    const uint64_t *rx = P.tp_x[P.tp_rank] + ((uint64_t)site * P.tp_size * kTpCtas + blockIdx.x) * kTpRows;
    for (uint32_t i = threadIdx.x; i < r.count && ok; i += blockDim.x)
    {
        float t = 0.f;
        for (uint32_t q = 0; q < P.tp_size && ok; ++q)
        {
            const uint64_t *slot = rx + (uint64_t)q * kTpCtas * kTpRows + i;
            uint64_t v = ld_relaxed_sys_u64(slot);
            if ((uint32_t)(v >> 32) != epoch)
            {
                const uint64_t t0 = global_ns();
                while ((uint32_t)((v = ld_relaxed_sys_u64(slot)) >> 32) != epoch)
                {
                    if (ld_acquire_u32(P.err) != 0)
                    {
                        ok = false;
                        break;
                    }
                    if (global_ns() - t0 > kWaitLimitNs)
                    {
                        atomicOr(P.err, kErrPeerTimeout);
                        ok = false;
                        break;
                    }
                }
            }
            t += __uint_as_float((uint32_t)v);
        }
        if (ok)
        {
            const uint32_t u = r.u0 + i;
            P.x[u] = __float2half_rn(__half2float(__ldcg(P.x + u)) + round_f16(t));
        }
    }
    return __syncthreads_and(ok) != 0;
}

// Producer cursor of one warp over its chunk sequence (step, layer, kind, k).
struct Cursor
{
    uint32_t step, layer, kind, k;
    bool done;
    // geometry of the current phase for this warp, set when the cursor enters the phase
    uint32_t nk;         // tiles of this warp in the phase
    uint32_t Ks, K, rows, last;
    uint32_t grp, ks;    // the next tile: row group and K segment (tile t = w + warps * k)
    const __half *base;  // this CTA's region of the phase matrix in the decode copy
};

// Tiles of this CTA in a phase: ceil(rows / 16) row groups x Ks segments, tile t = group * Ks + segment.
__device__ __forceinline__ uint32_t cta_tiles(const TileGeom &g, uint32_t count)
{
    return (count * g.nm + kTileRows - 1) / kTileRows * g.Ks;
}

// This CTA's region of a phase matrix in the decode copy: its rows' bytes of the row-major matrix.
__device__ __forceinline__ const __half *tiled_region(const PersistParams &P, uint32_t kind, uint32_t layer,
                                                      const TileGeom &g, const UnitRange &r)
{
    const __half *base = kind == PK_LOGITS ? P.tiled_logits : P.tiled[layer * 4 + kind];
    return base + (uint64_t)r.u0 * g.nm * g.K;
}

// Loads the geometry of the cursor's (kind, layer) phase; the per-tile advance is then divisions-free.
__device__ __forceinline__ void cursor_enter(const PersistParams &P, Cursor &c, uint32_t w)
{
    const TileGeom &g = P.tg[c.kind];
    const UnitRange r = cta_units(c.kind);
    const uint32_t T = cta_tiles(g, r.count);
    c.nk = T > w ? (T - w + P.warps - 1) / P.warps : 0;
    c.Ks = g.Ks;
    c.K = g.K;
    c.rows = r.count * g.nm;
    c.last = g.last;
    c.grp = w / g.Ks;
    c.ks = w % g.Ks;
    c.base = tiled_region(P, c.kind, c.layer, g, r);
}

// Tile t + warps from tile t: (grp, ks) of t = grp * Ks + ks.
__device__ __forceinline__ void tile_step(uint32_t &grp, uint32_t &ks, uint32_t Ks, uint32_t warps)
{
    ks += warps;
    while (ks >= Ks)
    {
        ks -= Ks;
        ++grp;
    }
}

__device__ __forceinline__ void cursor_settle(const PersistParams &P, Cursor &c, uint32_t w)
{
    // Skip phases where this warp has no chunk.
    while (!c.done && c.k >= c.nk)
    {
        c.k = 0;
        if (c.kind == PK_LOGITS)
        {
            c.kind = PK_QKV;
            c.layer = 0;
            if (++c.step >= P.n_steps)
                c.done = true;
        }
        else if (c.kind == PK_DOWN)
        {
            if (++c.layer >= P.L)
                c.kind = PK_LOGITS;
            else
                c.kind = PK_QKV;
        }
        else
            ++c.kind;
        if (!c.done)
            cursor_enter(P, c, w);
    }
}

// Issues the single bulk copy of the cursor's tile into `dst` (lane 0).
__device__ __forceinline__ void cursor_issue(const PersistParams &P, const Cursor &c, uint32_t w, unsigned char *dst,
                                             uint64_t *bar, uint64_t policy)
{
    const uint32_t lane = threadIdx.x & 31;
    if (lane != 0)
        return;
    const uint32_t r0 = c.grp * kTileRows, nvalid = min(kTileRows, c.rows - r0);
    const uint32_t width = c.ks + 1 == c.Ks ? c.last : kSegHalves;
    const __half *src = c.base + (uint64_t)r0 * c.K + (uint64_t)c.ks * nvalid * kSegHalves;
    const uint32_t bytes = nvalid * width * 2;
    mbar_arrive_expect_tx(bar, bytes);
    fence_proxy_async(); // this warp's earlier reads of the stage precede the async refill
    if (policy)
        bulk_g2s_hint(dst, src, bytes, bar, policy);
    else
        bulk_g2s(dst, src, bytes, bar);
}

// Per-warp pipeline state.
struct WarpPipe
{
    uint64_t *bar;        // spw barriers
    unsigned char *stage; // spw stages of kTileBytes
    uint32_t consumed;    // chunks consumed so far (global count)
    uint32_t issued;      // chunks issued so far
    Cursor cur;           // next chunk to issue (warp-uniform)
    uint64_t policy;      // L2 policy of the stage loads (0: default)
};

// Issues the next tile into its stage.
__device__ __forceinline__ void pipe_advance(const PersistParams &P, WarpPipe &wp, uint32_t warp)
{
    const uint32_t slot = wp.issued & (P.spw - 1);
    cursor_issue(P, wp.cur, warp, wp.stage + (size_t)slot * kTileBytes, &wp.bar[slot], wp.policy);
    ++wp.issued;
    ++wp.cur.k;
    tile_step(wp.cur.grp, wp.cur.ks, wp.cur.Ks, P.warps);
    cursor_settle(P, wp.cur, warp);
}

// Prefetches into L2 this CTA's rows of phase (kind, layer) beyond the tiles the warps' stages take
// first (up to l2_bytes): each CTA's rows of a matrix are contiguous, so a few large requests cover
// them. Issued when the CTA reaches a grid barrier, it keeps HBM streaming through the barrier,
// the next input staging and the attention phases. One thread.
__device__ __forceinline__ void prefetch_slice(const PersistParams &P, uint32_t kind, uint32_t layer)
{
    if (P.l2_bytes == 0)
        return;
    const TileGeom &g = P.tg[kind];
    const UnitRange r = cta_units(kind);
    const uint64_t region = (uint64_t)r.count * g.nm * g.K * 2, staged = (uint64_t)P.warps * P.spw * kTileBytes;
    if (staged >= region)
        return;
    const char *c = reinterpret_cast<const char *>(tiled_region(P, kind, layer, g, r)) + staged;
    const uint64_t n = min((uint64_t)P.l2_bytes, region - staged);
    for (uint64_t o = 0; o < n; o += 65536)
        bulk_prefetch_l2(c + o, (uint32_t)min((uint64_t)65536, n - o));
}

// Epilogue of one unit of a GEMV phase (executed by one lane).
template <bool TP>
__device__ __forceinline__ void persist_epilogue(const PersistParams &P, uint32_t kind, const LayerW &lw, uint32_t u,
                                                 const float *s, uint32_t pos)
{
    const DecodeDims &dd = P.dd;
    switch (kind)
    {
    case PK_QKV: {
        const uint32_t HD = dd.H * dd.hd, row = 2 * u, which = row / HD, r = row % HD;
        float v0 = round_f16(s[0]), v1 = round_f16(s[1]);
        const uint32_t head = r / dd.hd, d = r % dd.hd;
        if (which < 2)
        {
            const uint32_t w = d / 2;
            // rope_den[w] = powf(base, 2w / hd), computed once on the device
            const float theta = (float)pos / __ldg(P.rope_den + w);
            const float c = cosf(theta), sn = sinf(theta);
            const float o0 = c * v0 - sn * v1, o1 = sn * v0 + c * v1;
            v0 = o0;
            v1 = o1;
        }
        const __half2 hv = __floats2half2_rn(v0, v1);
        if (which == 0)
            *reinterpret_cast<__half2 *>(P.q + r) = hv;
        else
        {
            __half *cache = which == 1 ? lw.kcache : lw.vcache;
            *reinterpret_cast<__half2 *>(cache + ((uint64_t)head * dd.ctx + pos) * dd.hd + d) = hv;
        }
        break;
    }
    case PK_WO:
    case PK_DOWN:
        if constexpr (TP) // partial over this rank's K slice, staged for tp_allreduce_rows
            s_tp_stage[u - cta_units(kind).u0] = s[0];
        else
            P.x[u] = __float2half_rn(__half2float(__ldcg(P.x + u)) + round_f16(s[0]));
        break;
    case PK_UPGATE:
        P.m[u] = __float2half_rn(round_f16(s[0]) * round_f16(silu_f32(s[1])));
        break;
    default:
        P.logits[u] = __float2half_rn(s[0]);
        break;
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

// c += A(16x16, row) * B(16x8, col), fp16 inputs, fp32 accumulation.
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr uint32_t kFineMaxSegs = 64;
// Segment states of the fine-grained down phase in this CTA: 0 not staged, 1 being staged, 2 ready.
__shared__ uint32_t s_seg[kFineMaxSegs];

__device__ __forceinline__ void st_release_gpu_u32(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Makes input segment ks (columns 256 ks .. 256 ks + width) of a gated phase ready in xs: the first
// warp to need it waits (bounded) until flags[first .. last] all reached `epoch`, then copies the
// columns from src (L2); other warps that need it meanwhile wait (bounded) for that copy.
// Warp-uniform; false on a timed-out wait or a reported error.
__device__ __forceinline__ bool fine_segment(const PersistParams &P, uint32_t ks, uint32_t width, __half *xs,
                                             const __half *src, const uint32_t *flags, uint32_t first, uint32_t last,
                                             uint32_t epoch)
{
    const uint32_t lane = threadIdx.x & 31;
    uint32_t st = 0;
    if (lane == 0)
        st = atomicCAS(&s_seg[ks], 0u, 1u);
    st = __shfl_sync(0xffffffffu, st, 0);
    if (st == 2)
    {
        __threadfence_block();
        return true;
    }
    const uint64_t t0 = global_ns();
    if (st == 1)
    {
        // another warp stages it
        bool ok = true;
        if (lane == 0)
            while (*reinterpret_cast<volatile uint32_t *>(&s_seg[ks]) != 2u)
            {
                if (global_ns() - t0 > kWaitLimitNs || ld_acquire_u32(P.err) != 0)
                {
                    ok = false;
                    break;
                }
                __nanosleep(32);
            }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __threadfence_block();
        return ok;
    }
    // this warp stages it: lane 0 acquires every producer's flag, polling with a growing sleep so that
    // waiting warps do not flood the flags' L2 lines; __syncwarp then orders the lanes' loads after it
    bool okw = true;
    if (lane == 0)
    {
        uint32_t nap = 32;
        for (uint32_t b = first; b <= last && okw; ++b)
            while (ld_acquire_u32(flags + b) < epoch)
            {
                if (global_ns() - t0 > kWaitLimitNs || ld_acquire_u32(P.err) != 0)
                {
                    atomicOr(P.err, kErrBarrierTimeout);
                    okw = false;
                    break;
                }
                __nanosleep(nap);
                nap = nap < 512 ? 2 * nap : nap;
            }
    }
    okw = __shfl_sync(0xffffffffu, okw, 0);
    if (!okw)
        return false;
    __syncwarp();
    const uint32_t n4 = width / 8; // 16-byte chunks, at most 32
    if (lane < n4)
        reinterpret_cast<uint4 *>(xs + ks * kSegHalves)[lane] =
            __ldcg(reinterpret_cast<const uint4 *>(src + ks * kSegHalves) + lane);
    __syncwarp();
    __threadfence_block();
    if (lane == 0)
        atomicExch(&s_seg[ks], 2u);
    return true;
}

// One GEMV phase: consumes this warp's tiles (partials to `part`), then the CTA sums the partials
// of each of its units in segment order and runs the epilogue. Returns false when a wait timed out
// in any warp of the CTA.
template <int NM, bool TP, bool TRACE, bool GATED = false>
__device__ __forceinline__ bool persist_gemv(const PersistParams &P, uint32_t kind, uint32_t layer, WarpPipe &wp,
                                             const __half *xs, float *part, uint32_t pos, SyncState &tr,
                                             uint32_t gate_epoch = 0)
{
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom &g = P.tg[kind];
    const UnitRange r = cta_units(kind);
    const uint32_t groups = (r.count * NM + kTileRows - 1) / kTileRows, pitch = groups * kTileRows;
    const uint32_t T = groups * g.Ks;
    const uint32_t nk = T > warp ? (T - warp + P.warps - 1) / P.warps : 0;
    const LayerW &lw = P.layers[kind == PK_LOGITS ? 0 : layer];
    const bool wt = TRACE && P.wtrace && blockIdx.x == 0 && lane == 0; // per-warp pipeline accounting
    unsigned long long t_wait = 0, t_cons = 0, t_comp = 0;
    bool ok = true;
    uint32_t grp = warp / g.Ks, ks = warp % g.Ks; // tile t = warp + warps * k = grp * Ks + ks
    for (uint32_t k = 0; k < nk; ++k, tile_step(grp, ks, g.Ks, P.warps))
    {
        if constexpr (GATED)
        {
            const uint32_t width = ks + 1 == g.Ks ? g.last : kSegHalves;
            bool okg;
            if (kind == PK_WO) // input: the attention output; producers: the heads the segment spans
                okg = fine_segment(P, ks, width, const_cast<__half *>(xs), P.attn, P.head_flag, ks * kSegHalves / P.dd.hd,
                                   (ks * kSegHalves + width - 1) / P.dd.hd, gate_epoch);
            else // PK_DOWN: input m; producers: the up/gate CTAs of the segment
                okg = fine_segment(P, ks, width, const_cast<__half *>(xs), P.m, P.cta_flag, __ldg(P.dn_seg + 2 * ks),
                                   __ldg(P.dn_seg + 2 * ks + 1), gate_epoch);
            if (!okg)
            {
                ok = false;
                break;
            }
        }
        const uint32_t gi = wp.consumed, s = gi & (P.spw - 1);
        const long long c0 = wt ? clock64() : 0;
        const bool okw = mbar_wait_bounded(&wp.bar[s], (gi >> P.spw_shift) & 1u, kWaitLimitNs);
        if (__any_sync(0xffffffffu, !okw))
        {
            ok = false;
            break;
        }
        const long long c1 = wt ? clock64() : 0;
        t_wait += (unsigned long long)(c1 - c0);
        const uint32_t width = ks + 1 == g.Ks ? g.last : kSegHalves;
        const unsigned char *st = wp.stage + (size_t)s * kTileBytes;
        // ldmatrix rows: lanes 0-15 -> tile rows 0-15 at chunk 2j, lanes 16-31 -> rows 0-15 at chunk 2j + 1
        const uint32_t tr = lane & 15, half = lane >> 4, nchunks = width >> 3;
        const uint32_t row_addr = smem_u32(st + tr * width * 2);
        // two accumulator chains (even / odd k-steps) halve the dependent MMA latency
        float c[4] = {0.f, 0.f, 0.f, 0.f}, d[4] = {0.f, 0.f, 0.f, 0.f};
        if (width == kSegHalves)
        {
            // Full tile: every 16 B chunk c of row r sits at c ^ (r & 7). For chunk 4i + h (h < 4) that
            // is 4 (i ^ (r >> 2 & 1)) + (h ^ (r & 3)), so each row's ldmatrix address is one of two
            // per-lane bases (i even / odd) plus 64 i bytes. The input vector (the B operand, equal in
            // all 8 columns) comes from one ldmatrix.x4 whose 8 row addresses per matrix coincide:
            // matrix m holds xs[kk + 8m .. kk + 8m + 7], so lane l receives the pair at 2 (l & 3).
            const uint32_t lo = tr & 3, b64 = 64 * ((tr >> 2) & 1);
            const uint32_t a_base = row_addr + 16 * (half ^ lo), e_base = row_addr + 16 * ((2 + half) ^ lo);
            const uint32_t a_ev = a_base + b64, a_od = a_base - b64, e_ev = e_base + b64, e_od = e_base - b64;
            const uint32_t xb = smem_u32(xs + ks * kSegHalves) + 16 * (lane >> 3);
#pragma unroll
            for (uint32_t i = 0; i < kSegHalves / 32; ++i)
            {
                uint32_t a0, a1, a2, a3, e0, e1, e2, e3, x0, x1, x2, x3;
                ldsm_x4(((i & 1) ? a_od : a_ev) + 64 * i, a0, a1, a2, a3);
                ldsm_x4(((i & 1) ? e_od : e_ev) + 64 * i, e0, e1, e2, e3);
                ldsm_x4(xb + 64 * i, x0, x1, x2, x3);
                mma_16816(c, a0, a1, a2, a3, x0, x1);
                mma_16816(d, e0, e1, e2, e3, x2, x3);
            }
        }
        else
        {
            const uint32_t *xk = reinterpret_cast<const uint32_t *>(xs + ks * kSegHalves + 2 * (lane & 3));
            uint32_t kk = 0;
            for (; kk + 32 <= width; kk += 32)
            {
                uint32_t a0, a1, a2, a3, e0, e1, e2, e3;
                ldsm_x4(row_addr + 16 * tile_chunk((kk >> 3) + half, tr, nchunks), a0, a1, a2, a3);
                ldsm_x4(row_addr + 16 * tile_chunk((kk >> 3) + 2 + half, tr, nchunks), e0, e1, e2, e3);
                mma_16816(c, a0, a1, a2, a3, xk[kk / 2], xk[kk / 2 + 4]);
                mma_16816(d, e0, e1, e2, e3, xk[kk / 2 + 8], xk[kk / 2 + 12]);
            }
            if (kk < width)
            {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(row_addr + 16 * tile_chunk((kk >> 3) + half, tr, nchunks), a0, a1, a2, a3);
                mma_16816(c, a0, a1, a2, a3, xk[kk / 2], xk[kk / 2 + 4]);
            }
        }
        if ((lane & 3) == 0)
        {
            const uint32_t row = grp * kTileRows + (lane >> 2);
            part[ks * pitch + row] = c[0] + d[0];
            part[ks * pitch + row + 8] = c[2] + d[2];
        }
        __syncwarp();
        const long long c2 = wt ? clock64() : 0;
        t_comp += (unsigned long long)(c2 - c1);
        if (!wp.cur.done)
            pipe_advance(P, wp, warp);
        ++wp.consumed;
        if (wt)
            t_cons += (unsigned long long)(clock64() - c1);
    }
    if (wt)
    {
        unsigned long long *o = P.wtrace + ((size_t)warp * PK_COUNT + kind) * 4;
        atomicAdd(o, t_wait);
        atomicAdd(o + 1, t_cons);
        atomicAdd(o + 2, (unsigned long long)nk);
        atomicAdd(o + 3, t_comp);
    }
    if (!__syncthreads_and(ok))
        return false;
    trace_mark(P, tr);
    // Unit sums over the segments in order, a thread per unit.
    for (uint32_t ul = threadIdx.x; ul < r.count; ul += blockDim.x)
    {
        float sums[NM];
#pragma unroll
        for (int m = 0; m < NM; ++m)
        {
            float a = 0.f;
            for (uint32_t ks = 0; ks < g.Ks; ++ks)
                a += part[ks * pitch + ul * NM + m];
            sums[m] = a;
        }
        persist_epilogue<TP>(P, kind, lw, r.u0 + ul, sums, pos);
    }
    return true;
}

// Attention of one layer over (head, key-split) items, at most one per CTA: the scores node
// s_j = fp16(scale * q.k_j), the softmax node p_j = fp16(exp(s_j - M) / L) with M, L over the
// whole head, and the attention output fp16(sum_j p_j v_j). A split publishes its (max, sum exp)
// and waits (bounded) for its sibling splits' statistics on a per-head counter instead of a grid
// barrier; the last split of a head to publish its partial output combines the splits in order.
// Keys are read `lpk` lanes per key (8 fp16 per lane). For Lk == hd the reference reads V as
// [hd, Lk] (src/core/vkllm_op_matmul.c:14-30): split 0 then computes o[w] = sum_k p_k V[w][k] from
// the stored scores and the other splits contribute 0. `aepoch` counts the attention phases of
// this launch. Returns false on a timed-out wait or a reported error.
template <bool FINE, bool TRACE>
__device__ __forceinline__ bool persist_attention(const PersistParams &P, uint32_t layer, uint32_t pos,
                                                  uint32_t aepoch, float *scratch, float *red)
{
    const DecodeDims &dd = P.dd;
    const LayerW &lw = P.layers[layer];
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    const uint32_t Lk = pos + 1, ns = P.att_split, hd = dd.hd, pieces = hd / 8;
    uint32_t lpk = 1;
    while (lpk < pieces)
        lpk <<= 1;
    const uint32_t G = min(P.att_groups, nt / lpk), gi = tid / lpk, pc = tid % lpk;
    const bool lane_on = gi < G && pc < pieces;
    const uint32_t chunk = (Lk + ns - 1) / ns, hd_al = (hd + 31) & ~31u;
    float *qs = scratch;             // [hd]
    float *sc = qs + hd_al;          // [chunk] this split's scores
    float *acc = sc + ((chunk + 31) & ~31u); // [G][hd] per-group partial outputs
    __shared__ uint32_t flag_s;
    const uint32_t target = ns * (aepoch + 1);
    // tracing: CTA 0's thread 0 stamps the sub-steps of each item in shared memory (no live registers)
    __shared__ long long att_ts[kAttTraceSlots];
    auto amark = [&](uint32_t k) {
        if (TRACE && P.wtrace && blockIdx.x == 0 && threadIdx.x == 0)
            att_ts[k] = clock64();
    };
    for (uint32_t it = blockIdx.x; it < dd.H * ns; it += gridDim.x)
    {
        amark(0);
        const uint32_t h = it / ns, split = it % ns;
        const uint32_t j0 = split * chunk, j1 = min(Lk, j0 + chunk);
        const uint32_t nkeys = j1 > j0 ? j1 - j0 : 0, rounds = (nkeys + G - 1) / G;
        for (uint32_t d = tid; d < hd; d += nt)
            qs[d] = __half2float(__ldcg(P.q + h * hd + d));
        __syncthreads();
        amark(1);
        // lane piece pc of key row j: krow[j * pieces], of value row j: vrow[j * pieces]
        const uint4 *krow = reinterpret_cast<const uint4 *>(lw.kcache + (uint64_t)h * dd.ctx * hd) + pc;
        const uint4 *vrow = reinterpret_cast<const uint4 *>(lw.vcache + (uint64_t)h * dd.ctx * hd) + pc;
        auto load_row = [&](const uint4 *rows, uint32_t j) {
            return (lane_on && j < j1) ? __ldcg(rows + (uint64_t)j * pieces) : make_uint4(0, 0, 0, 0);
        };
        float mx = -FLT_MAX;
        // this lane's 8 query values stay in registers for all its keys
        float qr[8];
        {
            const float4 a = lane_on ? *reinterpret_cast<const float4 *>(qs + 8 * pc) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 b = lane_on ? *reinterpret_cast<const float4 *>(qs + 8 * pc + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            qr[0] = a.x, qr[1] = a.y, qr[2] = a.z, qr[3] = a.w, qr[4] = b.x, qr[5] = b.y, qr[6] = b.z, qr[7] = b.w;
        }
        // scores of key j (every lane calls it: the lpk lanes of a key sum with shuffles)
        auto score_key = [&](const uint4 &raw, uint32_t j) {
            const bool valid = lane_on && j < j1;
            float a = 0.f;
            if (valid)
            {
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
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
            if (valid)
            {
                const float s = round_f16(a * dd.scale);
                if (pc == 0)
                {
                    sc[j - j0] = s;
                    P.scores[(uint64_t)h * dd.ctx + j] = __float2half_rn(s);
                }
                mx = fmaxf(mx, s);
            }
        };
        // The key rows of the first kAttWindow rounds load at once; later rounds one round ahead.
        uint4 win[kAttWindow];
#pragma unroll
        for (uint32_t r = 0; r < kAttWindow; ++r)
            win[r] = load_row(krow, j0 + gi + G * r);
        uint4 nxt = load_row(krow, j0 + gi + G * kAttWindow);
#pragma unroll
        for (uint32_t r = 0; r < kAttWindow; ++r)
            if (r < rounds)
                score_key(win[r], j0 + gi + G * r);
        for (uint32_t rr = kAttWindow; rr < rounds; ++rr)
        {
            const uint4 raw = nxt;
            if (rr + 1 < rounds)
                nxt = load_row(krow, j0 + gi + G * (rr + 1));
            score_key(raw, j0 + gi + G * rr);
        }
        amark(2);
        // the value rows of the window load while the statistics are reduced and the siblings wait
        if (Lk != hd)
        {
#pragma unroll
            for (uint32_t r = 0; r < kAttWindow; ++r)
                win[r] = load_row(vrow, j0 + gi + G * r);
        }
        // this split's max and sum of exp (the reference's reductions over the whole row, in parts)
        mx = warp_max(mx);
        if ((tid & 31) == 0)
            red[tid >> 5] = mx;
        __syncthreads();
        float m = -FLT_MAX;
        for (uint32_t w = 0; w < (nt >> 5); ++w)
            m = fmaxf(m, red[w]);
        float l = 0.f;
        for (uint32_t j = tid; j < nkeys; j += nt)
            l += expf(sc[j] - m);
        __syncthreads();
        l = block_sum(l, red);
        amark(3);
        if (tid == 0)
        {
            bool ok = true;
            P.part[h * ns + split] = make_float2(nkeys ? m : -FLT_MAX, nkeys ? l : 0.f);
            uint32_t prev;
            asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.head_cnt + h) : "memory");
            if (prev + 1 < target)
            {
                const uint64_t t0 = global_ns();
                while (ld_acquire_u32(P.head_cnt + h) < target)
                {
                    if (ld_acquire_u32(P.err) != 0)
                    {
                        ok = false;
                        break;
                    }
                    if (global_ns() - t0 > kWaitLimitNs)
                    {
                        atomicOr(P.err, kErrBarrierTimeout);
                        ok = false;
                        break;
                    }
                }
            }
            flag_s = ok ? 1u : 0u;
        }
        __syncthreads();
        if (!flag_s)
            return false;
        amark(4);
        // the head's max and sum over its splits (ns <= 32: one lane per split), broadcast in smem
        if (tid < 32)
        {
            const float2 pl = tid < ns ? __ldcg(P.part + h * ns + tid) : make_float2(-FLT_MAX, 0.f);
            const float Mw = warp_max(pl.x);
            const float Lw = warp_sum(pl.y > 0.f ? pl.y * expf(pl.x - Mw) : 0.f);
            if (tid == 0)
            {
                red[0] = Mw;
                red[1] = Lw;
            }
        }
        __syncthreads();
        amark(5);
        const float M = red[0], L = red[1];
        const __half *vb = lw.vcache + (uint64_t)h * dd.ctx * hd;
        float *op = P.opart + ((uint64_t)h * ns + split) * hd;
        if (Lk == hd)
        {
            for (uint32_t w = tid; w < hd; w += nt)
            {
                float o = 0.f;
                if (split == 0)
                {
                    const __half *vr = vb + (uint64_t)w * hd;
                    const __half *sr = P.scores + (uint64_t)h * dd.ctx;
                    for (uint32_t k = 0; k < Lk; ++k)
                        o = fmaf(round_f16(expf(__half2float(__ldcg(sr + k)) - M) / L), __half2float(__ldcg(vr + k)),
                                 o);
                }
                op[w] = o;
            }
        }
        else
        {
            // the softmax node's output p_j = fp16(exp(s_j - M) / L), once per key, in place of s_j
            for (uint32_t i = tid; i < nkeys; i += nt)
                sc[i] = round_f16(expf(sc[i] - M) / L);
            __syncthreads();
            float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            auto accumulate = [&](const uint4 &raw, uint32_t j) {
                if (lane_on && j < j1)
                {
                    const float pj = sc[j - j0];
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                    {
                        const float2 f = __half22float2(hh[e]);
                        a[2 * e] = fmaf(pj, f.x, a[2 * e]);
                        a[2 * e + 1] = fmaf(pj, f.y, a[2 * e + 1]);
                    }
                }
            };
            uint4 vn = load_row(vrow, j0 + gi + G * kAttWindow);
#pragma unroll
            for (uint32_t r = 0; r < kAttWindow; ++r)
                if (r < rounds)
                    accumulate(win[r], j0 + gi + G * r);
            for (uint32_t rr = kAttWindow; rr < rounds; ++rr)
            {
                const uint4 raw = vn;
                if (rr + 1 < rounds)
                    vn = load_row(vrow, j0 + gi + G * (rr + 1));
                accumulate(raw, j0 + gi + G * rr);
            }
            // the key groups of a warp (32 / lpk of them) are summed with shuffles, then the warps'
            // sums in smem, in warp order
#pragma unroll
            for (int e = 0; e < 8; ++e)
                for (uint32_t o = lpk; o < 32; o <<= 1)
                    a[e] += __shfl_xor_sync(0xffffffffu, a[e], o);
            const uint32_t lane = tid & 31, nwarp = nt >> 5;
            if (lane < lpk && pc < pieces)
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    acc[(tid >> 5) * hd + 8 * pc + e] = a[e];
            __syncthreads();
            // the warps' rows summed by 4 threads per output (warps q, q + 4, ...), then 2 shuffles
            for (uint32_t t = tid; t < ((4 * hd + 31) & ~31u); t += nt)
            {
                const uint32_t d = t >> 2, qq = t & 3;
                float o = 0.f;
                if (d < hd)
                    for (uint32_t w = qq; w < nwarp; w += 4)
                        o += acc[w * hd + d];
                o += __shfl_xor_sync(0xffffffffu, o, 1);
                o += __shfl_xor_sync(0xffffffffu, o, 2);
                if (qq == 0 && d < hd)
                    op[d] = o;
            }
        }
        __syncthreads();
        amark(6);
        if (tid == 0)
        {
            uint32_t prev;
            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.head_done + h) : "memory");
            flag_s = prev + 1 == target ? 1u : 0u; // the head's last split combines
        }
        __syncthreads();
        if (flag_s)
            for (uint32_t d = tid; d < hd; d += nt)
            {
                float o = 0.f;
#pragma unroll 4
                for (uint32_t c = 0; c < ns; ++c)
                    o += __ldcg(P.opart + ((uint64_t)h * ns + c) * hd + d);
                P.attn[h * hd + d] = __float2half_rn(o);
            }
        __syncthreads();
        if (FINE && flag_s && tid == 0) // the head's output is complete: the Wo tiles reading it may start
        {
            __threadfence();
            st_release_gpu_u32(P.head_flag + h, aepoch + 1);
        }
        amark(7);
        if (TRACE && P.wtrace && blockIdx.x == 0 && threadIdx.x == 0)
        {
            for (uint32_t k = 0; k + 1 < kAttTraceSlots; ++k)
                atomicAdd(P.wtrace + kAttTraceBase + k, (unsigned long long)(att_ts[k + 1] - att_ts[k]));
            atomicAdd(P.wtrace + kAttTraceBase + kAttTraceSlots - 1, 1ull);
        }
    }
    return true;
}

// Stages the RMSNORM node's output fp16((x * g) * rsqrt(mean(x^2) + eps)) as fp16 (x read from L2).
__device__ __forceinline__ void stage_rmsnorm_h(const __half *__restrict__ x, const float *__restrict__ g, uint32_t K,
                                                float eps, __half *xs, float *red)
{
    const uint32_t nchunk = K / 8;
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    // one 16-byte chunk per thread is kept in registers between the two passes (K <= 8 * threads)
    const bool one = nchunk <= blockDim.x;
    const uint4 v0 = (one && threadIdx.x < nchunk) ? __ldcg(x4 + threadIdx.x) : make_uint4(0, 0, 0, 0);
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < nchunk; i += blockDim.x)
    {
        const uint4 v = one ? v0 : __ldcg(x4 + i);
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const float2 f = __half22float2(h[j]);
            s = fmaf(f.x, f.x, s);
            s = fmaf(f.y, f.y, s);
        }
    }
    const float alpha = rsqrtf(block_sum(s, red) / (float)K + eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    uint4 *xs4 = reinterpret_cast<uint4 *>(xs);
    for (uint32_t i = threadIdx.x; i < nchunk; i += blockDim.x)
    {
        const uint4 v = one ? v0 : __ldcg(x4 + i);
        const float4 ga = g4[2 * i], gb = g4[2 * i + 1];
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        uint4 o;
        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const float2 f = __half22float2(h[j]);
            oh[j] = __floats2half2_rn((f.x * gg[2 * j]) * alpha, (f.y * gg[2 * j + 1]) * alpha);
        }
        xs4[i] = o;
    }
    __syncthreads();
}

// Stages an fp16 vector written by other CTAs (read from L2).
__device__ __forceinline__ void stage_copy_h(const __half *__restrict__ x, uint32_t K, __half *xs)
{
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    uint4 *xs4 = reinterpret_cast<uint4 *>(xs);
    for (uint32_t i = threadIdx.x; i < K / 8; i += blockDim.x)
        xs4[i] = __ldcg(x4 + i);
    __syncthreads();
}

// TP: tensor parallelism (P.tp_size > 1); FINE: the fine-grained Wo and down phases (P.fine); TRACE:
// the per-warp pipeline accounting (P.wtrace). Each combination is its own instantiation, so the
// kernel a launch runs holds no code of the others (their branches cost time in the tile loops).
template <bool TP, bool FINE, bool TRACE>
__global__ void __launch_bounds__(kPersistMaxWarps * 32, 1) k_decode_persistent(PersistParams P)
{
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    __half *xs = reinterpret_cast<__half *>(smem + kStreamBarBytes);
    float *part = reinterpret_cast<float *>(smem + kStreamBarBytes + P.xs_bytes);
    float *scratch = reinterpret_cast<float *>(smem + kStreamBarBytes); // attention phases: xs + part
    unsigned char *stages = smem + kStreamBarBytes + P.xs_bytes + P.part_bytes;
    __shared__ float sred[32];
    __shared__ uint32_t xfail_s; // the tensor-parallel argmax exchange timed out

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const DecodeDims &dd = P.dd;
    WarpPipe wp;
    wp.bar = bars + warp * P.spw;
    wp.stage = stages + (size_t)warp * P.spw * kTileBytes;
    wp.consumed = 0;
    wp.issued = 0;
    // this CTA's units of every phase (the cursor needs them first)
    if (threadIdx.x < PK_COUNT)
    {
        const uint32_t *t = P.utab + threadIdx.x * (gridDim.x + 1) + blockIdx.x;
        s_units[threadIdx.x] = UnitRange{__ldg(t), __ldg(t + 1) - __ldg(t)};
    }
    __syncthreads();
    wp.cur = Cursor{};
    wp.cur.kind = PK_QKV;
    wp.cur.done = P.n_steps == 0;
    if (!wp.cur.done)
        cursor_enter(P, wp.cur, warp);
    bool ok = true;
    SyncState tr{1, 0}; // thread 0: trace entry 0 is the start
    if (P.trace_cta && threadIdx.x == 0) // the last row of the arrival trace: each CTA's SM
    {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        P.trace_cta[(uint64_t)(kCtaTraceBarriers - 1) * gridDim.x + blockIdx.x] = smid;
    }
    if (threadIdx.x == 0)
        xfail_s = 0;
    if (P.trace && blockIdx.x == 0 && threadIdx.x == 0 && P.trace_cap > 0)
        P.trace[0] = global_ns();
    if (lane == 0)
    {
        for (uint32_t s = 0; s < P.spw; ++s)
            mbar_init(&wp.bar[s], 1);
        fence_barrier_init();
        fence_proxy_async();
    }
    __syncwarp();
    wp.policy = P.l2_hint ? l2_evict_first_policy() : 0;
    cursor_settle(P, wp.cur, warp);
    // Fill every stage: the first weights do not depend on anything.
    while (!wp.cur.done && wp.issued < P.spw)
    {
        cursor_issue(P, wp.cur, warp, wp.stage + (size_t)wp.issued * kTileBytes, &wp.bar[wp.issued], wp.policy);
        ++wp.issued;
        ++wp.cur.k;
        tile_step(wp.cur.grp, wp.cur.ks, wp.cur.Ks, P.warps);
        cursor_settle(P, wp.cur, warp);
    }

    // Every CTA tracks the token and position itself (each computes the same argmax); CTA 0
    // publishes them to the step state for the host.
    uint32_t pos = __ldcg(&P.st->pos), tok0 = __ldcg(&P.st->token);
    for (uint32_t step = 0; ok && step < P.n_steps; ++step)
    {
        if (pos >= dd.ctx)
        {
            if (blockIdx.x == 0 && threadIdx.x == 0)
                atomicOr(P.err, kErrPosition);
            ok = false;
            break;
        }
        const uint32_t tok = tok0 < P.Vg ? tok0 : P.unk; // src/shaders/vkllm_embedding.comp:57-60
        // The residual rows this CTA owns (the Wo / down output rows) start as the embedding.
        {
            const UnitRange r = cta_units(PK_WO);
            for (uint32_t i = threadIdx.x; i < r.count; i += blockDim.x)
                P.x[r.u0 + i] = P.embed[(uint64_t)tok * dd.D + r.u0 + i];
        }
        for (uint32_t l = 0; ok && l < P.L; ++l)
        {
            const LayerW &lw = P.layers[l];
            if (l == 0)
                stage_rmsnorm_h(P.embed + (uint64_t)tok * dd.D, lw.attn_norm, dd.D, dd.eps, xs, sred);
            else
                stage_rmsnorm_h(P.x, lw.attn_norm, dd.D, dd.eps, xs, sred);
            trace_mark(P, tr);
            ok = persist_gemv<2, TP, TRACE>(P, PK_QKV, l, wp, xs, part, pos, tr);
            if (threadIdx.x == 0)
                prefetch_slice(P, PK_WO, l);
            if (!__syncthreads_and(ok) || !grid_sync(P, tr))
            {
                ok = false;
                break;
            }
            if constexpr (FINE)
            {
                // Wo tiles wait only for the heads their input columns span
                if (!persist_attention<FINE, TRACE>(P, l, pos, step * P.L + l, scratch, sred))
                {
                    ok = false;
                    break;
                }
                if (threadIdx.x < kFineMaxSegs)
                    s_seg[threadIdx.x] = 0;
                __syncthreads();
                trace_mark(P, tr);
                ok = persist_gemv<1, TP, TRACE, true>(P, PK_WO, l, wp, xs, part, pos, tr, step * P.L + l + 1);
            }
            else
            {
                if (!persist_attention<FINE, TRACE>(P, l, pos, step * P.L + l, scratch, sred) || !grid_sync(P, tr))
                {
                    ok = false;
                    break;
                }
                stage_copy_h(P.attn, dd.H * dd.hd, xs);
                trace_mark(P, tr);
                ok = persist_gemv<1, TP, TRACE>(P, PK_WO, l, wp, xs, part, pos, tr);
            }
            if (threadIdx.x == 0)
                prefetch_slice(P, PK_UPGATE, l);
            if (TP && __syncthreads_and(ok))
                ok = tp_allreduce_rows(P, 0, P.tp_base[0] + step * P.L + l + 1);
            if (!__syncthreads_and(ok) || !grid_sync(P, tr))
            {
                ok = false;
                break;
            }
            stage_rmsnorm_h(P.x, lw.ffn_norm, dd.D, dd.eps, xs, sred);
            trace_mark(P, tr);
            ok = persist_gemv<2, TP, TRACE>(P, PK_UPGATE, l, wp, xs, part, pos, tr);
            if (threadIdx.x == 0)
                prefetch_slice(P, PK_DOWN, l);
            if constexpr (FINE)
            {
                // publish this CTA's up/gate rows, then stage the down input segment by segment
                const uint32_t fe = step * P.L + l + 1;
                if (!__syncthreads_and(ok))
                {
                    ok = false;
                    break;
                }
                if (threadIdx.x == 0)
                {
                    __threadfence();
                    st_release_gpu_u32(P.cta_flag + blockIdx.x, fe);
                }
                if (threadIdx.x < kFineMaxSegs)
                    s_seg[threadIdx.x] = 0;
                __syncthreads();
                trace_mark(P, tr);
                ok = persist_gemv<1, TP, TRACE, true>(P, PK_DOWN, l, wp, xs, part, pos, tr, fe);
            }
            else
            {
                if (!__syncthreads_and(ok) || !grid_sync(P, tr))
                {
                    ok = false;
                    break;
                }
                stage_copy_h(P.m, dd.F, xs);
                trace_mark(P, tr);
                ok = persist_gemv<1, TP, TRACE>(P, PK_DOWN, l, wp, xs, part, pos, tr);
            }
            if (threadIdx.x == 0)
                prefetch_slice(P, l + 1 < P.L ? PK_QKV : PK_LOGITS, l + 1 < P.L ? l + 1 : 0);
            if (TP && __syncthreads_and(ok))
                ok = tp_allreduce_rows(P, 1, P.tp_base[1] + step * P.L + l + 1);
            if (!__syncthreads_and(ok) || !grid_sync(P, tr))
            {
                ok = false;
                break;
            }
        }
        if (!ok)
            break;
        stage_rmsnorm_h(P.x, P.out_norm, dd.D, dd.eps, xs, sred);
        trace_mark(P, tr);
        ok = persist_gemv<1, TP, TRACE>(P, PK_LOGITS, 0, wp, xs, part, pos, tr);
        if (threadIdx.x == 0 && step + 1 < P.n_steps)
            prefetch_slice(P, PK_QKV, 0);
        if (!__syncthreads_and(ok))
        {
            ok = false;
            break;
        }
        // Per-CTA argmax partials over its logits rows, per class i mod 32: the first (smallest
        // index) strict maximum (src/shaders/vkllm_arg_max.comp:54-69).
        {
            const UnitRange r = cta_units(PK_LOGITS);
            if (warp == 0)
            {
                // class of a row = its vocabulary index (v0 + local row) mod 32
                float bv = -FLT_MAX;
                uint32_t bi = 0xffffffffu;
                const uint32_t first = r.u0 + ((lane + 32 - ((P.v0 + r.u0) & 31)) & 31);
                for (uint32_t i = first; i < r.u0 + r.count; i += 32)
                {
                    const float v = __half2float(__ldcg(P.logits + i));
                    if (bi == 0xffffffffu || v > bv)
                    {
                        bv = v;
                        bi = P.v0 + i;
                    }
                }
                P.am_val[blockIdx.x * 32 + lane] = bv;
                P.am_idx[blockIdx.x * 32 + lane] = bi;
            }
        }
        if (!grid_sync(P, tr))
        {
            ok = false;
            break;
        }
        // Every CTA combines the partials: class `lane` over the CTAs (warps take CTAs w, w + nw,
        // ...; the largest value wins, ties to the smallest index, which is the in-order scan's
        // result since a class's indices grow with the CTA), then the 16/8/4/2/1 tree over the
        // classes that keeps the left operand unless the right one is strictly greater
        // (vkllm_arg_max.comp:77-90).
        {
            float *cv_s = scratch;                                              // [nw][32]
            uint32_t *ci_s = reinterpret_cast<uint32_t *>(scratch + 32 * 32); // [nw][32]
            const uint32_t nw = blockDim.x >> 5;
            float v = -FLT_MAX;
            uint32_t idx = 0xffffffffu;
            for (uint32_t b = warp; b < gridDim.x; b += nw)
            {
                const uint32_t ci = __ldcg(P.am_idx + b * 32 + lane);
                const float cv = __ldcg(P.am_val + b * 32 + lane);
                if (ci == 0xffffffffu)
                    continue;
                if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))
                {
                    v = cv;
                    idx = ci;
                }
            }
            cv_s[warp * 32 + lane] = v;
            ci_s[warp * 32 + lane] = idx;
            __syncthreads();
            if (warp == 0)
            {
                v = -FLT_MAX;
                idx = 0xffffffffu;
                for (uint32_t w = 0; w < nw; ++w)
                {
                    const uint32_t ci = ci_s[w * 32 + lane];
                    const float cv = cv_s[w * 32 + lane];
                    if (ci == 0xffffffffu)
                        continue;
                    if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))
                    {
                        v = cv;
                        idx = ci;
                    }
                }
                if constexpr (TP)
                {
                    // this rank's class results -> every rank (CTA 0 sends), then every CTA combines the
                    // ranks' results per class with the same rule (indices grow with the rank)
                    const uint32_t epoch = P.tp_base[2] + step + 1;
                    if (blockIdx.x == 0)
                    {
                        for (uint32_t q = 0; q < P.tp_size; ++q)
                        {
                            P.tp_amv[q][P.tp_rank * 32 + lane] = v;
                            P.tp_ami[q][P.tp_rank * 32 + lane] = idx;
                        }
                        __syncwarp();
                        if (lane == 0)
                        {
                            __threadfence_system();
                            for (uint32_t q = 0; q < P.tp_size; ++q)
                                st_relaxed_sys_u32(P.tp_flag[q] + (2 * kTpCtas) * kTpMax + P.tp_rank, epoch);
                        }
                    }
                    bool okw = true;
                    if (lane == 0)
                    {
                        const uint32_t *mine = P.tp_flag[P.tp_rank] + (2 * kTpCtas) * kTpMax;
                        const uint64_t t0 = global_ns();
                        for (uint32_t q = 0; q < P.tp_size && okw; ++q)
                            while (ld_acquire_sys_u32(mine + q) < epoch)
                            {
                                if (ld_acquire_u32(P.err) != 0 || global_ns() - t0 > kWaitLimitNs)
                                {
                                    atomicOr(P.err, kErrPeerTimeout);
                                    okw = false;
                                    break;
                                }
                            }
                    }
                    okw = __shfl_sync(0xffffffffu, okw, 0);
                    v = -FLT_MAX;
                    idx = 0xffffffffu;
                    for (uint32_t q = 0; okw && q < P.tp_size; ++q)
                    {
                        const uint32_t ci = __ldcg(P.tp_ami[P.tp_rank] + q * 32 + lane);
                        const float cv = __ldcg(P.tp_amv[P.tp_rank] + q * 32 + lane);
                        if (ci == 0xffffffffu)
                            continue;
                        if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))
                        {
                            v = cv;
                            idx = ci;
                        }
                    }
                    if (!okw && lane == 0)
                        xfail_s = 1u;
                }
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
                    ci_s[0] = idx;
                    if (blockIdx.x == 0)
                    {
                        P.st->token = idx;
                        if (P.st->step < P.ring_len)
                            P.ring[P.st->step] = idx;
                        P.st->step += 1;
                        P.st->pos = pos + 1;
                    }
                }
            }
            __syncthreads();
            tok0 = ci_s[0];
            pos += 1;
            const bool xfail = xfail_s != 0;
            __syncthreads();
            if (xfail)
            {
                ok = false;
                break;
            }
        }
    }
    if (!ok)
    {
        if (threadIdx.x == 0)
            atomicOr(P.err, kErrMbarTimeout);
    }
    // Copies this warp issued and did not consume must land before the shared memory is released
    // (none on the normal path: the cursor stops after the last step).
    for (uint32_t gi = wp.consumed; gi < wp.issued; ++gi)
        (void)mbar_wait_bounded(&wp.bar[gi % P.spw], (gi / P.spw) & 1u, kWaitLimitNs / 4);
    __syncwarp();
}

using PersistKernel = void (*)(PersistParams);

// The instantiation for tensor parallelism `tp`, the fine-grained phases `fine` and tracing `trace`.
inline PersistKernel persist_kernel(bool tp, bool fine, bool trace)
{
    if (trace)
    {
        if (tp)
            return fine ? k_decode_persistent<true, true, true> : k_decode_persistent<true, false, true>;
        return fine ? k_decode_persistent<false, true, true> : k_decode_persistent<false, false, true>;
    }
    if (tp)
        return fine ? k_decode_persistent<true, true, false> : k_decode_persistent<true, false, false>;
    return fine ? k_decode_persistent<false, true, false> : k_decode_persistent<false, false, false>;
}

} // namespace vkb
