// Fused decode engine: owns the decode workspace of one model, captures one decode step as a CUDA
// Graph, and runs it for vkllm_graph_run (graphs carrying a plan) and for the device-resident
// token loop of vkllm_b200.h.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../runtime/internal.h"
#include "decode_kernels.cuh"
#include "decode_persistent.cuh"
#include "nccl_api.h"
#include "plan.h"
#include "prefill_kernels.cuh"
#include "../kernels/kernels.h"
#include "vkllm_b200.h"
#include "vkllm_kvcache.h"
#include "vkllm_models_llama2.h"

namespace vkb
{

struct TpComm;

struct Engine
{
    vkllm_context *ctx = nullptr;
    DecodeDims dd{};
    std::vector<LayerW> layers;
    const __half *embed = nullptr, *wout = nullptr;
    const float *out_norm = nullptr;
    uint32_t unk = 0;
    // workspace
    void *ws = nullptr;
    __half *x = nullptr, *q = nullptr, *attn = nullptr, *m = nullptr, *logits = nullptr, *scores = nullptr;
    float2 *part = nullptr;
    float *opart = nullptr;
    uint32_t *counters = nullptr, *logit_counter = nullptr, *ring = nullptr;
    StepState *state = nullptr;
    // launch geometry
    unsigned grid_stream = 0, grid_embed = 0;
    StreamGeom g_qkv{}, g_wo{}, g_upgate{}, g_down{}, g_logits{};
    // captured step
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint32_t kernels_per_step = 0;
    // persistent decode (one cooperative launch runs n steps)
    bool persistent = false;
    PersistParams pp{};
    size_t pp_smem = 0;
    LayerW *d_layers = nullptr;
    float *am_val = nullptr;
    uint32_t *am_idx = nullptr, *bar = nullptr; // bar[0] = barrier arrivals, then 2 x H attention counters
    uint32_t launches = 0;                      // kernel launches enqueued by the last decode call
    TpComm *tp = nullptr;                       // tensor-parallel exchange (shards only)
    bool tp_nccl = false;                       // shards decode on the per-op kernels + NCCL collectives
    float *tp_sum = nullptr;                    // [D] this rank's Wo / down partials, then their allreduce
    uint32_t *tp_cls = nullptr, *tp_cls_all = nullptr; // argmax class candidates: [64], [world][64]
    __half *tiled = nullptr;                    // decode copy of the weights (persistent kernel's tile layout)
    void *d_tiled_ptrs = nullptr;               // [layer * 4 + phase] pointers into `tiled`
    float *rope_den = nullptr;                  // RoPE denominators of the persistent kernel
    // persistent kernel's row partition: [kind][grid + 1] prefix offsets of each CTA's units
    std::vector<uint32_t> htab;
    uint32_t *utab = nullptr;                   // htab on the device, then the down-phase segment producers
    std::vector<uint32_t> seg_host;             // [2 * kFineMaxSegs] first / last producer CTA per segment
    uint32_t unit_cap[PK_COUNT] = {}; // most units a CTA may hold in a phase (sizes the partials)
    // fused prefill (graphs with S > 1): workspace grown to the largest S seen
    void *pf_ws = nullptr;
    size_t pf_cap = 0;
};

// Peer-memory exchange of a tensor-parallel rank: one device buffer, exported with CUDA IPC, holding
// the receive areas and flags its peers write into (layout in tp_layout), plus the peers' buffers
// opened from their handles.
struct TpComm
{
    uint32_t rank = 0, world = 1, D = 0;
    void *buf = nullptr;
    size_t bytes = 0;
    void *peer[kTpMax] = {};
    bool connected = false;
    uint32_t base[3] = {0, 0, 0}; // exchanges done per site (Wo, down, argmax)
    ncclComm_t nccl = nullptr;    // the NCCL exchange's communicator (vkllm_b200_tp_nccl_connect)
};

struct TpLayout
{
    size_t x, flag, amv, ami, total;
};

inline TpLayout tp_layout(uint32_t world, uint32_t D)
{
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    TpLayout t;
    t.x = 0;
    (void)D;
    t.flag = t.x + al((size_t)2 * world * kTpCtas * kTpRows * 8); // 8-byte (epoch, value) slots
    t.amv = t.flag + al((size_t)3 * kTpCtas * kTpMax * 4);
    t.ami = t.amv + al((size_t)kTpMax * 32 * 4);
    t.total = t.ami + al((size_t)kTpMax * 32 * 4);
    return t;
}

namespace
{

// Launch with Programmatic Dependent Launch enabled: the kernel may start while its predecessor in
// the stream finishes; every decode kernel calls griddepcontrol.wait before reading its inputs.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

QkvOp op_qkv(Engine *e, const LayerW &lw)
{
    return QkvOp{lw, e->dd, e->x, e->q, e->state};
}
WoOp op_wo(Engine *e, const LayerW &lw)
{
    return WoOp{lw, e->dd, e->attn, e->x, e->tp_nccl ? e->tp_sum : nullptr};
}
UpGateOp op_upgate(Engine *e, const LayerW &lw)
{
    return UpGateOp{lw, e->dd, e->x, e->m};
}
DownOp op_down(Engine *e, const LayerW &lw)
{
    return DownOp{lw, e->dd, e->m, e->x, e->tp_nccl ? e->tp_sum : nullptr};
}
LogitsOp op_logits(Engine *e)
{
    return LogitsOp{e->wout,  e->out_norm,  e->dd,  e->x, e->logits, e->logit_counter, e->state, e->ring, e->dd.ctx,
                    e->pp.v0, e->tp_nccl ? e->tp_cls : nullptr};
}

// Tensor parallel (NCCL exchange): the ranks' partial rows summed in place (fp32), then the
// projection's rounding and the residual add.
cudaError_t tp_allreduce_residual(Engine *e, cudaStream_t s)
{
    const NcclApi *nc = nccl_api();
    ncclResult_t r = nc->AllReduce(e->tp_sum, e->tp_sum, e->dd.D, ncclFloat32, ncclSum, e->tp->nccl, s);
    if (r != ncclSuccess)
    {
        log_error("ncclAllReduce: %s", nc->GetErrorString(r));
        return cudaErrorUnknown;
    }
    k_tp_residual<<<(e->dd.D + 255) / 256, 256, 0, s>>>(e->x, e->tp_sum, e->dd.D);
    return cudaGetLastError();
}

template <class Op> cudaError_t launch_stream(Engine *e, const Op &op, const StreamGeom &g, cudaStream_t s)
{
    return launch_pdl(k_gemv_stream<Op>, dim3(e->grid_stream), dim3(32 * g.warps), stream_smem_bytes(g), s, op, g,
                      &e->state->error);
}

vkllm_err_t enqueue_step(Engine *e, cudaStream_t s)
{
    const DecodeDims &dd = e->dd;
    // the embedding table is whole on every rank: ids below the full vocabulary size are valid
    cudaError_t err = launch_pdl(k_dec_embed, dim3(e->grid_embed), dim3(256), 0, s, e->embed, e->pp.Vg, dd.D, e->unk,
                                 (const StepState *)e->state, e->x);
    dim3 agrid(dd.H, dd.nsplit);
    for (const LayerW &lw : e->layers)
    {
        if (err == cudaSuccess)
            err = launch_stream(e, op_qkv(e, lw), e->g_qkv, s);
        if (err == cudaSuccess)
            err = launch_pdl(k_dec_attn_scores, agrid, dim3(kAttnThreads), 0, s, lw, dd, (const __half *)e->q,
                             e->scores, e->part, (const StepState *)e->state);
        if (err == cudaSuccess)
            err = launch_pdl(k_dec_attn_pv, agrid, dim3(kAttnThreads), 0, s, lw, dd, (const __half *)e->scores,
                             (const float2 *)e->part, e->opart, e->counters, e->attn, (const StepState *)e->state);
        if (err == cudaSuccess)
            err = launch_stream(e, op_wo(e, lw), e->g_wo, s);
        if (err == cudaSuccess && e->tp_nccl)
            err = tp_allreduce_residual(e, s);
        if (err == cudaSuccess)
            err = launch_stream(e, op_upgate(e, lw), e->g_upgate, s);
        if (err == cudaSuccess)
            err = launch_stream(e, op_down(e, lw), e->g_down, s);
        if (err == cudaSuccess && e->tp_nccl)
            err = tp_allreduce_residual(e, s);
    }
    if (err == cudaSuccess)
        err = launch_stream(e, op_logits(e), e->g_logits, s);
    if (err == cudaSuccess && e->tp_nccl)
    {
        const NcclApi *nc = nccl_api();
        ncclResult_t r = nc->AllGather(e->tp_cls, e->tp_cls_all, 64, ncclUint32, e->tp->nccl, s);
        if (r != ncclSuccess)
        {
            log_error("ncclAllGather: %s", nc->GetErrorString(r));
            err = cudaErrorUnknown;
        }
        else
        {
            k_tp_argmax<<<1, 32, 0, s>>>(e->tp_cls_all, e->tp->world, e->state, e->ring, dd.ctx);
            err = cudaGetLastError();
        }
    }
    if (err == cudaSuccess)
        err = cudaGetLastError();
    if (err != cudaSuccess)
        return cuda_check(err, "decode step launch", __FILE__, __LINE__);
    return VKLLM_ERR_OK;
}

template <class Op> void allow_smem(const StreamGeom &g)
{
    if (cudaFuncSetAttribute(k_gemv_stream<Op>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)stream_smem_bytes(g)) != cudaSuccess)
        log_error("streaming GEMV: %zu bytes of dynamic shared memory refused: %s", stream_smem_bytes(g),
                  cudaGetErrorString(cudaGetLastError()));
}

// Dynamic shared memory a streaming GEMV of this op may use: `cap`, at most the opt-in limit less
// the kernel's static shared memory (the logits op's argmax arrays take 8 KB of it).
template <class Op> uint32_t stream_cap(vkllm_context *ctx, uint32_t cap)
{
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k_gemv_stream<Op>) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return cap;
    }
    const size_t limit = ctx->device->smem_optin > fa.sharedSizeBytes ? ctx->device->smem_optin - fa.sharedSizeBytes : 0;
    return (uint32_t)(cap < limit ? cap : limit);
}

// Persistent decode geometry: every phase kind shares the block size and stage layout.
// Decode copy of one phase matrix (the persistent kernel's tile layout): logical row R (mode 0: rows
// of s0, then s1, then s2; mode 1: rows alternate s0, s1, i.e. up/gate pairs) belongs to the CTA
// owning unit R / nm; within that CTA's rows, 16-row groups, then K segments, are contiguous tiles
// whose rows hold the segment's chunks swizzled by tile_chunk.
// Copies one matrix into the persistent kernel's tile layout. Source row R (mode 1: rows of s0 and s1
// interleaved; else s0, then s1, then s2) belongs to unit R / nm; CTA b owns units [tab[b], tab[b + 1])
// and its rows are contiguous in the copy, as tiles of 16 rows x 256 columns in (row group, segment)
// order, each tile contiguous with its 16-byte chunks swizzled by row (tile_chunk).
__global__ void k_relayout(__half *__restrict__ dst, const __half *s0, const __half *s1, const __half *s2,
                           uint32_t rows0, uint32_t rows1, int mode, uint32_t K, uint32_t total_rows, uint32_t nm,
                           const uint32_t *__restrict__ tab, uint32_t grid)
{
    __shared__ uint32_t st[kPersistMaxGrid + 1];
    for (uint32_t i = threadIdx.x; i <= grid; i += blockDim.x)
        st[i] = tab[i];
    __syncthreads();
    const uint32_t nch = K / 8;
    const uint64_t n = (uint64_t)total_rows * nch;
    const uint32_t Ks = (K + kSegHalves - 1) / kSegHalves, last = K - kSegHalves * (Ks - 1);
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint32_t R = (uint32_t)(t / nch), c = (uint32_t)(t % nch);
        const __half *src;
        if (mode == 1)
            src = ((R & 1u) ? s1 : s0) + (uint64_t)(R >> 1) * K;
        else if (R < rows0)
            src = s0 + (uint64_t)R * K;
        else if (R < rows0 + rows1)
            src = s1 + (uint64_t)(R - rows0) * K;
        else
            src = s2 + (uint64_t)(R - rows0 - rows1) * K;
        const uint32_t u = R / nm;
        uint32_t lo = 0, hi = grid; // st[lo] <= u < st[hi]: the owner is the CTA whose range holds u
        while (hi - lo > 1)
        {
            const uint32_t mid = (lo + hi) >> 1;
            if (st[mid] <= u)
                lo = mid;
            else
                hi = mid;
        }
        const uint32_t b = lo, u0 = st[b], cnt = st[b + 1] - st[b];
        const uint32_t rl = R - u0 * nm, rows_b = cnt * nm;
        const uint32_t g = rl / kTileRows, r = rl % kTileRows, nv = min(kTileRows, rows_b - g * kTileRows);
        const uint32_t ks = c / (kSegHalves / 8), cc = c % (kSegHalves / 8);
        const uint32_t width = ks + 1 == Ks ? last : kSegHalves;
        const uint64_t off = (uint64_t)u0 * nm * K + (uint64_t)g * kTileRows * K + (uint64_t)ks * nv * kSegHalves +
                             (uint64_t)r * width + (uint64_t)tile_chunk(cc, r, width / 8) * 8;
        *reinterpret_cast<uint4 *>(dst + off) = *reinterpret_cast<const uint4 *>(src + (uint64_t)c * 8);
    }
}

__global__ void k_rope_den(float *den, uint32_t half_hd, uint32_t hd, float base)
{
    for (uint32_t w = threadIdx.x; w < half_hd; w += blockDim.x)
        den[w] = powf(base, (float)(2 * w) / (float)hd);
}

// Uploads the row partition (e->htab) and rewrites the decode copy of the weights for it; the
// per-matrix start pointers do not depend on the partition. Enqueued on `st`.
cudaError_t relayout_weights(Engine *e, cudaStream_t st, std::vector<const __half *> *ptrs)
{
    const DecodeDims &dd = e->dd;
    const uint32_t HD = dd.H * dd.hd, L = (uint32_t)e->layers.size(), grid = (uint32_t)e->ctx->device->sm_count;
    cudaError_t err = cudaMemcpyAsync(e->utab, e->htab.data(), sizeof(uint32_t) * e->htab.size(),
                                      cudaMemcpyHostToDevice, st);
    if (err != cudaSuccess)
        return err;
    {
        // producers of each 256-column input segment of the down phase: the first and last CTA whose
        // up/gate units (columns of m) intersect it (fine-grained down phase)
        const uint32_t Ks = e->pp.tg[PK_DOWN].Ks;
        const uint32_t *tu = e->htab.data() + (size_t)PK_UPGATE * (grid + 1);
        e->seg_host.assign(2 * kFineMaxSegs, 0);
        for (uint32_t k = 0; k < Ks && k < kFineMaxSegs; ++k)
        {
            const uint32_t c0 = k * kSegHalves, c1 = std::min(dd.F, c0 + kSegHalves);
            uint32_t first = grid, last = 0;
            for (uint32_t b = 0; b < grid; ++b)
                if (tu[b] < c1 && tu[b + 1] > c0)
                {
                    first = std::min(first, b);
                    last = std::max(last, b);
                }
            e->seg_host[2 * k] = first < grid ? first : 0;
            e->seg_host[2 * k + 1] = first < grid ? last : 0;
        }
        err = cudaMemcpyAsync(e->utab + e->htab.size(), e->seg_host.data(), sizeof(uint32_t) * e->seg_host.size(),
                              cudaMemcpyHostToDevice, st);
        if (err != cudaSuccess)
            return err;
    }
    const uint32_t *tq = e->utab + PK_QKV * (grid + 1), *two = e->utab + PK_WO * (grid + 1),
                   *tu = e->utab + PK_UPGATE * (grid + 1), *td = e->utab + PK_DOWN * (grid + 1),
                   *tl = e->utab + PK_LOGITS * (grid + 1);
    const unsigned rb = grid * 8;
    __half *cur = e->tiled;
    if (ptrs)
        ptrs->assign(4 * L, nullptr);
    for (uint32_t l = 0; l < L; ++l)
    {
        const LayerW &w = e->layers[l];
        if (ptrs)
            (*ptrs)[4 * l + PK_QKV] = cur;
        k_relayout<<<rb, 256, 0, st>>>(cur, w.wq, w.wk, w.wv, HD, HD, 0, dd.D, 3 * HD, 2, tq, grid);
        cur += (size_t)3 * HD * dd.D;
        if (ptrs)
            (*ptrs)[4 * l + PK_WO] = cur;
        k_relayout<<<rb, 256, 0, st>>>(cur, w.wo, nullptr, nullptr, dd.D, 0, 0, HD, dd.D, 1, two, grid);
        cur += (size_t)dd.D * HD;
        if (ptrs)
            (*ptrs)[4 * l + PK_UPGATE] = cur;
        k_relayout<<<rb, 256, 0, st>>>(cur, w.wu, w.wg, nullptr, 0, 0, 1, dd.D, 2 * dd.F, 2, tu, grid);
        cur += (size_t)2 * dd.F * dd.D;
        if (ptrs)
            (*ptrs)[4 * l + PK_DOWN] = cur;
        k_relayout<<<rb, 256, 0, st>>>(cur, w.wd, nullptr, nullptr, dd.D, 0, 0, dd.F, dd.D, 1, td, grid);
        cur += (size_t)dd.D * dd.F;
    }
    k_relayout<<<rb, 256, 0, st>>>(cur, e->wout, nullptr, nullptr, dd.V, 0, 0, dd.D, dd.V, 1, tl, grid);
    e->pp.tiled_logits = cur;
    return cudaGetLastError();
}

void setup_persistent(Engine *e, vkllm_context *ctx, uint32_t att_split, uint32_t spw, uint32_t l2_kb)
{
    const char *mode = getenv("VKLLM_B200_DECODE");
    if (mode && strcmp(mode, "graph") == 0)
        return;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device->ordinal);
    if (!coop)
        return;
    const DecodeDims &dd = e->dd;
    const uint32_t HD = dd.H * dd.hd;
    PersistParams &P = e->pp;
    P.dd = dd;
    P.L = (uint32_t)e->layers.size();
    P.embed = e->embed;
    P.wout = e->wout;
    P.out_norm = e->out_norm;
    P.unk = e->unk;
    P.x = e->x;
    P.q = e->q;
    P.m = e->m;
    P.logits = e->logits;
    P.scores = e->scores;
    P.part = e->part;
    P.opart = e->opart;
    P.am_val = e->am_val;
    P.am_idx = e->am_idx;
    P.st = e->state;
    P.ring = e->ring;
    P.ring_len = dd.ctx;
    P.bar_count = e->bar;
    P.head_cnt = e->bar + 1;
    P.head_done = e->bar + 1 + dd.H;
    P.cta_flag = e->bar + 1 + 2 * dd.H;
    P.head_flag = e->bar + 1 + 2 * dd.H + kPersistMaxGrid;
    P.attn = e->attn;
    P.err = &e->state->error;
    P.att_split = att_split;
    P.l2_bytes = l2_kb * 1024;
    // weight-tile loads mark their L2 lines evict-first (they are read once per step), so the K/V rows
    // and the barrier prefetches stay resident: 7B 2.844 -> 2.813 ms/token. "0" turns it off.
    const char *hint = getenv("VKLLM_B200_PERSIST_L2_HINT");
    P.l2_hint = hint ? (uint32_t)atoi(hint) : 1u;

    // Weight tiles of 16 rows x 256 columns; every K must be a multiple of 16 (MMA k-step).
    if (dd.D % 16 != 0 || HD % 16 != 0 || dd.F % 16 != 0)
        return;
    auto tile_geom = [](uint32_t units, uint32_t nm, uint32_t K) {
        TileGeom g;
        g.units = units;
        g.nm = nm;
        g.K = K;
        g.Ks = (K + kSegHalves - 1) / kSegHalves;
        g.last = K - kSegHalves * (g.Ks - 1);
        return g;
    };
    P.tg[PK_QKV] = tile_geom(3 * HD / 2, 2, dd.D);
    P.tg[PK_WO] = tile_geom(dd.D, 1, HD);
    P.tg[PK_UPGATE] = tile_geom(dd.F, 2, dd.D);
    P.tg[PK_DOWN] = tile_geom(dd.D, 1, dd.F);
    P.tg[PK_LOGITS] = tile_geom(dd.V, 1, dd.D);
    const uint32_t grid = (uint32_t)ctx->device->sm_count;
    if (grid > kPersistMaxGrid)
        return;
    // Row partition: CTA b owns units [tab[b], tab[b + 1]) of each phase, equal shares to start with
    // (balance_persistent may move units between CTAs later, up to unit_cap per CTA).
    e->htab.assign((size_t)PK_COUNT * (grid + 1), 0);
    for (int k = 0; k < PK_COUNT; ++k)
    {
        const uint32_t units = P.tg[k].units, base = units / grid, rem = units % grid;
        for (uint32_t b = 0; b <= grid; ++b)
            e->htab[(size_t)k * (grid + 1) + b] = b * base + (b < rem ? b : rem);
        e->unit_cap[k] = (units + grid - 1) / grid + (units / grid) / 4 + 1; // +25 %
    }
    uint32_t maxk = dd.D > HD ? dd.D : HD;
    if (dd.F > maxk)
        maxk = dd.F;
    size_t part_floats = 0;
    for (int k = 0; k < PK_COUNT; ++k)
    {
        const TileGeom &g = P.tg[k];
        const uint32_t rows = e->unit_cap[k] * g.nm;
        const size_t need = (size_t)(rows + kTileRows - 1) / kTileRows * kTileRows * g.Ks;
        part_floats = need > part_floats ? need : part_floats;
    }
    P.spw = spw < 1 ? 1 : (spw > kStreamMaxSpw ? kStreamMaxSpw : spw);
    P.spw_shift = 0; // a power of two (rounded down), so the kernel finds stages with masks and shifts
    while ((2u << P.spw_shift) <= P.spw)
        ++P.spw_shift;
    P.spw = 1u << P.spw_shift;
    P.xs_bytes = (maxk * 2 + 127) / 128 * 128;
    P.part_bytes = (uint32_t)((part_floats * 4 + 127) / 128 * 128);
    // Attention scratch (aliases xs + part): q, the split's scores, and per key-group partial
    // outputs [groups][hd]; at least 8 key groups, up to one per lpk threads of a full CTA. The
    // argmax combine needs 2 x 32 x 32 words of it.
    const uint32_t hd_al = (dd.hd + 31) & ~31u, chunk = (dd.ctx + att_split - 1) / att_split,
                   chunk_al = (chunk + 31) & ~31u;
    uint32_t lpk = 1;
    while (lpk < dd.hd / 8)
        lpk <<= 1;
    const uint32_t groups_full = 1024 / lpk;
    {
        const uint32_t min_floats = hd_al + chunk_al + 8 * dd.hd, argmax_floats = 2048;
        const uint32_t need = 4 * (min_floats > argmax_floats ? min_floats : argmax_floats);
        if (need > P.xs_bytes + P.part_bytes)
            P.part_bytes = (need - P.xs_bytes + 127) / 128 * 128;
        const uint32_t avail = (P.xs_bytes + P.part_bytes) / 4 - hd_al - chunk_al;
        P.att_groups = avail / dd.hd < groups_full ? avail / dd.hd : groups_full;
    }
    if (dd.hd % 8 != 0 || dd.hd > 256)
        return;
    // dynamic shared memory may use the opt-in limit minus the kernel's static shared memory (the
    // largest over the instantiations: tensor parallelism is configured after this setup)
    cudaFuncAttributes fa{};
    for (int v = 0; v < 8; ++v)
    {
        cudaFuncAttributes fv{};
        if (cudaFuncGetAttributes(&fv, persist_kernel(v & 1, v & 2, v & 4)) != cudaSuccess)
        {
            (void)cudaGetLastError();
            return;
        }
        fa.sharedSizeBytes = fv.sharedSizeBytes > fa.sharedSizeBytes ? fv.sharedSizeBytes : fa.sharedSizeBytes;
    }
    const size_t optin = ctx->device->smem_optin > fa.sharedSizeBytes ? ctx->device->smem_optin - fa.sharedSizeBytes : 0;
    const size_t fixed = kStreamBarBytes + P.xs_bytes + P.part_bytes;
    uint32_t warps = optin > fixed ? (uint32_t)((optin - fixed) / ((size_t)P.spw * kTileBytes)) : 0;
    if (warps > (uint32_t)kPersistMaxWarps)
        warps = kPersistMaxWarps;
    if (warps < 8 || P.att_groups < warps) // attention sums one partial row per warp in the scratch
        return;
    P.warps = warps;
    e->pp_smem = fixed + (size_t)warps * P.spw * kTileBytes;
    const char *trace = getenv("VKLLM_B200_TRACE");
    if (trace && atoi(trace) != 0)
    {
        P.trace_cap = 1u << 16;
        if (cudaMalloc(&P.trace, sizeof(uint64_t) * P.trace_cap) != cudaSuccess)
        {
            (void)cudaGetLastError();
            P.trace = nullptr;
            P.trace_cap = 0;
        }
        if (cudaMalloc(&P.trace_last, sizeof(uint64_t) * P.trace_cap) != cudaSuccess)
        {
            (void)cudaGetLastError();
            P.trace_last = nullptr;
        }
        if (grid <= kCtaTraceMaxCtas &&
            cudaMalloc(&P.trace_cta, sizeof(uint64_t) * kCtaTraceBarriers * grid) != cudaSuccess)
        {
            (void)cudaGetLastError();
            P.trace_cta = nullptr;
        }
        const size_t wbytes = sizeof(unsigned long long) * (kStreamMaxWarps * PK_COUNT * 4 + kAttTraceSlots);
        if (cudaMalloc(&P.wtrace, wbytes) != cudaSuccess || cudaMemset(P.wtrace, 0, wbytes) != cudaSuccess)
        {
            (void)cudaGetLastError();
            P.wtrace = nullptr;
        }
    }
    int blocks = 1;
    for (int v = 0; v < 8 && blocks >= 1; ++v)
    {
        int bv = 0;
        if (cudaFuncSetAttribute(persist_kernel(v & 1, v & 2, v & 4), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)e->pp_smem) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bv, persist_kernel(v & 1, v & 2, v & 4), 32 * warps,
                                                          e->pp_smem) != cudaSuccess)
            bv = 0;
        blocks = bv < blocks ? bv : blocks;
    }
    if (blocks < 1)
    {
        (void)cudaGetLastError();
        return;
    }
    // Decode copy of the weights in the tile layout (one bulk copy per tile).
    const uint32_t L = (uint32_t)e->layers.size();
    const size_t per_layer = (size_t)3 * HD * dd.D + (size_t)dd.D * HD + (size_t)2 * dd.F * dd.D + (size_t)dd.D * dd.F;
    const size_t halves = per_layer * L + (size_t)dd.V * dd.D;
    if (cudaMalloc(&e->tiled, halves * sizeof(__half)) != cudaSuccess ||
        cudaMalloc(&e->d_tiled_ptrs, sizeof(__half *) * 4 * L) != cudaSuccess)
    {
        (void)cudaGetLastError();
        log_info("no room for the decode copy of the weights (%zu MB); decode runs on the CUDA-graph path",
                 halves * 2 >> 20);
        if (e->tiled)
            cudaFree(e->tiled);
        e->tiled = nullptr;
        return;
    }
    cudaStream_t st = ctx->runtime->stream;
    if (cudaMalloc(&e->utab, sizeof(uint32_t) * (e->htab.size() + 2 * kFineMaxSegs)) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return;
    }
    P.utab = e->utab;
    P.dn_seg = e->utab + e->htab.size();
    // Fine-grained Wo and down phases (VKLLM_B200_PERSIST_FINE=1; off by default: at 7B they measured
    // 3.01 against 2.87 ms per token for the grid barriers with a full staging of the input). The
    // phases' segments must fit the per-CTA state table.
    const char *fine = getenv("VKLLM_B200_PERSIST_FINE");
    P.fine = fine && atoi(fine) != 0 && P.tg[PK_DOWN].Ks <= kFineMaxSegs && P.tg[PK_WO].Ks <= kFineMaxSegs ? 1u : 0u;
    std::vector<const __half *> ptrs;
    if (relayout_weights(e, st, &ptrs) != cudaSuccess ||
        cudaMemcpyAsync(e->d_tiled_ptrs, ptrs.data(), sizeof(__half *) * 4 * L, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return;
    }
    P.tiled = (const __half *const *)e->d_tiled_ptrs;
    if (cudaMalloc(&e->rope_den, sizeof(float) * 128) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return;
    }
    k_rope_den<<<1, 128, 0, st>>>(e->rope_den, dd.hd / 2, dd.hd, dd.rope_base);
    P.rope_den = e->rope_den;
    if (cudaMalloc(&e->d_layers, sizeof(LayerW) * e->layers.size()) != cudaSuccess)
    {
        (void)cudaGetLastError();
        return;
    }
    cudaMemcpy(e->d_layers, e->layers.data(), sizeof(LayerW) * e->layers.size(), cudaMemcpyHostToDevice);
    P.layers = e->d_layers;
    e->persistent = true;
}

// Enqueues n decode steps as cooperative persistent launches (at most 64 steps per launch).
vkllm_err_t run_persistent(Engine *e, uint32_t n, cudaStream_t s)
{
    e->launches = 0;
    while (n > 0)
    {
        const uint32_t k = n > 64 ? 64 : n;
        // barrier arrivals and per-head attention counters (they only grow during a launch)
        VKB_CUDA(cudaMemsetAsync(e->bar, 0, 4 * (1 + 3 * (size_t)e->dd.H + kPersistMaxGrid), s));
        PersistParams P = e->pp;
        P.n_steps = k;
        if (e->tp)
        {
            // every rank runs the same launches, so the per-site exchange counts stay in step
            for (int i = 0; i < 3; ++i)
                P.tp_base[i] = e->tp->base[i];
            e->tp->base[0] += k * P.L;
            e->tp->base[1] += k * P.L;
            e->tp->base[2] += k;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)e->ctx->device->sm_count); // one co-resident CTA per SM
        cfg.blockDim = dim3(32 * P.warps);
        cfg.dynamicSmemBytes = e->pp_smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        VKB_CUDA(cudaLaunchKernelEx(&cfg, persist_kernel(P.tp_size > 1, P.fine != 0, P.wtrace != nullptr), P));
        e->launches += 1;
        n -= k;
    }
    return VKLLM_ERR_OK;
}

// Splits `units` over CTAs in proportion to `w` (largest remainders), each CTA in [1, cap].
std::vector<uint32_t> apportion(uint32_t units, const std::vector<double> &w, uint32_t cap)
{
    const size_t n = w.size();
    std::vector<uint32_t> c(n, 1);
    if (units < n)
        return c; // more CTAs than units: the caller keeps its split (sum check)
    std::vector<double> want(n);
    double tw = 0.0;
    for (double x : w)
        tw += x;
    for (size_t i = 0; i < n; ++i)
        want[i] = (double)units * w[i] / tw;
    uint32_t left = units - (uint32_t)n;
    // hand out units one at a time to the CTA furthest below its share (n and units are small)
    while (left > 0)
    {
        size_t best = n;
        double gap = -1e30;
        for (size_t i = 0; i < n; ++i)
            if (c[i] < cap && want[i] - c[i] > gap)
            {
                gap = want[i] - c[i];
                best = i;
            }
        if (best == n)
            break;
        ++c[best];
        --left;
    }
    return c;
}

// Per-SM speed differs systematically (the same SMs finish their share of a phase several us late in
// every step), so the persistent kernel's row partition is calibrated once per engine: `rounds`
// one-step launches at the last cache position (whose KV row any real decode rewrites before it is
// read), each CTA's time per phase taken from its grid-barrier arrival times, and each phase's units
// re-split in proportion to the measured rate units / time (damped). Any partition gives the same
// results: a row's reduction does not depend on the CTA that computes it. The step state is restored.
void balance_persistent(Engine *e, uint32_t rounds)
{
    const DecodeDims &dd = e->dd;
    const uint32_t grid = (uint32_t)e->ctx->device->sm_count, L = (uint32_t)e->layers.size();
    const uint32_t nb = 5 * L + 1; // grid barriers of one step
    if (!e->persistent || e->tp || rounds == 0 || nb >= kCtaTraceBarriers || dd.ctx < 2)
        return;
    cudaStream_t st = e->ctx->runtime->stream;
    const bool own_trace = e->pp.trace_cta == nullptr;
    if (own_trace && cudaMalloc(&e->pp.trace_cta, sizeof(uint64_t) * kCtaTraceBarriers * grid) != cudaSuccess)
    {
        (void)cudaGetLastError();
        e->pp.trace_cta = nullptr;
        return;
    }
    StepState saved{};
    std::vector<uint64_t> a((size_t)nb * grid);
    bool ok = cudaStreamSynchronize(st) == cudaSuccess &&
              cudaMemcpy(&saved, e->state, sizeof(saved), cudaMemcpyDeviceToHost) == cudaSuccess;
    // the K and V rows at the last position of every layer and head are kept aside and put back
    const size_t row = (size_t)dd.hd * sizeof(__half), pitch = (size_t)dd.ctx * row;
    __half *kept = nullptr;
    ok = ok && cudaMalloc(&kept, row * dd.H * 2 * L) == cudaSuccess;
    auto keep_rows = [&](bool save) {
        bool good = true;
        for (uint32_t l = 0; l < L && good; ++l)
            for (int kv = 0; kv < 2 && good; ++kv)
            {
                char *cache = (char *)(kv ? e->layers[l].vcache : e->layers[l].kcache) + (size_t)(dd.ctx - 1) * row;
                char *side = (char *)kept + (size_t)(2 * l + kv) * dd.H * row;
                good = save ? cudaMemcpy2DAsync(side, row, cache, pitch, row, dd.H, cudaMemcpyDeviceToDevice, st) ==
                                  cudaSuccess
                            : cudaMemcpy2DAsync(cache, pitch, side, row, row, dd.H, cudaMemcpyDeviceToDevice, st) ==
                                  cudaSuccess;
            }
        return good;
    };
    const bool kept_ok = ok && keep_rows(true);
    ok = kept_ok;
    for (uint32_t it = 0; ok && it < rounds; ++it)
    {
        k_set_state<<<1, 1, 0, st>>>(e->state, nullptr, 1, dd.ctx - 1);
        StepState after{};
        ok = run_persistent(e, 1, st) == VKLLM_ERR_OK && cudaStreamSynchronize(st) == cudaSuccess &&
             cudaMemcpy(&after, e->state, sizeof(after), cudaMemcpyDeviceToHost) == cudaSuccess &&
             after.error == 0 &&
             cudaMemcpy(a.data(), e->pp.trace_cta, sizeof(uint64_t) * a.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
        if (!ok)
            break;
        auto rel = [&](uint32_t b) { // release of barrier b ~ its last arrival
            uint64_t m = 0;
            for (uint32_t c = 0; c < grid; ++c)
                m = a[(size_t)b * grid + c] > m ? a[(size_t)b * grid + c] : m;
            return m;
        };
        for (int k = 0; k < PK_COUNT; ++k)
        {
            // the barrier that ends phase k of layer l; QKV of layer 0 has no barrier before it
            std::vector<double> t(grid, 0.0);
            uint32_t n = 0;
            for (uint32_t l = 0; l < (k == PK_LOGITS ? 1u : L); ++l)
            {
                const uint32_t b = k == PK_LOGITS ? 5 * L : 5 * l + (k == PK_QKV ? 0 : k + 1);
                if (b == 0)
                    continue;
                const uint64_t r0 = rel(b - 1);
                for (uint32_t c = 0; c < grid; ++c)
                {
                    const uint64_t x = a[(size_t)b * grid + c];
                    t[c] += x > r0 ? (double)(x - r0) : 0.0;
                }
                ++n;
            }
            if (n == 0)
                continue;
            uint32_t *tab = e->htab.data() + (size_t)k * (grid + 1);
            std::vector<double> w(grid);
            bool sane = true;
            for (uint32_t c = 0; c < grid; ++c)
            {
                const double cnt = (double)(tab[c + 1] - tab[c]);
                sane = sane && t[c] > 0.0;
                w[c] = sane ? cnt / t[c] : 0.0;
            }
            if (!sane)
                continue;
            {
                double lo = t[0], hi = t[0], mean = 0.0;
                for (uint32_t c = 0; c < grid; ++c)
                {
                    lo = t[c] < lo ? t[c] : lo;
                    hi = t[c] > hi ? t[c] : hi;
                    mean += t[c] / grid;
                }
                log_info("persistent decode balance round %u, phase %d: per-CTA time %.2f us mean, %.2f us spread",
                         it, k, mean / n / 1e3, (hi - lo) / n / 1e3);
            }
            // damped: halfway from the current split to the rate-proportional one
            double tw = 0.0;
            for (double x : w)
                tw += x;
            const uint32_t units = tab[grid];
            for (uint32_t c = 0; c < grid; ++c)
                w[c] = 0.5 * (double)(tab[c + 1] - tab[c]) + 0.5 * (double)units * w[c] / tw;
            const std::vector<uint32_t> cnt = apportion(units, w, e->unit_cap[k]);
            uint32_t sum = 0;
            for (uint32_t c = 0; c < grid; ++c)
                sum += cnt[c];
            if (sum != units)
                continue;
            for (uint32_t c = 0; c < grid; ++c)
                tab[c + 1] = tab[c] + cnt[c];
        }
        ok = relayout_weights(e, st, nullptr) == cudaSuccess && cudaStreamSynchronize(st) == cudaSuccess;
    }
    if (!ok)
    {
        (void)cudaGetLastError();
        log_info("persistent decode: row balancing skipped, equal shares kept");
        for (int k = 0; k < PK_COUNT; ++k)
        {
            const uint32_t units = e->pp.tg[k].units, base = units / grid, rem = units % grid;
            for (uint32_t b = 0; b <= grid; ++b)
                e->htab[(size_t)k * (grid + 1) + b] = b * base + (b < rem ? b : rem);
        }
        if (relayout_weights(e, st, nullptr) != cudaSuccess)
            (void)cudaGetLastError();
    }
    saved.error = 0;
    if (kept_ok && !keep_rows(false))
        (void)cudaGetLastError();
    cudaMemcpyAsync(e->state, &saved, sizeof(saved), cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    if (kept)
        cudaFree(kept);
    if (own_trace)
    {
        cudaFree(e->pp.trace_cta);
        e->pp.trace_cta = nullptr;
    }
}

vkllm_err_t engine_create(vkllm_context *ctx, vkllm_models_llama2 *model, Engine **out)
{
    _CHECK_ARGS(model->weights.blocks && model->weights.kvcache && model->weights.tok_embed_weights &&
                model->weights.output_weight && model->weights.output_norm_weight);
    Engine *e = new Engine();
    e->ctx = ctx;
    DecodeDims &dd = e->dd;
    const uint32_t tp = model->b200.tp_size > 1 ? model->b200.tp_size : 1;
    dd.D = model->meta.embedding_length;
    dd.H = model->meta.head_count / tp;            // heads of this shard
    dd.V = model->weights.output_weight->shapes[2]; // vocabulary rows of this shard
    dd.ctx = model->meta.context_length;
    dd.eps = model->meta.layer_norm_rms_epsilon;
    dd.rope_base = model->meta.rope_freq_base;
    block_weights *b0 = model->weights.blocks->data[0];
    uint32_t HD = b0->WQ->shapes[2];
    dd.hd = HD / dd.H;
    dd.F = b0->WU->shapes[2];
    dd.scale = 1.0f / sqrtf((float)dd.hd);
    int sms = ctx->device->sm_count;
    uint32_t ns = (uint32_t)((2 * sms + dd.H - 1) / dd.H);
    dd.nsplit = ns < 1 ? 1 : (ns > 32 ? 32 : ns);
    e->unk = model->meta.padding_token_id;
    // Shape requirements of the fused kernels (anything else runs node by node).
    bool ok = dd.D % 8 == 0 && dd.F % 8 == 0 && HD % 8 == 0 && dd.hd % 4 == 0 && dd.hd <= 256 && dd.D % 2 == 0 &&
              HD * tp == dd.D && model->weights.tok_embed_weights->shapes[3] == dd.D &&
              model->weights.tok_embed_weights->dtype == vkllm_dtype_float16 &&
              model->weights.output_weight->shapes[2] == dd.V && model->weights.output_weight->shapes[3] == dd.D &&
              model->weights.output_weight->dtype == vkllm_dtype_float16 &&
              model->weights.output_norm_weight->dtype == vkllm_dtype_float32 &&
              model->weights.tok_embed_weights->shapes[2] == dd.V * tp;
    vkllm_kvcache *kv = model->weights.kvcache;
    for (uint32_t l = 0; ok && l < model->meta.block_count; ++l)
    {
        block_weights *bw = model->weights.blocks->data[l];
        ok = bw && bw->WQ && bw->WK && bw->WV && bw->WO && bw->WU && bw->WG && bw->WD && bw->attn_norm_weight &&
             bw->ffn_norm_weight && bw->WQ->dtype == vkllm_dtype_float16 && bw->WK->dtype == vkllm_dtype_float16 &&
             bw->WV->dtype == vkllm_dtype_float16 && bw->WO->dtype == vkllm_dtype_float16 &&
             bw->WU->dtype == vkllm_dtype_float16 && bw->WG->dtype == vkllm_dtype_float16 &&
             bw->WD->dtype == vkllm_dtype_float16 && bw->attn_norm_weight->dtype == vkllm_dtype_float32 &&
             bw->ffn_norm_weight->dtype == vkllm_dtype_float32 && bw->WQ->shapes[2] == HD &&
             bw->WQ->shapes[3] == dd.D && bw->WK->shapes[2] == HD && bw->WV->shapes[2] == HD &&
             bw->WO->shapes[2] == dd.D && bw->WO->shapes[3] == HD && bw->WU->shapes[2] == dd.F &&
             bw->WG->shapes[2] == dd.F && bw->WD->shapes[2] == dd.D && bw->WD->shapes[3] == dd.F &&
             l < kv->kcaches->used_n && kv->kcaches->data[l]->shapes[3] == dd.hd &&
             kv->kcaches->data[l]->shapes[1] == dd.H && kv->kcaches->data[l]->shapes[2] == dd.ctx;
        if (!ok)
            break;
        LayerW lw;
        lw.wq = (const __half *)dev_ptr(ctx, bw->WQ);
        lw.wk = (const __half *)dev_ptr(ctx, bw->WK);
        lw.wv = (const __half *)dev_ptr(ctx, bw->WV);
        lw.wo = (const __half *)dev_ptr(ctx, bw->WO);
        lw.wu = (const __half *)dev_ptr(ctx, bw->WU);
        lw.wg = (const __half *)dev_ptr(ctx, bw->WG);
        lw.wd = (const __half *)dev_ptr(ctx, bw->WD);
        lw.attn_norm = (const float *)dev_ptr(ctx, bw->attn_norm_weight);
        lw.ffn_norm = (const float *)dev_ptr(ctx, bw->ffn_norm_weight);
        lw.kcache = (__half *)dev_ptr(ctx, kv->kcaches->data[l]);
        lw.vcache = (__half *)dev_ptr(ctx, kv->vcaches->data[l]);
        e->layers.push_back(lw);
    }
    if (!ok)
    {
        delete e;
        log_info("model shape not covered by the fused decode engine; graphs run node by node");
        return VKLLM_ERR_ARGS;
    }
    e->embed = (const __half *)dev_ptr(ctx, model->weights.tok_embed_weights);
    e->wout = (const __half *)dev_ptr(ctx, model->weights.output_weight);
    e->out_norm = (const float *)dev_ptr(ctx, model->weights.output_norm_weight);

    // Attention key splits of the persistent path: about one (head, split) item per SM.
    const uint32_t att_split = (uint32_t)sms / dd.H > 0 ? ((uint32_t)sms / dd.H > 32 ? 32 : (uint32_t)sms / dd.H) : 1;
    const uint32_t max_split = att_split > dd.nsplit ? att_split : dd.nsplit;
    // Workspace layout (256-byte aligned pieces).
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    size_t off_x = 0, off_q = off_x + al(dd.D * 2), off_attn = off_q + al(HD * 2), off_m = off_attn + al(HD * 2),
           off_logits = off_m + al((size_t)dd.F * 2), off_scores = off_logits + al((size_t)dd.V * 2),
           off_part = off_scores + al((size_t)dd.H * dd.ctx * 2), off_opart = off_part + al((size_t)dd.H * max_split * 8),
           off_cnt = off_opart + al((size_t)dd.H * max_split * dd.hd * 4), off_lcnt = off_cnt + al(dd.H * 4),
           off_ring = off_lcnt + al(4), off_state = off_ring + al((size_t)dd.ctx * 4),
           off_amv = off_state + al(sizeof(StepState)), off_ami = off_amv + al((size_t)sms * 32 * 4),
           off_bar = off_ami + al((size_t)sms * 32 * 4),
           off_tp = off_bar + al(4 * (1 + 3 * (size_t)dd.H + kPersistMaxGrid)), // + per-CTA and per-head flags
           total = off_tp + al((size_t)dd.D * 4) + al(64 * 4) + al(64 * 4 * (size_t)kTpMax);
    if (cudaMalloc(&e->ws, total) != cudaSuccess)
    {
        (void)cudaGetLastError();
        delete e;
        return VKLLM_ERR_ALLOC;
    }
    cudaMemsetAsync(e->ws, 0, total, ctx->runtime->stream);
    char *w = (char *)e->ws;
    e->x = (__half *)(w + off_x);
    e->q = (__half *)(w + off_q);
    e->attn = (__half *)(w + off_attn);
    e->m = (__half *)(w + off_m);
    e->logits = (__half *)(w + off_logits);
    e->scores = (__half *)(w + off_scores);
    e->part = (float2 *)(w + off_part);
    e->opart = (float *)(w + off_opart);
    e->counters = (uint32_t *)(w + off_cnt);
    e->logit_counter = (uint32_t *)(w + off_lcnt);
    e->ring = (uint32_t *)(w + off_ring);
    e->state = (StepState *)(w + off_state);
    e->am_val = (float *)(w + off_amv);
    e->am_idx = (uint32_t *)(w + off_ami);
    e->bar = (uint32_t *)(w + off_bar);
    e->tp_sum = (float *)(w + off_tp);
    e->tp_cls = (uint32_t *)(w + off_tp + al((size_t)dd.D * 4));
    e->tp_cls_all = (uint32_t *)(w + off_tp + al((size_t)dd.D * 4) + al(64 * 4));

    // Streaming GEMV geometry: one CTA per SM; chunks of at most ~8 KB, one stage per warp and as
    // many warps (<= 32) as ~220 KB of shared memory holds next to the fp32 input vector.
    // Tuning overrides: VKLLM_B200_STREAM_SMEM_KB (shared memory per CTA), VKLLM_B200_STREAM_CHUNK_KB
    // (target chunk), VKLLM_B200_STREAM_CTAS_PER_SM (grid = SMs x this).
    auto env_u32 = [](const char *n, uint32_t d) {
        const char *v = getenv(n);
        return v && atoi(v) > 0 ? (uint32_t)atoi(v) : d;
    };
    const uint32_t kTarget = env_u32("VKLLM_B200_STREAM_CHUNK_KB", 8) * 1024;
    const uint32_t kSmemCap = env_u32("VKLLM_B200_STREAM_SMEM_KB", 220) * 1024;
    const uint32_t kSpw = env_u32("VKLLM_B200_STREAM_SPW", 1);
    e->grid_stream = (unsigned)sms * env_u32("VKLLM_B200_STREAM_CTAS_PER_SM", 1);
    e->g_qkv = make_stream_geom(3 * HD / 2, 2, dd.D, dd.D, kTarget, stream_cap<QkvOp>(ctx, kSmemCap), kSpw);
    e->g_wo = make_stream_geom(dd.D, 1, HD, HD, kTarget, stream_cap<WoOp>(ctx, kSmemCap), kSpw);
    e->g_upgate = make_stream_geom(dd.F, 2, dd.D, dd.D, kTarget, stream_cap<UpGateOp>(ctx, kSmemCap), kSpw);
    e->g_down = make_stream_geom(dd.D, 1, dd.F, dd.F, kTarget, stream_cap<DownOp>(ctx, kSmemCap), kSpw);
    e->g_logits = make_stream_geom(dd.V, 1, dd.D, dd.D, kTarget, stream_cap<LogitsOp>(ctx, kSmemCap), kSpw);
    for (const StreamGeom *g : {&e->g_qkv, &e->g_wo, &e->g_upgate, &e->g_down, &e->g_logits})
    {
        if (g->warps < 4 || stream_smem_bytes(*g) > ctx->device->smem_optin)
        {
            log_info("model rows too long for the streaming GEMV's shared memory; graphs run node by node");
            cudaFree(e->ws);
            delete e;
            return VKLLM_ERR_ARGS;
        }
    }
    allow_smem<QkvOp>(e->g_qkv);
    allow_smem<WoOp>(e->g_wo);
    allow_smem<UpGateOp>(e->g_upgate);
    allow_smem<DownOp>(e->g_down);
    allow_smem<LogitsOp>(e->g_logits);
    e->grid_embed = (dd.D / 8 + 255) / 256;
    e->kernels_per_step = 2 + 6 * (uint32_t)e->layers.size();
    // Persistent kernel: VKLLM_B200_PERSIST_SPW overrides the weight-tile stages per warp,
    // VKLLM_B200_PERSIST_L2_KB the next-phase weights per CTA prefetched into L2 at each barrier
    // (80 KB measured best at 7B: 0 -> 2.891, 32 -> 2.846, 48 -> 2.814, 64 -> 2.803, 80 -> 2.787,
    // 96 -> 2.788, 128 -> 2.810 ms/token on one box; 64 / 80 / 96 -> 2.813 / 2.810 / 2.813 on another).
    const char *l2kb = getenv("VKLLM_B200_PERSIST_L2_KB"); // "0" turns it off
    setup_persistent(e, ctx, att_split, env_u32("VKLLM_B200_PERSIST_SPW", 1), l2kb ? (uint32_t)atoi(l2kb) : 80u);
    e->pp.tp_size = tp;
    e->pp.tp_rank = tp > 1 ? model->b200.tp_rank : 0;
    e->pp.v0 = e->pp.tp_rank * dd.V;
    e->pp.Vg = dd.V * tp;
    TpComm *tpc = (TpComm *)model->b200.tp_comm;
    const char *tp_x = getenv("VKLLM_B200_TP_EXCHANGE"); // "nccl": the NCCL exchange when both are connected
    if (tp > 1 && tpc && tpc->nccl && (!tpc->connected || (tp_x && strcmp(tp_x, "nccl") == 0)))
    {
        // NCCL exchange: the per-op kernels of the graph path on the shards, with an ncclAllReduce of
        // the Wo and down partial rows and an ncclAllGather of the argmax candidates, captured below.
        e->persistent = false;
        e->tp = tpc;
        e->tp_nccl = true;
        e->kernels_per_step += 2 * (uint32_t)e->layers.size() + 1; // residual adds and the argmax
    }
    else if (tp > 1)
    {
        // Tensor-parallel shards decode on the persistent kernel, whose Wo / down epilogues exchange
        // the partial sums over peer memory.
        TpComm *c = tpc;
        if (!e->persistent || !c || !c->connected || (uint32_t)sms > kTpCtas ||
            e->htab[PK_WO * ((size_t)sms + 1) + 1] > kTpRows || (dd.D + sms - 1) / sms > kTpRows)
        {
            log_error("tensor-parallel decode needs the persistent kernel and vkllm_b200_tp_connect, or "
                      "vkllm_b200_tp_nccl_connect, first");
            if (e->d_layers)
                cudaFree(e->d_layers);
            cudaFree(e->ws);
            delete e;
            return VKLLM_ERR_ARGS;
        }
        const TpLayout t = tp_layout(c->world, dd.D);
        for (uint32_t q = 0; q < c->world; ++q)
        {
            char *b = (char *)c->peer[q];
            e->pp.tp_x[q] = (uint64_t *)(b + t.x);
            e->pp.tp_flag[q] = (uint32_t *)(b + t.flag);
            e->pp.tp_amv[q] = (float *)(b + t.amv);
            e->pp.tp_ami[q] = (uint32_t *)(b + t.ami);
        }
        e->tp = c;
        *out = e;
        return VKLLM_ERR_OK; // no CUDA-graph path for shards
    }

    // Capture one decode step.
    cudaStream_t cs;
    if (cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking) != cudaSuccess)
    {
        cudaFree(e->ws);
        delete e;
        return VKLLM_ERR_VULKAN;
    }
    cudaStreamSynchronize(ctx->runtime->stream);
    (void)cudaGetLastError(); // errors of earlier calls were reported where they happened
    vkllm_err_t err = VKLLM_ERR_OK;
    if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        err = VKLLM_ERR_VULKAN;
    if (err == VKLLM_ERR_OK)
    {
        vkllm_err_t le = enqueue_step(e, cs);
        cudaError_t ce = cudaStreamEndCapture(cs, &e->graph);
        if (le != VKLLM_ERR_OK || ce != cudaSuccess)
            err = VKLLM_ERR_VULKAN;
    }
    if (err == VKLLM_ERR_OK && cudaGraphInstantiate(&e->exec, e->graph, 0) != cudaSuccess)
        err = VKLLM_ERR_VULKAN;
    cudaStreamDestroy(cs);
    if (err != VKLLM_ERR_OK)
    {
        log_error("capturing the decode step failed: %s", cudaGetErrorString(cudaGetLastError()));
        if (e->graph)
            cudaGraphDestroy(e->graph);
        cudaFree(e->ws);
        delete e;
        return err;
    }
    // VKLLM_B200_PERSIST_BALANCE: calibration rounds of the row partition (default 8; 0 keeps equal
    // shares). 7B, same box: 0 -> 2.791, 5 -> 2.760, 8 -> 2.755-2.757, 12 -> 2.751-2.756 ms/token.
    // (With the slower kernel of before, 0 -> 2.857, 3 -> 2.869, 6 -> 2.864: the CTAs that finished
    // a phase first kept HBM busy with the next phase's tiles; with fewer instructions per tile the
    // slowest CTA at each barrier is what the step waits for.)
    const char *bal = getenv("VKLLM_B200_PERSIST_BALANCE");
    balance_persistent(e, bal ? (uint32_t)atoi(bal) : 8u);
    *out = e;
    return VKLLM_ERR_OK;
}

vkllm_err_t get_engine(vkllm_context *ctx, vkllm_models_llama2 *model, Engine **out)
{
    if (!model->b200.engine)
    {
        Engine *e = nullptr;
        _CHECK(engine_create(ctx, model, &e));
        model->b200.engine = e;
    }
    Engine *e = (Engine *)model->b200.engine;
    if (e->ctx != ctx)
        return VKLLM_ERR_ARGS;
    *out = e;
    return VKLLM_ERR_OK;
}

} // namespace

void engine_destroy(vkllm_context *ctx, vkllm_models_llama2 *model)
{
    (void)ctx;
    Engine *e = (Engine *)model->b200.engine;
    if (!e)
        return;
    if (e->ctx && e->ctx->runtime)
        cudaStreamSynchronize(e->ctx->runtime->stream);
    if (e->pf_ws)
        cudaFree(e->pf_ws);
    if (e->exec)
        cudaGraphExecDestroy(e->exec);
    if (e->graph)
        cudaGraphDestroy(e->graph);
    cudaFree(e->ws);
    if (e->d_layers)
        cudaFree(e->d_layers);
    if (e->tiled)
        cudaFree(e->tiled);
    if (e->d_tiled_ptrs)
        cudaFree(e->d_tiled_ptrs);
    if (e->rope_den)
        cudaFree(e->rope_den);
    if (e->pp.trace)
        cudaFree(e->pp.trace);
    if (e->pp.wtrace)
        cudaFree(e->pp.wtrace);
    if (e->pp.trace_last)
        cudaFree(e->pp.trace_last);
    if (e->pp.trace_cta)
        cudaFree(e->pp.trace_cta);
    if (e->utab)
        cudaFree(e->utab);
    delete e;
    model->b200.engine = nullptr;
}

// ------------------------------------------------------------------------------------------------
// Fused prefill: the llama2 graph of S > 1 tokens (src/models/vkllm_models_llama2.c:488-602) as
// per-layer kernels: RMSNORM, the Q/K/V projections on the tensor-core GEMM, RoPE with the KV-cache
// rows (k_pf_rope_kv), attention in one kernel (k_pf_attention), Wo, the residual BIN, RMSNORM,
// up and gate (SiLU) GEMMs, their product, down and the residual; then RMSNORM, the logits of all S
// rows and their argmax. The node order and rounding points are the graph's; the argmax of every
// row goes to the graph's mapped output and the last row's logits to the engine's logits buffer.
// Returns VKLLM_ERR_ARGS when this path does not apply (the graph then runs node by node).
namespace
{

template <int HD, bool PAIR>
bool pf_attention_launch(const __half *rq, const LayerW &lw, const DecodeDims &dd, uint32_t S, uint32_t p0,
                         __half *out, cudaStream_t s)
{
    static bool attr_set[64] = {}; // per device: the attribute is a property of the current device's function
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return false;
    if (!attr_set[dev])
    {
        if (cudaFuncSetAttribute(k_pf_attention<HD, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PfSmem<HD>::kBytes) != cudaSuccess)
        {
            (void)cudaGetLastError();
            return false;
        }
        attr_set[dev] = true;
    }
    const uint32_t tiles = (S + kPfBQ - 1) / kPfBQ;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(PAIR ? 2 * tiles : tiles, dd.H);
    lc.blockDim = dim3(kPfThreads);
    lc.dynamicSmemBytes = PfSmem<HD>::kBytes;
    lc.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = PAIR ? 2 : 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = PAIR ? 1 : 0;
    if (cudaLaunchKernelEx(&lc, k_pf_attention<HD, PAIR>, rq, (const __half *)lw.kcache, (const __half *)lw.vcache,
                           dd.ctx, S, p0, dd.H, dd.scale, out) != cudaSuccess)
    {
        log_error("prefill attention launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return false;
    }
    return true;
}

// VKLLM_B200_PF_ATT_PAIR=0: one CTA per (query tile, head) instead of a cluster of two that split the
// key blocks.
template <int HD>
bool pf_attention_hd(const __half *rq, const LayerW &lw, const DecodeDims &dd, uint32_t S, uint32_t p0, __half *out,
                     cudaStream_t s)
{
    const char *v = getenv("VKLLM_B200_PF_ATT_PAIR");
    const bool pair = !(v && atoi(v) == 0);
    return pair ? pf_attention_launch<HD, true>(rq, lw, dd, S, p0, out, s)
                : pf_attention_launch<HD, false>(rq, lw, dd, S, p0, out, s);
}

bool pf_attention(const __half *rq, const LayerW &lw, const DecodeDims &dd, uint32_t S, uint32_t p0, __half *out,
                  cudaStream_t s)
{
    switch (dd.hd)
    {
    case 32:
        return pf_attention_hd<32>(rq, lw, dd, S, p0, out, s);
    case 48:
        return pf_attention_hd<48>(rq, lw, dd, S, p0, out, s);
    case 64:
        return pf_attention_hd<64>(rq, lw, dd, S, p0, out, s);
    case 80:
        return pf_attention_hd<80>(rq, lw, dd, S, p0, out, s);
    case 96:
        return pf_attention_hd<96>(rq, lw, dd, S, p0, out, s);
    case 128:
        return pf_attention_hd<128>(rq, lw, dd, S, p0, out, s);
    default:
        return false;
    }
}

// C [M, N] = act(A [M, K] . B [N, K]^T), dense row-major, on the tensor-core GEMM. With B1 (and B2),
// B is the row concatenation [B; B1; B2] of matrices of N / groups rows each, read in place (one
// launch instead of one per matrix); act applies from column act_from on.
bool pf_gemm(const __half *A, const __half *B, __half *C, uint32_t M, uint32_t N, uint32_t K, int act, cudaStream_t s,
             const __half *B1 = nullptr, const __half *B2 = nullptr, uint32_t act_from = 0)
{
    const uint32_t groups = B2 ? 3 : (B1 ? 2 : 1);
    Desc4 da{{1, 1, M, K}, {0, 0, K, 1}}, db{{1, 1, N, K}, {0, 0, K, 1}}, dc{{1, 1, M, N}, {0, 0, N, 1}};
    GemmArgs g;
    if (!make_gemm_args(da, db, dc, true, A, B, C, 1.0f, act, &g))
        return false;
    if (groups > 1)
    {
        g.B1 = B1;
        g.B2 = B2;
        g.b_group_n = N / groups;
    }
    g.act_from = act_from;
    return gemm_tcgen05_launch(g, s);
}

bool prefill_applies(const Engine *e)
{
    const char *env = getenv("VKLLM_B200_PREFILL");
    if (env && atoi(env) == 0)
        return false;
    const DecodeDims &dd = e->dd;
    const bool hd_ok = dd.hd == 32 || dd.hd == 48 || dd.hd == 64 || dd.hd == 80 || dd.hd == 96 || dd.hd == 128;
    return hd_ok && !e->tp && dd.H * dd.hd == dd.D && dd.D % 8 == 0 && dd.F % 8 == 0 && dd.V % 8 == 0 &&
           dd.D / 8 <= 1024;
}

} // namespace

vkllm_err_t prefill_run(Engine *e, const uint32_t *tok, uint32_t S, uint32_t p0, uint32_t *out, cudaStream_t s)
{
    const DecodeDims &dd = e->dd;
    if (!prefill_applies(e) || (uint64_t)p0 + S > dd.ctx)
        return VKLLM_ERR_ARGS;
    const uint32_t D = dd.D, F = dd.F, V = dd.V, HD = dd.H * dd.hd;
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t sd = al((size_t)S * D * 2), shd = al((size_t)S * HD * 2), sf = al((size_t)S * F * 2),
                 sv = al((size_t)S * V * 2);
    const size_t need = 3 * sd + 5 * shd + 3 * sf + sv;
    if (need > e->pf_cap)
    {
        if (e->pf_ws)
        {
            VKB_CUDA(cudaStreamSynchronize(s));
            cudaFree(e->pf_ws);
            e->pf_ws = nullptr;
            e->pf_cap = 0;
        }
        VKB_CUDA(cudaMalloc(&e->pf_ws, need));
        e->pf_cap = need;
    }
    char *w = (char *)e->pf_ws;
    __half *x = (__half *)w, *n = (__half *)(w + sd), *y = (__half *)(w + 2 * sd);
    // q, k, v side by side ([S][3 HD]) when one grouped GEMM makes them, else three [S][HD] blocks
    __half *qkv = (__half *)(w + 3 * sd), *rq = (__half *)(w + 3 * sd + 3 * shd), *att = (__half *)(w + 3 * sd + 4 * shd);
    // up and gate side by side ([S][2F]) when grouped, else two [S][F] blocks; then m [S][F]
    __half *ug = (__half *)(w + 3 * sd + 5 * shd), *mm = (__half *)(w + 3 * sd + 5 * shd + 2 * sf);
    __half *lg = (__half *)(w + 3 * sd + 5 * shd + 3 * sf);
    // grouped GEMMs load B tiles that straddle two matrices in 32-row pieces
    const bool grouped = HD % 32 == 0 && F % 32 == 0;
    const uint32_t ldq = grouped ? 3 * HD : HD, ldu = grouped ? 2 * F : F;
    __half *q = qkv, *k = grouped ? qkv + HD : qkv + (uint64_t)S * HD, *v = grouped ? qkv + 2 * HD : qkv + 2ull * S * HD;
    __half *up = ug, *gt = grouped ? ug + F : ug + (uint64_t)S * F;
    k_pf_embed<<<S, 128, 0, s>>>(tok, e->embed, dd.V, D, e->unk, x);
    const uint64_t rope_threads = (uint64_t)S * HD / 8, gate_threads = (uint64_t)S * F / 8;
    // the residual adds and the RMSNORMs after them run as one pass per row (the next layer's attention
    // norm comes with the down projection's residual, the output norm with the last one's)
    if (!launch_rmsnorm_rows(x, e->layers[0].attn_norm, n, S, D, dd.eps, s))
        return VKLLM_ERR_ARGS;
    for (size_t li = 0; li < e->layers.size(); ++li)
    {
        const LayerW &lw = e->layers[li];
        bool ok = true;
        if (grouped)
            ok = ok && pf_gemm(n, lw.wq, qkv, S, 3 * HD, D, 0, s, lw.wk, lw.wv);
        else
            ok = ok && pf_gemm(n, lw.wq, q, S, HD, D, 0, s) && pf_gemm(n, lw.wk, k, S, HD, D, 0, s) &&
                 pf_gemm(n, lw.wv, v, S, HD, D, 0, s);
        if (!ok)
            return VKLLM_ERR_ARGS;
        k_pf_rope_kv<<<(unsigned)((rope_threads + 255) / 256), 256, 0, s>>>(q, k, v, ldq, S, dd.H, dd.hd, p0, dd.ctx,
                                                                            dd.rope_base, rq, lw.kcache, lw.vcache);
        ok = pf_attention(rq, lw, dd, S, p0, att, s) && pf_gemm(att, lw.wo, y, S, D, HD, 0, s) &&
             launch_residual_rmsnorm_rows(x, y, lw.ffn_norm, n, S, D, dd.eps, s);
        if (grouped) // [up | silu(gate)]: SiLU from column F on
            ok = ok && pf_gemm(n, lw.wu, ug, S, 2 * F, D, 1, s, lw.wg, nullptr, F);
        else
            ok = ok && pf_gemm(n, lw.wu, up, S, F, D, 0, s) && pf_gemm(n, lw.wg, gt, S, F, D, 1, s);
        if (!ok)
            return VKLLM_ERR_ARGS;
        k_pf_gate_mul<<<(unsigned)((gate_threads + 255) / 256), 256, 0, s>>>(up, gt, ldu, S, F, mm);
        const float *next_norm = li + 1 < e->layers.size() ? e->layers[li + 1].attn_norm : e->out_norm;
        ok = pf_gemm(mm, lw.wd, y, S, D, F, 0, s) && launch_residual_rmsnorm_rows(x, y, next_norm, n, S, D, dd.eps, s);
        if (!ok)
            return VKLLM_ERR_ARGS;
    }
    if (!pf_gemm(n, e->wout, lg, S, V, D, 0, s) ||
        !launch_argmax_rows(lg, S, V, out, s))
        return VKLLM_ERR_ARGS;
    VKB_CUDA(cudaMemcpyAsync(e->logits, lg + (uint64_t)(S - 1) * V, (size_t)V * 2, cudaMemcpyDeviceToDevice, s));
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

vkllm_err_t plan_run(vkllm_context *ctx, vkllm_graph *graph)
{
    Plan *p = (Plan *)graph->b200_plan;
    if (!p || p->seq_len == 0 || graph->output_node != p->output || graph->nodes->used_n != p->n_nodes)
        return VKLLM_ERR_ARGS;
    if (p->input_toks->dtype != vkllm_dtype_uint32 || !p->output->data.mapped)
        return VKLLM_ERR_ARGS;
    Engine *e = nullptr;
    if (get_engine(ctx, p->model, &e) != VKLLM_ERR_OK)
        return VKLLM_ERR_ARGS;
    if (p->seq_len > 1)
    {
        cudaStream_t s = (cudaStream_t)graph->commands->stream;
        const uint32_t *tok = (const uint32_t *)dev_ptr(ctx, p->input_toks);
        uint32_t *out = (uint32_t *)p->output->data.dev;
        if (!tok || !out)
            return VKLLM_ERR_ALLOC;
        vkllm_err_t err = prefill_run(e, tok, p->seq_len, p->offsets, out, s);
        if (err != VKLLM_ERR_OK)
            return err;
        _CHECK(vkllm_commands_submit(ctx, graph->commands));
        _CHECK(vkllm_commands_wait_exec(ctx, graph->commands));
        return VKLLM_ERR_OK;
    }
    if (p->offsets >= e->dd.ctx)
        return VKLLM_ERR_ARGS;
    cudaStream_t s = (cudaStream_t)graph->commands->stream;
    const uint32_t *tok = (const uint32_t *)dev_ptr(ctx, p->input_toks);
    uint32_t *out = (uint32_t *)p->output->data.dev;
    if (!tok || !out)
        return VKLLM_ERR_ALLOC;
    k_set_state<<<1, 1, 0, s>>>(e->state, tok, 0, p->offsets);
    if (e->persistent)
        _CHECK(run_persistent(e, 1, s));
    else
        VKB_CUDA(cudaGraphLaunch(e->exec, s));
    k_emit_token<<<1, 1, 0, s>>>(e->state, out);
    VKB_CUDA(cudaGetLastError());
    _CHECK(vkllm_commands_submit(ctx, graph->commands));
    _CHECK(vkllm_commands_wait_exec(ctx, graph->commands));
    return VKLLM_ERR_OK;
}

void graph_cache_detach(vkllm_context *ctx, Plan *plan);

void plan_free(vkllm_context *ctx, vkllm_graph *graph)
{
    graph_cache_detach(ctx, (Plan *)graph->b200_plan);
    free(graph->b200_plan);
    graph->b200_plan = nullptr;
}

// ------------------------------------------------------------------------------------------------
// Counter-based generator for random weights: element i of tensor t is the Irwin-Hall sum of 12
// 16-bit uniforms drawn from splitmix64(key + 3i + j), j = 0..2, centred and scaled to std_dev,
// rounded to fp16. Integer sums are exact and the single fp32 product rounds identically on host
// and device, so vkllm_b200_random_f16_host reproduces the device bits.
__host__ __device__ inline uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__host__ __device__ inline float random_value(uint64_t key, uint64_t i, float scale)
{
    int64_t s = 0;
    for (int j = 0; j < 3; ++j)
    {
        uint64_t h = splitmix64(key + 3 * i + (uint64_t)j);
        s += (int64_t)(h & 0xffff) + (int64_t)((h >> 16) & 0xffff) + (int64_t)((h >> 32) & 0xffff) +
             (int64_t)(h >> 48);
    }
    float t = (float)(int32_t)(s - 393210);
    return t * scale;
}

__global__ void k_fill_random_f16(__half *dst, uint64_t n, uint64_t key, float scale)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(random_value(key, i, scale));
}

// Shard [rows, cols] of a [*, full_cols] matrix at (row0, col0): element (i, c) is element
// (row0 + i) * full_cols + col0 + c of the full tensor, so shards hold exactly the full matrix's bits.
__global__ void k_fill_random_f16_2d(__half *dst, uint64_t rows, uint64_t cols, uint64_t full_cols, uint64_t row0,
                                     uint64_t col0, uint64_t key, float scale)
{
    const uint64_t n = rows * cols;
    for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n; t += (uint64_t)gridDim.x * blockDim.x)
    {
        const uint64_t i = t / cols, c = t % cols;
        dst[t] = __float2half_rn(random_value(key, (row0 + i) * full_cols + col0 + c, scale));
    }
}

__global__ void k_fill_const_f32(float *dst, uint64_t n, float v)
{
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

static uint64_t tensor_key(uint64_t seed, uint64_t tensor_id)
{
    return splitmix64(seed ^ splitmix64(tensor_id + 0x5851F42D4C957F2Dull));
}

vkllm_err_t fill_random_f16(vkllm_context *ctx, void *dst, uint64_t n, uint64_t seed, uint64_t tensor_id, float std_dev)
{
    float scale = std_dev * (1.0f / 65536.0f);
    k_fill_random_f16<<<ctx->device->sm_count * 8, 256, 0, ctx->runtime->stream>>>((__half *)dst, n,
                                                                                     tensor_key(seed, tensor_id), scale);
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

vkllm_err_t fill_random_f16_shard(vkllm_context *ctx, void *dst, uint64_t rows, uint64_t cols, uint64_t full_cols,
                                  uint64_t row0, uint64_t col0, uint64_t seed, uint64_t tensor_id, float std_dev)
{
    float scale = std_dev * (1.0f / 65536.0f);
    k_fill_random_f16_2d<<<ctx->device->sm_count * 8, 256, 0, ctx->runtime->stream>>>(
        (__half *)dst, rows, cols, full_cols, row0, col0, tensor_key(seed, tensor_id), scale);
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

vkllm_err_t fill_const_f32(vkllm_context *ctx, void *dst, uint64_t n, float v)
{
    k_fill_const_f32<<<(unsigned)((n + 255) / 256 > 1024 ? 1024 : (n + 255) / 256), 256, 0, ctx->runtime->stream>>>(
        (float *)dst, n, v);
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

static uint16_t f32_to_f16_rne(float f)
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

} // namespace vkb

using namespace vkb;

extern "C" void vkllm_b200_random_f16_host_shard(uint64_t seed, uint64_t tensor_id, float std_dev, uint64_t full_cols,
                                                 uint32_t row0, uint32_t rows, uint32_t col0, uint32_t cols,
                                                 uint16_t *out)
{
    const float scale = std_dev * (1.0f / 65536.0f);
    const uint64_t key = tensor_key(seed, tensor_id);
    for (uint64_t i = 0; i < rows; ++i)
        for (uint64_t c = 0; c < cols; ++c)
            out[i * cols + c] = f32_to_f16_rne(random_value(key, (row0 + i) * full_cols + col0 + c, scale));
}

extern "C" void vkllm_b200_random_f16_host(uint64_t seed, uint64_t tensor_id, float std_dev, uint64_t first,
                                           uint64_t n, uint16_t *out)
{
    uint64_t key = tensor_key(seed, tensor_id);
    float scale = std_dev * (1.0f / 65536.0f);
    for (uint64_t i = 0; i < n; ++i)
        out[i] = f32_to_f16_rne(random_value(key, first + i, scale));
}

extern "C" vkllm_err_t vkllm_b200_engine_prepare(struct vkllm_context *context, struct vkllm_models_llama2 *model)
{
    _CHECK_ARGS(context && model);
    Engine *e;
    return get_engine(context, model, &e);
}

extern "C" vkllm_err_t vkllm_b200_engine_set_state(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                   uint32_t token, uint32_t pos)
{
    _CHECK_ARGS(context && model);
    Engine *e;
    _CHECK(get_engine(context, model, &e));
    _CHECK_ARGS(pos < e->dd.ctx);
    k_set_state<<<1, 1, 0, context->runtime->stream>>>(e->state, nullptr, token, pos);
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_engine_decode_steps(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                      uint32_t n)
{
    _CHECK_ARGS(context && model);
    Engine *e;
    _CHECK(get_engine(context, model, &e));
    if (e->persistent)
        return run_persistent(e, n, context->runtime->stream);
    for (uint32_t i = 0; i < n; ++i)
        VKB_CUDA(cudaGraphLaunch(e->exec, context->runtime->stream));
    e->launches = n * e->kernels_per_step;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_engine_read_tokens(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                     uint32_t *out, uint32_t n)
{
    _CHECK_ARGS(context && model && out);
    Engine *e;
    _CHECK(get_engine(context, model, &e));
    _CHECK_ARGS(n <= e->dd.ctx);
    VKB_CUDA(cudaStreamSynchronize(context->runtime->stream));
    StepState st;
    VKB_CUDA(cudaMemcpy(&st, e->state, sizeof(st), cudaMemcpyDeviceToHost));
    if (st.error)
    {
        log_error("decode step failed on the device (error word 0x%x: 0x1 position past the KV cache, "
                  "0x100 copy wait timed out, 0x200 grid barrier timed out)", st.error);
        return (st.error & ~1u) ? VKLLM_ERR_VULKAN : VKLLM_ERR_ARGS;
    }
    VKB_CUDA(cudaMemcpy(out, e->ring, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_engine_read_logits(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                     uint16_t *out, uint32_t n)
{
    _CHECK_ARGS(context && model && out);
    Engine *e;
    _CHECK(get_engine(context, model, &e));
    _CHECK_ARGS(n <= e->dd.V);
    VKB_CUDA(cudaStreamSynchronize(context->runtime->stream));
    VKB_CUDA(cudaMemcpy(out, e->logits, (size_t)n * 2, cudaMemcpyDeviceToHost));
    return VKLLM_ERR_OK;
}

extern "C" uint32_t vkllm_b200_engine_kernels_per_step(struct vkllm_context *context, struct vkllm_models_llama2 *model)
{
    if (!context || !model || !model->b200.engine)
        return 0;
    Engine *e = (Engine *)model->b200.engine;
    return e->persistent ? 1u : e->kernels_per_step;
}

// Times `iters` back-to-back launches of one decode kernel (layers cycled so each launch streams
// its own weights from HBM, as inside a step) with CUDA events on the context stream. Reports the
// mean duration per launch and the algorithmic bytes one launch must move.
extern "C" vkllm_err_t vkllm_b200_engine_bench_kernel(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                      const char *kernel, uint32_t iters, float *us_per_launch,
                                                      uint64_t *bytes_per_launch)
{
    _CHECK_ARGS(context && model && kernel && iters > 0 && us_per_launch && bytes_per_launch);
    Engine *e;
    _CHECK(get_engine(context, model, &e));
    const DecodeDims &dd = e->dd;
    const uint64_t HD = (uint64_t)dd.H * dd.hd;
    cudaStream_t s = context->runtime->stream;
    int which = -1;
    const char *names[] = {"qkv", "wo", "upgate", "down", "logits"};
    for (int i = 0; i < 5; ++i)
        if (strcmp(kernel, names[i]) == 0)
            which = i;
    _CHECK_ARGS(which >= 0);
    uint64_t bytes = 0;
    switch (which)
    {
    case 0:
        bytes = 3 * HD * dd.D * 2 + dd.D * 2 + dd.D * 4 + 2 * HD * 2 + HD * 2;
        break;
    case 1:
        bytes = (uint64_t)dd.D * HD * 2 + HD * 2 + 2ull * dd.D * 2;
        break;
    case 2:
        bytes = 2ull * dd.F * dd.D * 2 + dd.D * 2 + dd.D * 4 + (uint64_t)dd.F * 2;
        break;
    case 3:
        bytes = (uint64_t)dd.D * dd.F * 2 + (uint64_t)dd.F * 2 + 2ull * dd.D * 2;
        break;
    case 4:
        bytes = (uint64_t)dd.V * dd.D * 2 + dd.D * 2 + dd.D * 4 + (uint64_t)dd.V * 2;
        break;
    }
    k_set_state<<<1, 1, 0, s>>>(e->state, nullptr, 0, 0);
    cudaEvent_t a, b;
    VKB_CUDA(cudaEventCreate(&a));
    VKB_CUDA(cudaEventCreate(&b));
    auto launch = [&](uint32_t i) {
        const LayerW &lw = e->layers[i % e->layers.size()];
        switch (which)
        {
        case 0:
            launch_stream(e, op_qkv(e, lw), e->g_qkv, s);
            break;
        case 1:
            launch_stream(e, op_wo(e, lw), e->g_wo, s);
            break;
        case 2:
            launch_stream(e, op_upgate(e, lw), e->g_upgate, s);
            break;
        case 3:
            launch_stream(e, op_down(e, lw), e->g_down, s);
            break;
        case 4:
            launch_stream(e, op_logits(e), e->g_logits, s);
            break;
        }
    };
    for (uint32_t i = 0; i < 3; ++i)
        launch(i);
    VKB_CUDA(cudaEventRecord(a, s));
    for (uint32_t i = 0; i < iters; ++i)
        launch(i);
    VKB_CUDA(cudaEventRecord(b, s));
    VKB_CUDA(cudaEventSynchronize(b));
    float ms = 0.f;
    VKB_CUDA(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    VKB_CUDA(cudaGetLastError());
    *us_per_launch = ms * 1000.0f / (float)iters;
    *bytes_per_launch = bytes;
    return VKLLM_ERR_OK;
}

// ------------------------------------------------------------------------------------------------
// Allocation-free decode attention.
//
// Some callers cannot allocate device memory at the point where they run attention: code that runs
// while a CUDA stream is being captured into a graph (cudaMalloc is not allowed there), code inside
// a memory-pool-managed or pre-budgeted runtime that forbids allocations after start-up, and
// real-time paths that must not block on the driver's allocator. For them this entry point runs the
// same split-key decode attention kernels as the fused engine (k_dec_attn_scores + k_dec_attn_pv),
// with all their scratch memory (fp16 scores, per-split softmax statistics, per-split partial
// outputs, completion counters, the step word) in one file-scope device array instead of a
// workspace. The array is reserved when the library is loaded onto a device and stays there until
// the process exits.
namespace vkb
{
namespace
{

// Limits of the static scratch (about 1.1 MiB in total).
constexpr uint32_t kNoAllocMaxHeads = 64;
constexpr uint32_t kNoAllocMaxScoreRows = 262144; // heads * cache_rows
constexpr uint32_t kNoAllocMaxHeadDim = 256;
constexpr uint32_t kNoAllocSplits = 8;
constexpr size_t kNoAllocScoresBytes = (size_t)kNoAllocMaxScoreRows * 2;
constexpr size_t kNoAllocPartBytes = (size_t)kNoAllocMaxHeads * kNoAllocSplits * sizeof(float2);
constexpr size_t kNoAllocOpartBytes = (size_t)kNoAllocMaxHeads * kNoAllocSplits * kNoAllocMaxHeadDim * 4;
constexpr size_t kNoAllocCountersBytes = (size_t)kNoAllocMaxHeads * 4;
constexpr size_t kNoAllocOffPart = kNoAllocScoresBytes;
constexpr size_t kNoAllocOffOpart = kNoAllocOffPart + kNoAllocPartBytes;
constexpr size_t kNoAllocOffCounters = kNoAllocOffOpart + kNoAllocOpartBytes;
constexpr size_t kNoAllocOffState = kNoAllocOffCounters + kNoAllocCountersBytes;
constexpr size_t kNoAllocBytes = kNoAllocOffState + 256;

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_addr[64] = {};

// Device address of the scratch array on the current device, looked up once per device (the
// host-side symbol is only a stand-in and must never be handed to a kernel).
vkllm_err_t noalloc_scratch(void **out)
{
    int dev = 0;
    VKB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64)
        return VKLLM_ERR_DEV_NOT_FOUND;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev])
    {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess)
            return cuda_check(e, "cudaGetSymbolAddress(g_attn_noalloc_scratch)", __FILE__, __LINE__);
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return VKLLM_ERR_OK;
}

} // namespace
} // namespace vkb

extern "C" vkllm_err_t vkllm_b200_attention_decode_noalloc(const void *q, const void *kcache, const void *vcache,
                                                           uint32_t heads, uint32_t head_dim, uint32_t cache_rows,
                                                           uint32_t n_keys, float scale, void *out, void *stream)
{
    using namespace vkb;
    _CHECK_ARGS(q && kcache && vcache && out);
    _CHECK_ARGS(heads > 0 && head_dim > 0 && cache_rows > 0);
    _CHECK_ARGS(n_keys >= 1 && n_keys <= cache_rows);
    // Cache rows are read as 8-byte words (k_dec_attn_scores, k_dec_attn_pv); q and out per half.
    _CHECK_ARGS((((uintptr_t)kcache | (uintptr_t)vcache) & 7u) == 0);
    _CHECK_ARGS((((uintptr_t)q | (uintptr_t)out) & 1u) == 0);
    if (heads > kNoAllocMaxHeads || head_dim > kNoAllocMaxHeadDim || head_dim % 4 != 0 ||
        (uint64_t)heads * cache_rows > kNoAllocMaxScoreRows)
    {
        log_error("vkllm_b200_attention_decode_noalloc: heads=%u head_dim=%u cache_rows=%u exceed the static scratch "
                  "(heads <= %u, head_dim <= %u and a multiple of 4, heads * cache_rows <= %u)",
                  heads, head_dim, cache_rows, kNoAllocMaxHeads, kNoAllocMaxHeadDim, kNoAllocMaxScoreRows);
        return VKLLM_ERR_ARGS;
    }
    void *base = nullptr;
    _CHECK(noalloc_scratch(&base));
    char *sb = (char *)base;
    cudaStream_t s = (cudaStream_t)stream;
    LayerW lw;
    memset(&lw, 0, sizeof(lw));
    lw.kcache = (__half *)kcache;
    lw.vcache = (__half *)vcache;
    DecodeDims dd;
    memset(&dd, 0, sizeof(dd));
    dd.H = heads;
    dd.hd = head_dim;
    dd.ctx = cache_rows;
    dd.nsplit = kNoAllocSplits;
    dd.scale = scale;
    StepState *st = (StepState *)(sb + kNoAllocOffState);
    uint32_t *counters = (uint32_t *)(sb + kNoAllocOffCounters);
    // The array keeps the previous call's contents: the completion counters must start at zero.
    VKB_CUDA(cudaMemsetAsync(counters, 0, (size_t)heads * 4, s));
    k_set_state<<<1, 1, 0, s>>>(st, nullptr, 0, n_keys - 1);
    dim3 grid(heads, kNoAllocSplits);
    k_dec_attn_scores<<<grid, kAttnThreads, 0, s>>>(lw, dd, (const __half *)q, (__half *)sb, (float2 *)(sb + kNoAllocOffPart),
                                                   st);
    k_dec_attn_pv<<<grid, kAttnThreads, 0, s>>>(lw, dd, (const __half *)sb, (const float2 *)(sb + kNoAllocOffPart),
                                                (float *)(sb + kNoAllocOffOpart), counters, (__half *)out, st);
    VKB_CUDA(cudaGetLastError());
    return VKLLM_ERR_OK;
}

extern "C" uint32_t vkllm_b200_engine_last_launches(struct vkllm_context *context, struct vkllm_models_llama2 *model)
{
    if (!context || !model || !model->b200.engine)
        return 0;
    return ((Engine *)model->b200.engine)->launches;
}

extern "C" int vkllm_b200_engine_is_persistent(struct vkllm_context *context, struct vkllm_models_llama2 *model)
{
    if (!context || !model || !model->b200.engine)
        return 0;
    return ((Engine *)model->b200.engine)->persistent ? 1 : 0;
}

// Copies the barrier timestamps of the last persistent launch (CTA 0, %globaltimer ns): entry 0 is
// the kernel start, then one (arrival, release) pair per grid barrier. Returns the entry count.
extern "C" uint32_t vkllm_b200_engine_read_trace(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                 uint64_t *out, uint32_t cap)
{
    if (!context || !model || !model->b200.engine || !out)
        return 0;
    Engine *e = (Engine *)model->b200.engine;
    if (!e->pp.trace)
        return 0;
    cudaStreamSynchronize(context->runtime->stream);
    uint32_t n = cap < e->pp.trace_cap ? cap : e->pp.trace_cap;
    if (cudaMemcpy(out, e->pp.trace, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return n;
}

// %globaltimer of the last CTA's arrival per trace entry (at the release entry index of each grid
// barrier; other entries undefined). Returns the entry count, 0 when tracing is off.
extern "C" uint32_t vkllm_b200_engine_read_trace_last(struct vkllm_context *context,
                                                      struct vkllm_models_llama2 *model, uint64_t *out,
                                                      uint32_t cap)
{
    if (!context || !model || !model->b200.engine || !out)
        return 0;
    Engine *e = (Engine *)model->b200.engine;
    if (!e->pp.trace_last)
        return 0;
    cudaStreamSynchronize(context->runtime->stream);
    uint32_t n = cap < e->pp.trace_cap ? cap : e->pp.trace_cap;
    if (cudaMemcpy(out, e->pp.trace_last, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return n;
}

extern "C" uint32_t vkllm_b200_engine_read_cta_trace(struct vkllm_context *context,
                                                     struct vkllm_models_llama2 *model, uint64_t *out, uint32_t cap)
{
    if (!context || !model || !model->b200.engine || !out)
        return 0;
    Engine *e = (Engine *)model->b200.engine;
    if (!e->pp.trace_cta)
        return 0;
    cudaStreamSynchronize(context->runtime->stream);
    const uint32_t total = kCtaTraceBarriers * (uint32_t)e->ctx->device->sm_count;
    const uint32_t n = cap < total ? cap : total;
    if (cudaMemcpy(out, e->pp.trace_cta, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return n;
}

// Per-warp pipeline accounting of CTA 0 accumulated over all persistent launches since the engine
// was built (SM cycles): [warp][kind QKV, Wo, up/gate, down, logits][wait, consume, chunks, the
// compute share of consume]. Returns the entry count (32 * 5 * 4), 0 when tracing is off.
extern "C" uint32_t vkllm_b200_engine_read_warp_trace(struct vkllm_context *context,
                                                      struct vkllm_models_llama2 *model, uint64_t *out,
                                                      uint32_t cap)
{
    uint32_t n = kStreamMaxWarps * PK_COUNT * 4;
    if (!context || !model || !model->b200.engine || !out || cap < n)
        return 0;
    if (cap >= n + kAttTraceSlots)
        n += kAttTraceSlots;
    Engine *e = (Engine *)model->b200.engine;
    if (!e->pp.wtrace)
        return 0;
    cudaStreamSynchronize(context->runtime->stream);
    if (cudaMemcpy(out, e->pp.wtrace, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    return n;
}

// ------------------------------------------------------------------------------------------------
// Tensor parallelism: the peer-memory exchange between the ranks of a sharded model.

namespace vkb
{
void tp_comm_free(vkllm_models_llama2 *model)
{
    TpComm *c = (TpComm *)model->b200.tp_comm;
    if (!c)
        return;
    cudaDeviceSynchronize();
    for (uint32_t q = 0; q < c->world; ++q)
        if (q != c->rank && c->peer[q])
            cudaIpcCloseMemHandle(c->peer[q]);
    if (c->buf)
        cudaFree(c->buf);
    if (c->nccl)
        nccl_api()->CommDestroy(c->nccl);
    delete c;
    model->b200.tp_comm = nullptr;
}
} // namespace vkb

extern "C" vkllm_err_t vkllm_b200_tp_nccl_unique_id(void *id_out)
{
    _CHECK_ARGS(id_out);
    const NcclApi *nc = nccl_api();
    if (!nc)
        return VKLLM_ERR_VULKAN;
    ncclUniqueId id;
    ncclResult_t r = nc->GetUniqueId(&id);
    if (r != ncclSuccess)
    {
        log_error("ncclGetUniqueId: %s", nc->GetErrorString(r));
        return VKLLM_ERR_VULKAN;
    }
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(id_out, &id, sizeof(id));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_tp_nccl_connect(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                  const void *id)
{
    _CHECK_ARGS(context && model && id);
    _CHECK_ARGS(model->b200.tp_size > 1 && model->b200.tp_size <= kTpMax && model->b200.tp_rank < model->b200.tp_size);
    _CHECK_ARGS(!model->b200.engine);
    TpComm *c = (TpComm *)model->b200.tp_comm;
    _CHECK_ARGS(!c || !c->nccl);
    const NcclApi *nc = nccl_api();
    if (!nc)
        return VKLLM_ERR_VULKAN;
    VKB_CUDA(cudaSetDevice(context->device->ordinal));
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    ncclResult_t r = nc->CommInitRank(&comm, (int)model->b200.tp_size, uid, (int)model->b200.tp_rank);
    if (r != ncclSuccess)
    {
        log_error("ncclCommInitRank: %s", nc->GetErrorString(r));
        return VKLLM_ERR_VULKAN;
    }
    if (!c)
    {
        c = new TpComm();
        c->rank = model->b200.tp_rank;
        c->world = model->b200.tp_size;
        c->D = model->meta.embedding_length;
        model->b200.tp_comm = c;
    }
    c->nccl = comm;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_tp_init(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                          void *handle_out)
{
    _CHECK_ARGS(context && model && handle_out);
    _CHECK_ARGS(model->b200.tp_size > 1 && model->b200.tp_size <= kTpMax && model->b200.tp_rank < model->b200.tp_size);
    _CHECK_ARGS(!model->b200.engine);
    _CHECK_ARGS(!model->b200.tp_comm || !((TpComm *)model->b200.tp_comm)->buf);
    const bool fresh = !model->b200.tp_comm;
    TpComm *c = fresh ? new TpComm() : (TpComm *)model->b200.tp_comm;
    c->rank = model->b200.tp_rank;
    c->world = model->b200.tp_size;
    c->D = model->meta.embedding_length;
    const TpLayout t = tp_layout(c->world, c->D);
    c->bytes = t.total;
    if (cudaMalloc(&c->buf, c->bytes) != cudaSuccess || cudaMemset(c->buf, 0, c->bytes) != cudaSuccess)
    {
        (void)cudaGetLastError();
        if (c->buf)
            cudaFree(c->buf);
        c->buf = nullptr;
        if (fresh)
            delete c;
        return VKLLM_ERR_ALLOC;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, c->buf) != cudaSuccess)
    {
        (void)cudaGetLastError();
        cudaFree(c->buf);
        c->buf = nullptr;
        if (fresh)
            delete c;
        return VKLLM_ERR_VULKAN;
    }
    memcpy(handle_out, &h, sizeof(h));
    c->peer[c->rank] = c->buf;
    model->b200.tp_comm = c;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_b200_tp_connect(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                             const void *handles)
{
    _CHECK_ARGS(context && model && handles && model->b200.tp_comm);
    TpComm *c = (TpComm *)model->b200.tp_comm;
    _CHECK_ARGS(!c->connected);
    const cudaIpcMemHandle_t *hs = (const cudaIpcMemHandle_t *)handles;
    for (uint32_t q = 0; q < c->world; ++q)
    {
        if (q == c->rank)
            continue;
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hs[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        {
            log_error("tensor parallel: opening the buffer of rank %u failed: %s", q,
                      cudaGetErrorString(cudaGetLastError()));
            for (uint32_t r = 0; r < q; ++r)
                if (r != c->rank && c->peer[r])
                {
                    cudaIpcCloseMemHandle(c->peer[r]);
                    c->peer[r] = nullptr;
                }
            return VKLLM_ERR_VULKAN;
        }
        c->peer[q] = p;
    }
    c->connected = true;
    return VKLLM_ERR_OK;
}
