// Launchers shared by the op layer and the engine.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace vkb
{

// Batched C[z] = act(scale * A[z] . B[z]^T) for fp16 A [M, K] and B [N, K], both K-contiguous, C
// [M, N] N-contiguous, fp32 accumulation; z enumerates the output's (b, c) batch with broadcast
// offsets for A and B.
struct GemmArgs
{
    const void *A, *B;
    void *C;
    uint32_t M, N, K;
    uint64_t lda, ldb, ldc;           // row strides in elements
    uint32_t batch_c;                 // output C extent (z = b * batch_c + c)
    uint32_t batch;                   // output B * C
    uint64_t a_sb, a_sc, b_sb, b_sc;  // batch strides in elements (0 where broadcast)
    uint64_t c_sb, c_sc;
    float scale;
    int act;
    uint32_t act_from = 0; // act applies to output columns >= act_from (0: all)
    uint32_t b_tiled = 0;  // B is a gemm_tile_b copy (batch 1 only; ldb and the B strides are unused)
    // Grouped B (batch 1, row-major B): when b_group_n > 0, rows [0, b_group_n) of B come from B, the
    // next b_group_n from B1, the next from B2 (N = 2 or 3 groups), each [b_group_n, K] with row
    // stride ldb; every tile size in use must divide b_group_n, else the launch reports false.
    const void *B1 = nullptr, *B2 = nullptr;
    uint32_t b_group_n = 0;
    // Launch as a programmatic dependent of the previous kernel in the stream: the CTAs start while
    // it runs and load the first stages of B before waiting for its completion, so B must not be
    // written by that kernel (weights). Everything else (A, C, the split-K workspace) is touched
    // only after the wait.
    uint32_t pdl = 0;
};

// Row sources of one tiled B operand: rows [0, rows[0]) come from ptr[0], the next rows[1] from
// ptr[1], ... (each source row-major [rows][K]).
struct TileSrcs
{
    static constexpr uint32_t kMax = 4;
    const __half *ptr[kMax];
    uint32_t rows[kMax];
    uint32_t n;
};

// Elements of the tiled copy of an [N, K] B operand: [ceil(N/128)][ceil(K/64)][128][64] fp16, each
// 128 x 64 tile (one k-block of 128 rows) contiguous, so that the GEMM's B loads read whole 16 KB
// runs of HBM instead of 128-byte pieces of 128 rows. Padding rows and columns are zero.
uint64_t gemm_tiled_b_elems(uint32_t N, uint32_t K);

// Writes the tiled copy of the row-concatenation of `src` (K columns each) to `dst`.
bool gemm_tile_b(const TileSrcs &src, uint32_t K, __half *dst, cudaStream_t s);

// Fills `g` from 4-D descriptors when the tensor-core path applies (B read as [N, K] with unit
// inner stride, all row strides multiples of 8 elements, 16-byte aligned bases). Returns false
// otherwise.
bool make_gemm_args(const Desc4 &da, const Desc4 &db, const Desc4 &dc, bool trans_b, const void *a, const void *b,
                    void *c, float scale, int act, GemmArgs *g);

// Enqueues the tcgen05 GEMM; returns false when it cannot run on this device / shape.
bool gemm_tcgen05_launch(const GemmArgs &g, cudaStream_t s);

// The tcgen05 GEMM (tile 0: 128 x 128, 1: 128 x 256; 2, 3: the same loading 64 rows of A per stage,
// for M <= 64) with K split `splits` ways, writing its fp32
// partial sums [splits][batch][M][N] to `ws` instead of C (no reduction is launched; the caller sums
// the partials in split order, then applies scale / act / fp16 as the plain GEMM would).
// *splits_used receives the split count (<= splits: every split gets at least one 64-deep k-block).
bool gemm_tcgen05_partials(const GemmArgs &g, cudaStream_t s, uint32_t splits, float *ws, uint32_t *splits_used,
                           uint32_t tile = 0);

// Sticky error word of the tcgen05 GEMM on device `dev` (bit 0: a bounded wait expired).
uint32_t gemm_tcgen05_error(int dev);

// Dense row-major launchers of the RMSNORM, BIN and ARG_MAX node kernels (ops/op_elementwise.cu),
// used by the fused prefill step. Each returns false when the operands do not fit its vector path.
bool launch_rmsnorm_rows(const __half *x, const float *g, __half *y, uint32_t rows, uint32_t W, float eps,
                         cudaStream_t s);
bool launch_bin_h(const __half *a, const __half *b, __half *out, uint64_t n, int op, cudaStream_t s);
// x = fp16(x + y) (the residual BIN), then n = RMSNORM(x) with gains g, per row of W.
bool launch_residual_rmsnorm_rows(__half *x, const __half *y, const float *g, __half *n, uint32_t rows, uint32_t W,
                                  float eps, cudaStream_t s);
bool launch_argmax_rows(const __half *x, uint32_t rows, uint32_t W, uint32_t *out, cudaStream_t s);
// Tensor map over a KV cache laid out [seqs][heads][cap][hd] fp16: dims {hd, cap, heads, seqs}, box
// {64, box_rows, 1, 1} with 128-byte swizzle (16-byte piece c of box row r stored at piece c ^ (r & 7)),
// zero fill past cap. Needs hd a multiple of 64 and box_rows a multiple of 8 up to 256. Cached per
// (address, shape).
bool encode_kv_rows_map(CUtensorMap *m, const __half *base, uint32_t hd, uint32_t cap, uint32_t heads, uint32_t seqs,
                        uint32_t box_rows);

} // namespace vkb
