// VKLLM_OP_MATMUL and VKLLM_OP_FFN_UP_AND_GATE for the op-by-op executor
// (reference host: src/core/vkllm_op_matmul.c, src/core/vkllm_op_ffn_up_and_gate.c).
//
// Kernel choice follows the reference predicates (src/core/vkllm_op_matmul.c:14-30):
//   transposed_b = A.H == M && B.H == N && A.W == K && B.W == K   (B read as [N, K])
//   mat_mul_vec  = A.H == 1 && transposed_b                        (decode GEMV)
// fp16 GEMMs with 16-byte-aligned, K-contiguous operands run on the tcgen05 tensor-core kernel
// (kernels/gemm_tcgen05.cu); everything else on the CUDA-core kernels below. Accumulation is fp32.
#include <cfloat>

#include "../kernels/common.cuh"
#include "../kernels/kernels.h"
#include "../runtime/internal.h"
#include "vkllm_op_ffn_up_and_gate.h"
#include "vkllm_op_matmul.h"

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

bool is_transposed_b(const vkllm_tensor *t)
{
    const vkllm_tensor *a = t->srcs[0], *b = t->srcs[1];
    uint32_t M = t->shapes[2], N = t->shapes[3], K = a->shapes[3];
    return a->shapes[2] == M && b->shapes[2] == N && a->shapes[3] == K && b->shapes[3] == K;
}

bool is_mat_mul_vec(const vkllm_tensor *t)
{
    return t->srcs[0]->shapes[2] == 1 && is_transposed_b(t);
}

// ------------------------------------------------------------------------------------------------
// GEMV, one warp per output element (src/shaders/vkllm_mat_mul_vec.comp:94-150). Batch offsets use
// the channel index only, as the reference's unspecialised GEMV pipelines do
// (src/core/vkllm_pipeline.c:659-667 leave a/b_boardcast_type = AXIS0); a size-1 channel axis is
// reused instead of being read past its end.
template <typename T, bool VEC>
__global__ void k_gemv(const T *a, Desc4 da, const T *w, Desc4 dw, T *out, Desc4 dout, float scale, int act)
{
    uint64_t n_out = d4_count(dout);
    uint64_t gw = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (; gw < n_out; gw += nwarps)
    {
        uint32_t b, c, h, col;
        d4_unravel(dout.shape, gw, b, c, h, col);
        uint64_t a_off = (uint64_t)(da.shape[1] == 1 ? 0 : c) * da.stride[1] + (uint64_t)h * da.stride[2];
        uint64_t w_off = (uint64_t)(dw.shape[1] == 1 ? 0 : c) * dw.stride[1] + (uint64_t)col * dw.stride[2];
        uint32_t K = da.shape[3];
        float acc = 0.f;
        if constexpr (VEC)
        {
            // 16-byte chunks of 8 halves; K % 8 == 0 and 16-byte aligned rows are checked on the host.
            const uint4 *ap = reinterpret_cast<const uint4 *>(a + a_off);
            const uint4 *wp = reinterpret_cast<const uint4 *>(w + w_off);
            uint32_t nchunk = K / 8, i = lane;
            // eight 16-byte weight loads in flight per lane, summed in the same chunk order
            for (; i + 32 * 7 < nchunk; i += 32 * 8)
            {
                uint4 wv[8], av[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                {
                    wv[u] = ldg_stream(wp + i + 32 * u);
                    av[u] = ap[i + 32 * u];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    acc = dot8_f16(av[u], wv[u], acc);
            }
            for (; i < nchunk; i += 32)
                acc = dot8_f16(ap[i], ldg_stream(wp + i), acc);
        }
        else
        {
            for (uint32_t k = lane; k < K; k += 32)
                acc = fmaf(to_f32(a[a_off + (uint64_t)k * da.stride[3]]), to_f32(w[w_off + (uint64_t)k * dw.stride[3]]),
                           acc);
        }
        acc = warp_sum(acc) * scale;
        if (act == 1)
            acc = silu_f32(acc);
        if (lane == 0)
            out[d4_offset(dout, b, c, h, col)] = from_f32<T>(acc);
    }
}

// k_gemv for one input row (A [1, 1, 1, K], W rows contiguous, every output in one row): the row is
// staged once per block in shared memory, and each lane keeps 16 weight chunks of 16 bytes in flight
// instead of 8, so a 4096-wide row is one round trip to HBM. Each lane adds its chunks in the same
// order as k_gemv (i, i + 32, ...), then the same warp sum: the same bits.
constexpr uint32_t kGemvWideMaxK = 16384; // halves of the staged input row (32 KB)

// ldg_stream without `volatile`, so that the compiler may issue a whole group of these loads before
// the arithmetic that uses the first (a volatile load orders after the preceding dot products).
__device__ __forceinline__ uint4 ldg_stream_sched(const void *p)
{
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__global__ void __launch_bounds__(256) k_gemv_row(const __half *__restrict__ a, const __half *__restrict__ w,
                                                  uint64_t ldw, __half *__restrict__ out, uint32_t N, uint32_t K,
                                                  float scale, int act)
{
    __shared__ __align__(16) uint4 xs[kGemvWideMaxK / 8];
    const uint32_t nchunk = K / 8, lane = threadIdx.x & 31;
    for (uint32_t i = threadIdx.x; i < nchunk; i += blockDim.x)
        xs[i] = reinterpret_cast<const uint4 *>(a)[i];
    __syncthreads();
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += warps)
    {
        const uint4 *wp = reinterpret_cast<const uint4 *>(w + (uint64_t)n * ldw);
        float acc = 0.f;
        uint32_t i = lane;
        for (; i + 32 * 15 < nchunk; i += 32 * 16)
        {
            uint4 wv[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                wv[u] = ldg_stream_sched(wp + i + 32 * u);
#pragma unroll
            for (int u = 0; u < 16; ++u)
                acc = dot8_f16(xs[i + 32 * u], wv[u], acc);
        }
        for (; i < nchunk; i += 32)
            acc = dot8_f16(xs[i], ldg_stream_sched(wp + i), acc);
        acc = warp_sum(acc) * scale;
        if (act == 1)
            acc = silu_f32(acc);
        if (lane == 0)
            out[n] = __float2half_rn(acc);
    }
}

// ------------------------------------------------------------------------------------------------
// CUDA-core GEMM for any strides / broadcast / layout (src/shaders/vkllm_matmul_t0.comp,
// vkllm_matmul_t1.comp): 64x64 output tile per 256-thread block, 4x4 per thread, fp32 accumulation.
// B is [N, K] when TRANS_B, else [K, N].
template <typename T, bool TRANS_B>
__global__ void __launch_bounds__(256) k_gemm_simt(const T *A, Desc4 da, const T *B, Desc4 db, T *C, Desc4 dc,
                                                   float scale, int act)
{
    constexpr int BM = 64, BN = 64, BK = 16;
    __shared__ float sa[BK][BM + 4];
    __shared__ float sb[BK][BN + 4];
    uint32_t M = dc.shape[2], N = dc.shape[3], K = da.shape[3];
    uint32_t z = blockIdx.z;
    uint32_t cb = z / dc.shape[1], cc = z % dc.shape[1];
    uint64_t a_off = (uint64_t)(da.shape[0] == 1 ? 0 : cb) * da.stride[0] + (uint64_t)(da.shape[1] == 1 ? 0 : cc) * da.stride[1];
    uint64_t b_off = (uint64_t)(db.shape[0] == 1 ? 0 : cb) * db.stride[0] + (uint64_t)(db.shape[1] == 1 ? 0 : cc) * db.stride[1];
    uint64_t c_off = (uint64_t)cb * dc.stride[0] + (uint64_t)cc * dc.stride[1];
    uint32_t m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < K; k0 += BK)
    {
        for (int i = threadIdx.x; i < BM * BK; i += 256)
        {
            int r = i / BK, kk = i % BK;
            uint32_t m = m0 + r, k = k0 + kk;
            float v = 0.f;
            if (m < M && k < K)
                v = to_f32(A[a_off + (uint64_t)m * da.stride[2] + (uint64_t)k * da.stride[3]]);
            sa[kk][r] = v;
        }
        for (int i = threadIdx.x; i < BN * BK; i += 256)
        {
            int r = i / BK, kk = i % BK;
            uint32_t n = n0 + r, k = k0 + kk;
            float v = 0.f;
            if (n < N && k < K)
            {
                if (TRANS_B)
                    v = to_f32(B[b_off + (uint64_t)n * db.stride[2] + (uint64_t)k * db.stride[3]]);
                else
                    v = to_f32(B[b_off + (uint64_t)k * db.stride[2] + (uint64_t)n * db.stride[3]]);
            }
            sb[kk][r] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk)
        {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                av[i] = sa[kk][ty * 4 + i];
                bv[i] = sb[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        uint32_t m = m0 + ty * 4 + i;
        if (m >= M)
            continue;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            uint32_t n = n0 + tx * 4 + j;
            if (n >= N)
                continue;
            float v = acc[i][j] * scale;
            if (act == 1)
                v = silu_f32(v);
            C[c_off + (uint64_t)m * dc.stride[2] + (uint64_t)n * dc.stride[3]] = from_f32<T>(v);
        }
    }
}

// FFN_UP_AND_GATE intended math (src/shaders/vkllm_ffn_up_and_gate.comp:137-146):
// y = u * g / (1 + exp(-g)) with u = x.Wu^T, g = x.Wg^T in fp32. One warp per output element.
template <typename TI, typename TO>
__global__ void k_ffn_up_gate(const TI *x, Desc4 dx, const TI *wu, Desc4 du, const TI *wg, Desc4 dg, TO *out,
                              Desc4 dout)
{
    uint64_t n_out = d4_count(dout);
    uint64_t gw = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
    uint32_t lane = threadIdx.x & 31;
    uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (; gw < n_out; gw += nwarps)
    {
        uint32_t b, c, m, n;
        d4_unravel(dout.shape, gw, b, c, m, n);
        uint64_t xo = d4_offset(dx, b, c, m, 0);
        uint64_t uo = (uint64_t)n * du.stride[2], go = (uint64_t)n * dg.stride[2];
        float su = 0.f, sg = 0.f;
        for (uint32_t k = lane; k < dx.shape[3]; k += 32)
        {
            float xv = to_f32(x[xo + (uint64_t)k * dx.stride[3]]);
            su = fmaf(xv, to_f32(wu[uo + (uint64_t)k * du.stride[3]]), su);
            sg = fmaf(xv, to_f32(wg[go + (uint64_t)k * dg.stride[3]]), sg);
        }
        su = warp_sum(su);
        sg = warp_sum(sg);
        if (lane == 0)
            out[d4_offset(dout, b, c, m, n)] = from_f32<TO>(su * sg / (1.0f + expf(-sg)));
    }
}

vkllm_err_t launch_status(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return cuda_check(e, what, __FILE__, __LINE__);
    return VKLLM_ERR_OK;
}

bool broadcast_ok(uint32_t in, uint32_t out)
{
    return in == out || in == 1;
}

} // namespace

extern "C" vkllm_err_t vkllm_op_matmul_init(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0] && tensor->srcs[1]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_MATMUL);
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    uint32_t M = tensor->shapes[2], N = tensor->shapes[3], K = in0->shapes[3];
    bool tb = is_transposed_b(tensor);
    _CHECK_ARGS(in0->shapes[2] == M);
    if (tb)
        _CHECK_ARGS(in1->shapes[3] == K && in1->shapes[2] == N);
    else
        _CHECK_ARGS(in1->shapes[3] == N && in1->shapes[2] == K);
    _CHECK_ARGS(broadcast_ok(in0->shapes[0], tensor->shapes[0]) && broadcast_ok(in1->shapes[0], tensor->shapes[0]));
    _CHECK_ARGS(broadcast_ok(in0->shapes[1], tensor->shapes[1]) && broadcast_ok(in1->shapes[1], tensor->shapes[1]));
    bool vec = is_mat_mul_vec(tensor);
    if (in0->dtype == vkllm_dtype_float16 && in1->dtype == vkllm_dtype_float16)
    {
        if (tensor->dtype != vkllm_dtype_float16)
        {
            log_error("input dtype = fp16 and output dtype != fp16");
            return VKLLM_ERR_PIPELINE_NOT_FOUND;
        }
        tensor->pipeline = get_pipeline(context, vec ? "mat_mul_vec_f16f32" : (tb ? "matmul_t1_f16f32f16" : "matmul_t0_f16f32f16"),
                                        VKLLM_OP_MATMUL, vec ? 0 : (tb ? 1 : 2));
    }
    else if (in0->dtype == vkllm_dtype_float32 && in1->dtype == vkllm_dtype_float32)
    {
        if (tensor->dtype != vkllm_dtype_float32)
            return VKLLM_ERR_PIPELINE_NOT_FOUND;
        tensor->pipeline = get_pipeline(context, vec ? "mat_mul_vec_f32f32" : (tb ? "matmul_t1_f32f32f32" : "matmul_t0_f32f32f32"),
                                        VKLLM_OP_MATMUL, vec ? 3 : (tb ? 4 : 5));
    }
    else
        return VKLLM_ERR_PIPELINE_NOT_FOUND;
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

// B [Bb, Cb, K, N] (N contiguous) -> dense Bt [Bb * Cb][N][K]: 32 x 32 tiles through shared memory.
__global__ void k_transpose_kn(const __half *__restrict__ b, Desc4 db, __half *__restrict__ bt)
{
    __shared__ __half tile[32][33];
    const uint32_t K = db.shape[2], N = db.shape[3], z = blockIdx.z;
    const uint32_t zb = z / db.shape[1], zc = z % db.shape[1];
    const __half *src = b + (uint64_t)zb * db.stride[0] + (uint64_t)zc * db.stride[1];
    __half *dst = bt + (uint64_t)z * N * K;
    const uint32_t k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const uint32_t k = k0 + i, n = n0 + threadIdx.x;
        tile[i][threadIdx.x] = (k < K && n < N) ? src[(uint64_t)k * db.stride[2] + (uint64_t)n * db.stride[3]]
                                                : __float2half(0.f);
    }
    __syncthreads();
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y)
    {
        const uint32_t n = n0 + i, k = k0 + threadIdx.x;
        if (n < N && k < K)
            dst[(uint64_t)n * K + k] = tile[threadIdx.x][i];
    }
}

// C = A . B for B read as [K, N] (the attention probs . V product): B is transposed into a dense
// [N, K] scratch from the context's allocator, then the tensor-core GEMM runs with B^T. The scratch
// goes back to the cache right after the enqueue; the context's single stream orders its reuse.
bool matmul_tc_via_transpose(vkllm_context *context, const Desc4 &da, const Desc4 &db, const Desc4 &dc, const void *a,
                             const void *b, void *c, float scale, int act, cudaStream_t s)
{
    const uint32_t K = db.shape[2], N = db.shape[3], zn = db.shape[0] * db.shape[1];
    if (K % 8 != 0 || K != da.shape[3] || N != dc.shape[3] || zn == 0)
        return false;
    size_t cap = 0;
    const size_t bytes = (size_t)zn * N * K * sizeof(__half);
    void *bt = context->runtime->dev_alloc->alloc(bytes, &cap);
    if (!bt)
        return false;
    k_transpose_kn<<<dim3((N + 31) / 32, (K + 31) / 32, zn), dim3(32, 8), 0, s>>>((const __half *)b, db, (__half *)bt);
    Desc4 dbt;
    dbt.shape[0] = db.shape[0];
    dbt.shape[1] = db.shape[1];
    dbt.shape[2] = N;
    dbt.shape[3] = K;
    dbt.stride[3] = 1;
    dbt.stride[2] = K;
    dbt.stride[1] = N * K;
    dbt.stride[0] = db.shape[1] * N * K;
    GemmArgs g;
    bool ok = make_gemm_args(da, dbt, dc, true, a, bt, c, scale, act, &g) && gemm_tcgen05_launch(g, s);
    context->runtime->dev_alloc->release(bt);
    return ok;
}

extern "C" vkllm_err_t vkllm_op_matmul_run(vkllm_context *context, vkllm_commands *commands, vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor && tensor->srcs[0] && tensor->srcs[1]);
    // Shapes of graph nodes can change between runs (KV slices grow), so re-select every run.
    _CHECK(vkllm_op_matmul_init(context, commands, tensor));
    vkllm_tensor *in0 = tensor->srcs[0], *in1 = tensor->srcs[1];
    const vkllm_op_matmul_params *p = (const vkllm_op_matmul_params *)tensor->params;
    void *a = dev_ptr(context, in0), *b = dev_ptr(context, in1), *c = dev_ptr(context, tensor);
    _CHECK_ARGS(a && b && c);
    cudaStream_t s = stream_of(context, commands);
    Desc4 da = desc_of(in0), db = desc_of(in1), dc = desc_of(tensor);
    bool f16 = in0->dtype == vkllm_dtype_float16;
    timing_begin(context, tensor->pipeline, s);
    if (is_mat_mul_vec(tensor))
    {
        uint64_t n_out = d4_count(dc);
        unsigned grid = grid_1d(n_out * 32, 256);
        if (grid > 148u * 64u)
            grid = 148u * 64u;
        bool vec_ok = f16 && da.stride[3] == 1 && db.stride[3] == 1 && da.shape[3] % 8 == 0 &&
                      da.stride[1] % 8 == 0 && da.stride[2] % 8 == 0 && db.stride[1] % 8 == 0 &&
                      db.stride[2] % 8 == 0 && ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0;
        const bool one_row = n_out == dc.shape[3] && dc.stride[3] == 1 && da.shape[3] <= kGemvWideMaxK;
        if (f16 && vec_ok && one_row)
        {
            static int per_sm[64] = {};
            int dev = 0;
            cudaGetDevice(&dev);
            if (dev >= 0 && dev < 64 && per_sm[dev] == 0 &&
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[dev], k_gemv_row, 256, 0) != cudaSuccess)
            {
                (void)cudaGetLastError();
                per_sm[dev] = 1;
            }
            const uint64_t rows_grid = (n_out + 7) / 8;
            const uint64_t resident = (uint64_t)context->device->sm_count * (uint64_t)(per_sm[dev] > 0 ? per_sm[dev] : 1);
            k_gemv_row<<<(unsigned)(rows_grid < resident ? rows_grid : resident), 256, 0, s>>>(
                (const __half *)a, (const __half *)b, db.stride[2], (__half *)c, dc.shape[3], da.shape[3], p->scale,
                p->act);
        }
        else if (f16 && vec_ok)
            k_gemv<__half, true><<<grid, 256, 0, s>>>((const __half *)a, da, (const __half *)b, db, (__half *)c, dc,
                                                       p->scale, p->act);
        else if (f16)
            k_gemv<__half, false><<<grid, 256, 0, s>>>((const __half *)a, da, (const __half *)b, db, (__half *)c, dc,
                                                        p->scale, p->act);
        else
            k_gemv<float, false><<<grid, 256, 0, s>>>((const float *)a, da, (const float *)b, db, (float *)c, dc,
                                                       p->scale, p->act);
    }
    else
    {
        bool tb = is_transposed_b(tensor);
        bool done = false;
        if (f16)
        {
            // Tensor-core path: A [M,K] and B [N,K] with unit inner stride.
            GemmArgs g;
            if (tb && make_gemm_args(da, db, dc, tb, a, b, c, p->scale, p->act, &g))
                done = gemm_tcgen05_launch(g, s);
            else if (!tb)
                done = matmul_tc_via_transpose(context, da, db, dc, a, b, c, p->scale, p->act, s);
        }
        if (!done)
        {
            dim3 grid((dc.shape[2] + 63) / 64, (dc.shape[3] + 63) / 64, dc.shape[0] * dc.shape[1]);
            if (f16 && tb)
                k_gemm_simt<__half, true><<<grid, 256, 0, s>>>((const __half *)a, da, (const __half *)b, db,
                                                                (__half *)c, dc, p->scale, p->act);
            else if (f16)
                k_gemm_simt<__half, false><<<grid, 256, 0, s>>>((const __half *)a, da, (const __half *)b, db,
                                                                 (__half *)c, dc, p->scale, p->act);
            else if (tb)
                k_gemm_simt<float, true><<<grid, 256, 0, s>>>((const float *)a, da, (const float *)b, db, (float *)c,
                                                               dc, p->scale, p->act);
            else
                k_gemm_simt<float, false><<<grid, 256, 0, s>>>((const float *)a, da, (const float *)b, db,
                                                                (float *)c, dc, p->scale, p->act);
        }
    }
    timing_end(context, tensor->pipeline, s);
    return launch_status("matmul");
}

extern "C" vkllm_err_t vkllm_op_matmul_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}

// =================================================================================================
extern "C" vkllm_err_t vkllm_op_ffn_up_and_gate_init(vkllm_context *context, vkllm_commands *commands,
                                                     vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    _CHECK_ARGS(tensor->srcs[0] && tensor->srcs[1] && tensor->srcs[2]);
    _CHECK_ARGS(tensor->op == VKLLM_OP_FFN_UP_AND_GATE);
    vkllm_tensor *x = tensor->srcs[0], *wu = tensor->srcs[1], *wg = tensor->srcs[2];
    _CHECK_ARGS(x->dtype == wu->dtype && x->dtype == wg->dtype);
    _CHECK_ARGS(wu->shapes[3] == x->shapes[3] && wg->shapes[3] == x->shapes[3]);
    _CHECK_ARGS(wu->shapes[2] == tensor->shapes[3] && wg->shapes[2] == tensor->shapes[3]);
    _CHECK_ARGS(x->shapes[0] == tensor->shapes[0] && x->shapes[1] == tensor->shapes[1] &&
                x->shapes[2] == tensor->shapes[2]);
    if (x->dtype == vkllm_dtype_float16)
    {
        if (tensor->dtype == vkllm_dtype_float16)
            tensor->pipeline = get_pipeline(context, "ffn_f16f32f16", VKLLM_OP_FFN_UP_AND_GATE, 0);
        else if (tensor->dtype == vkllm_dtype_float32)
            tensor->pipeline = get_pipeline(context, "ffn_f16f32f32", VKLLM_OP_FFN_UP_AND_GATE, 1);
        else
            return VKLLM_ERR_PIPELINE_NOT_FOUND;
    }
    else if (x->dtype == vkllm_dtype_float32 && tensor->dtype == vkllm_dtype_float32)
        tensor->pipeline = get_pipeline(context, "ffn_f32f32f32", VKLLM_OP_FFN_UP_AND_GATE, 2);
    else
        return VKLLM_ERR_PIPELINE_NOT_FOUND;
    return dev_ptr(context, tensor) ? VKLLM_ERR_OK : VKLLM_ERR_ALLOC;
}

extern "C" vkllm_err_t vkllm_op_ffn_up_and_gate_run(vkllm_context *context, vkllm_commands *commands,
                                                    vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && commands && tensor);
    if (!tensor->pipeline)
        _CHECK(vkllm_op_ffn_up_and_gate_init(context, commands, tensor));
    vkllm_tensor *x = tensor->srcs[0], *wu = tensor->srcs[1], *wg = tensor->srcs[2];
    void *px = dev_ptr(context, x), *pu = dev_ptr(context, wu), *pg = dev_ptr(context, wg),
         *po = dev_ptr(context, tensor);
    _CHECK_ARGS(px && pu && pg && po);
    cudaStream_t s = stream_of(context, commands);
    Desc4 dout = desc_of(tensor);
    unsigned grid = grid_1d(d4_count(dout) * 32, 256);
    if (grid > 148u * 64u)
        grid = 148u * 64u;
    timing_begin(context, tensor->pipeline, s);
    if (x->dtype == vkllm_dtype_float16 && tensor->dtype == vkllm_dtype_float16)
        k_ffn_up_gate<__half, __half><<<grid, 256, 0, s>>>((const __half *)px, desc_of(x), (const __half *)pu,
                                                            desc_of(wu), (const __half *)pg, desc_of(wg), (__half *)po,
                                                            dout);
    else if (x->dtype == vkllm_dtype_float16)
        k_ffn_up_gate<__half, float><<<grid, 256, 0, s>>>((const __half *)px, desc_of(x), (const __half *)pu,
                                                           desc_of(wu), (const __half *)pg, desc_of(wg), (float *)po,
                                                           dout);
    else
        k_ffn_up_gate<float, float><<<grid, 256, 0, s>>>((const float *)px, desc_of(x), (const float *)pu, desc_of(wu),
                                                          (const float *)pg, desc_of(wg), (float *)po, dout);
    timing_end(context, tensor->pipeline, s);
    return launch_status("ffn_up_and_gate");
}

extern "C" vkllm_err_t vkllm_op_ffn_up_and_gate_post_run(vkllm_context *, vkllm_commands *, vkllm_tensor *)
{
    return VKLLM_ERR_OK;
}
