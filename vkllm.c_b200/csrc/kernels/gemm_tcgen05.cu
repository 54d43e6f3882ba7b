// Tensor-core GEMM for sm_100a (tcgen05). Placeholder dispatch: the tensor-core kernel is not
// enabled yet, so every GEMM runs on the CUDA-core kernel of ops/op_matmul.cu.
#include "kernels.h"

namespace vkb
{

bool make_gemm_args(const Desc4 &da, const Desc4 &db, const Desc4 &dc, bool trans_b, const void *a, const void *b,
                    void *c, float scale, int act, GemmArgs *g)
{
    (void)da, (void)db, (void)dc, (void)trans_b, (void)a, (void)b, (void)c, (void)scale, (void)act, (void)g;
    return false;
}

bool gemm_tcgen05_launch(const GemmArgs &g, cudaStream_t s)
{
    (void)g, (void)s;
    return false;
}

} // namespace vkb
