/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_matmul.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, matmul_op_host (tests/vkllm_test_op_matmul.c:33-165), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_matmul
#include "tests/vkllm_test_op_matmul.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_matmul(const void *a, const void *b, void *c, uint32_t Ba, uint32_t Ca, uint32_t Bb,
                                  uint32_t Cb, uint32_t M, uint32_t K, uint32_t N, const uint32_t sa[4],
                                  const uint32_t sb[4], const uint32_t sc[4], int dtype, int transposed_b, int act)
{
    matmul_op_host(a, b, c, Ba, Ca, Bb, Cb, M, K, N, sa, sb, sc, (vkllm_dtype_t)dtype, transposed_b != 0, act != 0);
}
