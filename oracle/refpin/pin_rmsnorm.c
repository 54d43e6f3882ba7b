/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_rmsnorm.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, rmsnorm_op_host (tests/vkllm_test_op_rmsnorm.c:14-106), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_rmsnorm
#include "tests/vkllm_test_op_rmsnorm.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_rmsnorm(const void *x, const void *g, void *y, const uint32_t shapes[4],
                                   const uint32_t strides[4], const uint32_t g_strides[4], int x_dtype, int g_dtype,
                                   int y_dtype)
{
    rmsnorm_op_host(x, g, y, shapes, strides, g_strides, (vkllm_dtype_t)x_dtype, (vkllm_dtype_t)g_dtype,
                    (vkllm_dtype_t)y_dtype);
}
