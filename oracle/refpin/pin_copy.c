/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_copy.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, copy_op_host (tests/vkllm_test_op_copy.c:16-68), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_copy
#include "tests/vkllm_test_op_copy.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_copy(const void *x, void *y, const uint32_t shapes[4], const uint32_t strides[4],
                                const uint32_t out_strides[4], int dtype)
{
    copy_op_host(x, y, shapes, strides, out_strides, (vkllm_dtype_t)dtype);
}
