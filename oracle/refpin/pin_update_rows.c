/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_update_rows.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, update_rows_op_host (tests/vkllm_test_op_update_rows.c:75-122), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_update_rows
#include "tests/vkllm_test_op_update_rows.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_update_rows(const void *src, void *cache, const uint32_t in_shapes[4],
                                       const uint32_t in_strides[4], const uint32_t out_shapes[4],
                                       const uint32_t out_strides[4], uint32_t offset_rows, int dtype)
{
    update_rows_op_host(src, cache, in_shapes, in_strides, out_shapes, out_strides, offset_rows, (vkllm_dtype_t)dtype);
}
