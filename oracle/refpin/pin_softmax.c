/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_softmax.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, softmax_op_host (tests/vkllm_test_op_softmax.c:14-119), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_softmax
#include "tests/vkllm_test_op_softmax.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_softmax(const void *x, void *y, const uint32_t shapes[4], const uint32_t strides[4],
                                   int dtype, int32_t seq_mask, uint32_t offsets)
{
    softmax_op_host(x, y, shapes, strides, (vkllm_dtype_t)dtype, seq_mask, offsets);
}
