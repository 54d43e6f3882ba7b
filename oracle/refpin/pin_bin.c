/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_bin.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, bin_op_host (tests/vkllm_test_op_bin.c:24-114), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_bin
#include "tests/vkllm_test_op_bin.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_bin(const void *a, const void *b, void *c, const uint32_t shapes[4], const uint32_t sa[4],
                               const uint32_t sb[4], const uint32_t sc[4], int dta, int dtb, int dtc, int32_t op)
{
    bin_op_host(a, b, c, shapes, sa, sb, sc, (vkllm_dtype_t)dta, (vkllm_dtype_t)dtb, (vkllm_dtype_t)dtc, op);
}
