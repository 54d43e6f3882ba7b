/* TEST INFRASTRUCTURE (oracle pin). Compiles the reference's own tests/vkllm_test_op_embedding.c from
 * where it lies (the include path points at the reference checkout) and exports its CPU reference
 * function, embedding_op_host (tests/vkllm_test_op_embedding.c:32-94), so that golden vectors come from the reference's code. The file's GPU test
 * bodies are compiled but unreachable and dropped at link time; nothing of this library reaches
 * the product. */
#define main refpin_unused_main_embedding
#include "tests/vkllm_test_op_embedding.c"
#undef main
#define REFPIN_EXPORT __attribute__((visibility("default")))

REFPIN_EXPORT void refpin_embedding(const uint32_t *ids, const void *table, void *out, const uint32_t id_shapes[4],
                                     const uint32_t table_shapes[4], const uint32_t out_shapes[4],
                                     const uint32_t id_strides[4], const uint32_t table_strides[4],
                                     const uint32_t out_strides[4], int dtype)
{
    embedding_op_host(ids, table, out, id_shapes, table_shapes, out_shapes, id_strides, table_strides, out_strides,
                      (vkllm_dtype_t)dtype);
}
