// The reference's token loop (tests/vkllm_test_infer_gguf.c:181-272) as one C-ABI call: per token a
// mapped input tensor, a new graph, vkllm_models_llama2_build_graph, vkllm_graph_init, the upload of
// the ids, vkllm_graph_run, vkllm_graph_post_run, the read of the last row of the mapped argmax
// output and vkllm_graph_free, all through the public entry points. It lets a caller (or a
// benchmark) drive the API loop from native code instead of paying a binding's per-call overhead.
#include <chrono>
#include <cstring>

#include "../runtime/internal.h"
#include "vkllm_b200.h"
#include "vkllm_models_llama2.h"

namespace
{

// Last row of the mapped u32 output [B, C, S, 1] (extract_output_tok of the reference loop).
uint32_t last_row_token(const vkllm_tensor *out)
{
    const uint32_t *d = (const uint32_t *)out->data.host;
    const uint64_t i = (uint64_t)(out->shapes[0] - 1) * (out->strides[0] / 4) +
                       (uint64_t)(out->shapes[1] - 1) * (out->strides[1] / 4) +
                       (uint64_t)(out->shapes[2] - 1) * (out->strides[2] / 4);
    return d[i];
}

} // namespace

extern "C" vkllm_err_t vkllm_b200_token_loop(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                             const uint32_t *prompt, uint32_t n_prompt, uint32_t offset,
                                             uint32_t n_tokens, uint32_t *out_tokens, double *host_us)
{
    _CHECK_ARGS(context && model && prompt && n_prompt > 0 && out_tokens);
    using clk = std::chrono::steady_clock;
    double host = 0.0;
    const uint32_t *ids = prompt;
    uint32_t n_ids = n_prompt, next = 0;
    for (uint32_t i = 0; i < n_tokens; ++i)
    {
        const auto t0 = clk::now();
        vkllm_tensor *input = nullptr;
        const uint32_t shape[4] = {1, 1, 1, n_ids};
        _CHECK(vkllm_tensor_new(context, "input_toks", shape, vkllm_dtype_uint32, VKLLM_OP_NONE, NULL, 0, NULL, 0,
                                true, &input));
        vkllm_graph *graph = nullptr;
        vkllm_err_t e = vkllm_graph_new(context, &graph);
        if (e != VKLLM_ERR_OK)
        {
            vkllm_tensor_free(context, input);
            return e;
        }
        e = vkllm_models_llama2_build_graph(context, model, input, graph, offset);
        if (e != VKLLM_ERR_OK && graph->nodes->used_n == 0) // the input never reached the graph
            vkllm_tensor_free(context, input);
        if (e == VKLLM_ERR_OK)
            e = vkllm_graph_init(context, graph);
        if (e == VKLLM_ERR_OK)
            e = vkllm_commands_upload(context, graph->commands, input, (const uint8_t *)ids,
                                      sizeof(uint32_t) * n_ids);
        const auto t1 = clk::now();
        if (e == VKLLM_ERR_OK)
            e = vkllm_graph_run(context, graph);
        const auto t2 = clk::now();
        if (e == VKLLM_ERR_OK)
            e = vkllm_graph_post_run(context, graph);
        if (e == VKLLM_ERR_OK)
            e = vkllm_tensor_invalid_cache(context, graph->output_node);
        if (e == VKLLM_ERR_OK)
            next = last_row_token(graph->output_node);
        vkllm_graph_free(context, graph);
        host += std::chrono::duration<double, std::micro>(t1 - t0).count() +
                std::chrono::duration<double, std::micro>(clk::now() - t2).count();
        if (e != VKLLM_ERR_OK)
            return e;
        out_tokens[i] = next;
        offset += n_ids;
        ids = &out_tokens[i];
        n_ids = 1;
    }
    if (host_us)
        *host_us = host;
    return VKLLM_ERR_OK;
}
