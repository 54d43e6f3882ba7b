// Tensor-DAG executor (reference: src/core/vkllm_graph.c).
#include <cstdlib>
#include <unordered_set>

#include "internal.h"
#include "vkllm_op_arg_max.h"
#include "vkllm_op_bin.h"
#include "vkllm_op_copy.h"
#include "vkllm_op_embedding.h"
#include "vkllm_op_ffn_up_and_gate.h"
#include "vkllm_op_matmul.h"
#include "vkllm_op_rmsnorm.h"
#include "vkllm_op_rope.h"
#include "vkllm_op_softmax.h"
#include "vkllm_op_update_rows.h"

namespace vkb
{
// Fused LLaMA-2 step for graphs carrying a plan (engine/engine.cu). Returns VKLLM_ERR_ARGS
// when the plan does not apply, in which case the graph runs node by node.
vkllm_err_t plan_run(vkllm_context *ctx, vkllm_graph *graph);
void plan_free(vkllm_context *ctx, vkllm_graph *graph);
// Structural graph cache (models/graph_cache.cpp): true when the nodes after the input went back to it.
bool graph_cache_give(vkllm_context *ctx, vkllm_graph *graph);
} // namespace vkb

namespace
{

typedef vkllm_err_t (*op_fn)(vkllm_context *, vkllm_commands *, vkllm_tensor *);

struct OpEntry
{
    op_fn init, run, post_run;
};

const OpEntry *op_entry(vkllm_op_t op)
{
    static const OpEntry table[VKLLM_OP_COUNTS] = {
        {nullptr, nullptr, nullptr}, // NONE
        {vkllm_op_copy_init, vkllm_op_copy_run, vkllm_op_copy_post_run},
        {vkllm_op_bin_init, vkllm_op_bin_run, vkllm_op_bin_post_run},
        {vkllm_op_embedding_init, vkllm_op_embedding_run, vkllm_op_embedding_post_run},
        {vkllm_op_rmsnorm_init, vkllm_op_rmsnorm_run, vkllm_op_rmsnorm_post_run},
        {vkllm_op_matmul_init, vkllm_op_matmul_run, vkllm_op_matmul_post_run},
        {vkllm_op_rope_init, vkllm_op_rope_run, vkllm_op_rope_post_run},
        {vkllm_op_softmax_init, vkllm_op_softmax_run, vkllm_op_softmax_post_run},
        {vkllm_op_ffn_up_and_gate_init, vkllm_op_ffn_up_and_gate_run, vkllm_op_ffn_up_and_gate_post_run},
        {vkllm_op_update_rows_init, vkllm_op_update_rows_run, vkllm_op_update_rows_post_run},
        {vkllm_op_arg_max_init, vkllm_op_arg_max_run, vkllm_op_arg_max_post_run},
        {nullptr, nullptr, nullptr}, // REF
    };
    if ((int)op < 0 || op >= VKLLM_OP_COUNTS)
        return nullptr;
    return &table[op];
}

enum Phase
{
    PH_INIT,
    PH_RUN,
    PH_POST
};

// Post-order DFS from `t` (sources first), visiting each node once, iteratively so that deep
// graphs (7B: ~650 nodes chained through 32 blocks) cannot exhaust the stack.
vkllm_err_t visit(vkllm_context *ctx, vkllm_commands *cmd, vkllm_tensor *root, Phase ph)
{
    std::unordered_set<vkllm_tensor *> visited;
    struct Frame
    {
        vkllm_tensor *t;
        int next_src;
    };
    std::vector<Frame> stack;
    stack.push_back({root, 0});
    while (!stack.empty())
    {
        Frame &f = stack.back();
        if (f.next_src == 0 && visited.count(f.t))
        {
            stack.pop_back();
            continue;
        }
        if (f.next_src < VKLLM_MAX_SRCS)
        {
            vkllm_tensor *s = f.t->srcs[f.next_src++];
            if (s && !visited.count(s))
                stack.push_back({s, 0});
            continue;
        }
        vkllm_tensor *t = f.t;
        stack.pop_back();
        if (visited.count(t))
            continue;
        visited.insert(t);
        const OpEntry *e = op_entry(t->op);
        if (!e)
        {
            log_error("Unknown operation type: %d", (int)t->op);
            return VKLLM_ERR_ARGS;
        }
        op_fn fn = ph == PH_INIT ? e->init : (ph == PH_RUN ? e->run : e->post_run);
        if (!fn)
            continue; // NONE / REF
        vkllm_err_t err = fn(ctx, cmd, t);
        if (err != VKLLM_ERR_OK)
        {
            log_error("%s of node %s (%s) failed: %s", ph == PH_INIT ? "init" : (ph == PH_RUN ? "run" : "post_run"),
                      t->name, vkllm_op_s(t->op), vkllm_err_s(err));
            return err;
        }
    }
    return VKLLM_ERR_OK;
}

bool fused_applies(vkllm_context *ctx, vkllm_graph *g)
{
    return g->b200_plan && ctx->runtime->exec_mode == VKLLM_EXEC_FUSED;
}

} // namespace

extern "C" vkllm_err_t vkllm_graph_new(struct vkllm_context *context, struct vkllm_graph **graph)
{
    _CHECK_ARGS(context && graph);
    vkllm_graph *p = (vkllm_graph *)calloc(1, sizeof(vkllm_graph));
    if (!p)
        return VKLLM_ERR_ALLOC;
    vkllm_err_t err = vkllm_array_tensor_new(&p->input_nodes, 8);
    if (err == VKLLM_ERR_OK)
        err = vkllm_array_tensor_new(&p->nodes, 128);
    if (err == VKLLM_ERR_OK)
        err = vkllm_commands_new(context, &p->commands);
    if (err != VKLLM_ERR_OK)
    {
        vkllm_array_tensor_free(p->nodes);
        vkllm_array_tensor_free(p->input_nodes);
        free(p);
        return err;
    }
    *graph = p;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_graph_add_input(struct vkllm_context *context, struct vkllm_graph *graph,
                                             struct vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && graph && tensor);
    _CHECK(vkllm_array_tensor_append(graph->input_nodes, tensor));
    _CHECK(vkllm_graph_add_node(context, graph, tensor));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_graph_add_node(struct vkllm_context *context, struct vkllm_graph *graph,
                                            struct vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && graph && tensor);
    return vkllm_array_tensor_append(graph->nodes, tensor);
}

extern "C" vkllm_err_t vkllm_graph_set_output(struct vkllm_context *context, struct vkllm_graph *graph,
                                              struct vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && graph && tensor);
    graph->output_node = tensor;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_graph_init(struct vkllm_context *context, struct vkllm_graph *graph)
{
    _CHECK_ARGS(context && graph && graph->output_node && graph->commands);
    if (fused_applies(context, graph))
    {
        // The fused step needs no per-node kernels; only the output node is initialised (its
        // pipeline is reported non-NULL as after a reference init).
        return op_entry(graph->output_node->op)->init(context, graph->commands, graph->output_node);
    }
    return visit(context, graph->commands, graph->output_node, PH_INIT);
}

extern "C" vkllm_err_t vkllm_graph_run(struct vkllm_context *context, struct vkllm_graph *graph)
{
    _CHECK_ARGS(context && graph && graph->output_node && graph->commands);
    if (fused_applies(context, graph))
    {
        vkllm_err_t e = vkb::plan_run(context, graph);
        if (e != VKLLM_ERR_ARGS)
            return e;
        // Plan not applicable (e.g. the caller edited the graph): fall through to node-by-node.
        _CHECK(visit(context, graph->commands, graph->output_node, PH_INIT));
    }
    _CHECK(vkllm_commands_begin(context, graph->commands));
    vkllm_err_t err = visit(context, graph->commands, graph->output_node, PH_RUN);
    _CHECK(vkllm_commands_end(context, graph->commands));
    _CHECK(vkllm_commands_submit(context, graph->commands));
    _CHECK(vkllm_commands_wait_exec(context, graph->commands));
    if (err == VKLLM_ERR_OK)
    {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess)
            return vkb::cuda_check(e, "graph kernels", __FILE__, __LINE__);
    }
    return err;
}

extern "C" vkllm_err_t vkllm_graph_post_run(struct vkllm_context *context, struct vkllm_graph *graph)
{
    _CHECK_ARGS(context && graph && graph->output_node && graph->commands);
    if (fused_applies(context, graph))
        return VKLLM_ERR_OK;
    return visit(context, graph->commands, graph->output_node, PH_POST);
}

extern "C" vkllm_err_t vkllm_graph_free(struct vkllm_context *context, struct vkllm_graph *graph)
{
    _CHECK_ARGS(context && graph);
    vkllm_commands_free(context, graph->commands);
    const size_t n = vkb::graph_cache_give(context, graph) ? 1 : graph->nodes->used_n;
    for (size_t i = 0; i < n; i++)
        vkllm_tensor_free(context, graph->nodes->data[i]);
    vkllm_array_tensor_free(graph->nodes);
    vkllm_array_tensor_free(graph->input_nodes);
    vkb::plan_free(context, graph);
    free(graph);
    return VKLLM_ERR_OK;
}
