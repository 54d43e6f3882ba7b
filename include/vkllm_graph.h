/* Tensor-DAG executor (reference: src/core/vkllm_graph.h:11-29, src/core/vkllm_graph.c).
 *
 * Same lifecycle as the reference: new -> add_input/add_node/set_output -> init -> run -> post_run
 * -> free, and vkllm_graph_free frees every node that was added. `run` enqueues the DAG reachable
 * from output_node in post-order on graph->commands' stream, then submits and waits, so outputs
 * (mapped tensors) are readable when it returns.
 *
 * Graphs built by vkllm_models_llama2_build_graph additionally carry a fused-execution plan: unless
 * the environment sets VKLLM_B200_STRICT=1, `run` then executes the fused LLaMA-2 step (CUDA Graph
 * replay for decode steps) instead of one kernel per node. Only the graph's output (and the KV
 * cache) are materialised in that mode; intermediate node buffers are left unallocated.
 */
#ifndef VKLLM_GRAPH_H
#define VKLLM_GRAPH_H

#include "vkllm_array.h"

#ifdef __cplusplus
extern "C" {
#endif

struct vkllm_tensor;
struct vkllm_context;
struct vkllm_commands;

VKLLM_DEF_ARRAY(tensor, struct vkllm_tensor *)

struct vkllm_graph
{
    struct vkllm_array_tensor *nodes;
    struct vkllm_array_tensor *input_nodes;
    struct vkllm_tensor *output_node;
    struct vkllm_commands *commands;
    void *b200_plan; /* fused-execution plan attached by vkllm_models_llama2_build_graph (NULL otherwise) */
};

extern vkllm_err_t vkllm_graph_new(struct vkllm_context *context, struct vkllm_graph **graph);
extern vkllm_err_t vkllm_graph_add_input(struct vkllm_context *context, struct vkllm_graph *graph,
                                         struct vkllm_tensor *tensor);
extern vkllm_err_t vkllm_graph_set_output(struct vkllm_context *context, struct vkllm_graph *graph,
                                          struct vkllm_tensor *tensor);
extern vkllm_err_t vkllm_graph_add_node(struct vkllm_context *context, struct vkllm_graph *graph,
                                        struct vkllm_tensor *tensor);
extern vkllm_err_t vkllm_graph_init(struct vkllm_context *context, struct vkllm_graph *graph);
extern vkllm_err_t vkllm_graph_run(struct vkllm_context *context, struct vkllm_graph *graph);
extern vkllm_err_t vkllm_graph_post_run(struct vkllm_context *context, struct vkllm_graph *graph);
extern vkllm_err_t vkllm_graph_free(struct vkllm_context *context, struct vkllm_graph *graph);

#ifdef __cplusplus
}
#endif
#endif
