// LLaMA-2 block builders: append the reference's node sequence
// (src/models/vkllm_llama2_layers.c:13-354) to a graph. Node names, ops, shapes and parameter
// blocks are the reference's, so the op-by-op executor computes the reference's rounding points.
#include <cmath>
#include <cstdio>
#include <cstring>

#include "../runtime/internal.h"
#include "vkllm_kvcache.h"
#include "vkllm_llama2_layers.h"
#include "vkllm_op_matmul.h"
#include "vkllm_op_rmsnorm.h"
#include "vkllm_op_softmax.h"

namespace
{

// buf = a + b, truncated to the buffer (node names are built per token, so no printf formatting).
void join(char *buf, size_t cap, const char *a, const char *b)
{
    size_t la = strnlen(a, cap - 1), lb = strnlen(b, cap - 1 - la);
    memcpy(buf, a, la);
    memcpy(buf + la, b, lb);
    buf[la + lb] = 0;
}

// Creates a node and appends it to the graph; frees it again if the append fails.
vkllm_err_t add(vkllm_context *ctx, vkllm_graph *g, const char *name, const uint32_t *shapes, vkllm_dtype_t dt,
                vkllm_op_t op, vkllm_tensor **srcs, uint32_t n, const void *params, size_t pbytes, bool mapped,
                vkllm_tensor **out)
{
    _CHECK(vkllm_tensor_new(ctx, name, shapes, dt, op, srcs, n, params, pbytes, mapped, out));
    vkllm_err_t e = vkllm_graph_add_node(ctx, g, *out);
    if (e != VKLLM_ERR_OK)
    {
        vkllm_tensor_free(ctx, *out);
        *out = nullptr;
    }
    return e;
}

// copy_ref + reshape + add to graph (+ optional permute), as the reference does for Q/K/V heads.
vkllm_err_t view(vkllm_context *ctx, vkllm_graph *g, vkllm_tensor *src, const uint32_t *shape, const uint32_t *perm,
                 vkllm_tensor **out)
{
    _CHECK(vkllm_tensor_copy_ref(ctx, src, out));
    vkllm_err_t e = VKLLM_ERR_OK;
    if (shape)
        e = vkllm_tensor_reshape(ctx, *out, shape);
    if (e == VKLLM_ERR_OK)
        e = vkllm_graph_add_node(ctx, g, *out);
    if (e != VKLLM_ERR_OK)
    {
        vkllm_tensor_free(ctx, *out);
        *out = nullptr;
        return e;
    }
    if (perm)
        e = vkllm_tensor_permute(ctx, *out, perm);
    return e;
}

} // namespace

extern "C" vkllm_err_t vkllm_llama2_build_ffn_layer(struct vkllm_context *context, struct vkllm_graph *graph,
                                                    struct vkllm_tensor *input,
                                                    struct vkllm_llama2_ffn_layer_params params, uint32_t block_idx)
{
    _CHECK_ARGS(context && graph && input && params.WD && params.WG && params.WU);
    char name[64], buf[128];
    snprintf(name, sizeof(name), "block.%u.ffn", block_idx);
    uint32_t B = input->shapes[0], C = input->shapes[1], S = input->shapes[2], F = params.WU->shapes[2];

    vkllm_tensor *norm, *up, *gate, *mul, *down, *out;
    vkllm_tensor *norm_srcs[] = {input, params.norm_weight};
    vkllm_op_rmsnorm_params np = {params.norm_power, params.norm_eps};
    join(buf, sizeof(buf), name, ".norm");
    _CHECK(add(context, graph, buf, input->shapes, input->dtype, VKLLM_OP_RMSNORM, norm_srcs, 2, &np, sizeof(np),
               false, &norm));

    uint32_t up_shape[4] = {B, C, S, F};
    vkllm_tensor *up_srcs[] = {norm, params.WU};
    vkllm_op_matmul_params up_p = {1.0f, 0};
    join(buf, sizeof(buf), name, ".up");
    _CHECK(add(context, graph, buf, up_shape, norm->dtype, VKLLM_OP_MATMUL, up_srcs, 2, &up_p, sizeof(up_p), false,
               &up));

    vkllm_tensor *gate_srcs[] = {norm, params.WG};
    vkllm_op_matmul_params gate_p = {1.0f, 1};
    join(buf, sizeof(buf), name, ".gate");
    _CHECK(add(context, graph, buf, up_shape, norm->dtype, VKLLM_OP_MATMUL, gate_srcs, 2, &gate_p, sizeof(gate_p),
               false, &gate));

    vkllm_tensor *mul_srcs[] = {up, gate};
    int32_t mul_op = 2;
    join(buf, sizeof(buf), name, ".mul");
    _CHECK(add(context, graph, buf, up_shape, gate->dtype, VKLLM_OP_BIN, mul_srcs, 2, &mul_op, sizeof(mul_op), false,
               &mul));

    uint32_t down_shape[4] = {B, C, S, params.WD->shapes[2]};
    vkllm_tensor *down_srcs[] = {mul, params.WD};
    vkllm_op_matmul_params down_p = {1.0f, 0};
    join(buf, sizeof(buf), name, ".down");
    _CHECK(add(context, graph, buf, down_shape, mul->dtype, VKLLM_OP_MATMUL, down_srcs, 2, &down_p, sizeof(down_p),
               false, &down));

    vkllm_tensor *add_srcs[] = {input, down};
    int32_t add_op = 0;
    join(buf, sizeof(buf), name, ".add");
    _CHECK(add(context, graph, buf, input->shapes, input->dtype, VKLLM_OP_BIN, add_srcs, 2, &add_op, sizeof(add_op),
               false, &out));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_llama2_build_self_attn_layer(struct vkllm_context *context, struct vkllm_graph *graph,
                                                          struct vkllm_kvcache *kvcache, struct vkllm_tensor *input,
                                                          struct vkllm_llama2_self_attn_layer_params params,
                                                          uint32_t block_idx)
{
    _CHECK_ARGS(context && graph && input && params.WQ && params.WK && params.WV && params.WO && kvcache);
    _CHECK_ARGS(params.num_head > 0);
    vkllm_op_rope_params rope_p;
    memset(&rope_p, 0, sizeof(rope_p));
    rope_p.offset = params.offsets;
    rope_p.base = params.freq_base;
    rope_p.neox_style = false;

    uint32_t hidden = params.WQ->shapes[3];
    uint32_t HD = params.WQ->shapes[2];
    uint32_t hd = HD / params.num_head;
    _CHECK_ARGS(hd * params.num_head == HD);
    _CHECK_ARGS(params.WK->shapes[0] == 1 && params.WK->shapes[1] == 1);
    _CHECK_ARGS(params.WV->shapes[0] == 1 && params.WV->shapes[1] == 1);
    _CHECK_ARGS(params.WK->shapes[2] == HD && params.WK->shapes[3] == hidden);
    _CHECK_ARGS(params.WV->shapes[2] == HD && params.WV->shapes[3] == hidden);
    _CHECK_ARGS(input->shapes[3] == hidden);
    uint32_t B = input->shapes[0], S = input->shapes[2], H = params.num_head;

    char name[64], buf[128];
    snprintf(name, sizeof(name), "block.%u.attn", block_idx);

    vkllm_tensor *norm, *Q, *K, *V;
    vkllm_tensor *norm_srcs[] = {input, params.norm_weight};
    vkllm_op_rmsnorm_params np = {params.norm_power, params.norm_eps};
    join(buf, sizeof(buf), name, ".norm");
    _CHECK(add(context, graph, buf, input->shapes, input->dtype, VKLLM_OP_RMSNORM, norm_srcs, 2, &np, sizeof(np),
               false, &norm));

    uint32_t qkv_shape[4] = {B, 1, S, HD};
    vkllm_op_matmul_params mp = {1.0f, 0};
    vkllm_tensor *q_srcs[] = {norm, params.WQ};
    join(buf, sizeof(buf), name, ".Q");
    _CHECK(add(context, graph, buf, qkv_shape, norm->dtype, VKLLM_OP_MATMUL, q_srcs, 2, &mp, sizeof(mp), false, &Q));
    vkllm_tensor *k_srcs[] = {norm, params.WK};
    join(buf, sizeof(buf), name, ".K");
    _CHECK(add(context, graph, buf, qkv_shape, norm->dtype, VKLLM_OP_MATMUL, k_srcs, 2, &mp, sizeof(mp), false, &K));
    vkllm_tensor *v_srcs[] = {norm, params.WV};
    join(buf, sizeof(buf), name, ".V");
    _CHECK(add(context, graph, buf, qkv_shape, norm->dtype, VKLLM_OP_MATMUL, v_srcs, 2, &mp, sizeof(mp), false, &V));

    // [B,1,S,H*hd] -> [B,S,H,hd] -> permute(0,2,1,3) -> [B,H,S,hd] views.
    uint32_t heads_shape[4] = {B, S, H, hd};
    uint32_t perm[4] = {0, 2, 1, 3};
    vkllm_tensor *Qr, *Kr, *Vr;
    _CHECK(view(context, graph, Q, heads_shape, perm, &Qr));
    _CHECK(view(context, graph, K, heads_shape, perm, &Kr));
    _CHECK(view(context, graph, V, heads_shape, perm, &Vr));

    vkllm_tensor *RQ, *RK;
    join(buf, sizeof(buf), name, ".RQ");
    _CHECK(add(context, graph, buf, Qr->shapes, Qr->dtype, VKLLM_OP_ROPE, &Qr, 1, &rope_p, sizeof(rope_p), false,
               &RQ));
    join(buf, sizeof(buf), name, ".RK");
    _CHECK(add(context, graph, buf, Kr->shapes, Kr->dtype, VKLLM_OP_ROPE, &Kr, 1, &rope_p, sizeof(rope_p), false,
               &RK));

    // RK / Vr become slice0 views [B,H,offsets+S,hd] of this layer's cache. The reference never
    // frees these two views; here they are appended to the graph so vkllm_graph_free releases them.
    vkllm_tensor *Vs = Vr;
    _CHECK(vkllm_kvcache_update(context, kvcache, &RK, &Vs, block_idx, params.offsets));
    _CHECK(vkllm_graph_add_node(context, graph, RK));
    _CHECK(vkllm_graph_add_node(context, graph, Vs));

    uint32_t Lk = RK->shapes[2];
    uint32_t scores_shape[4] = {B, H, S, Lk};
    vkllm_tensor *scores, *probs, *attn;
    vkllm_tensor *s_srcs[] = {RQ, RK};
    vkllm_op_matmul_params sp = {1.0f / sqrtf((float)hd), 0};
    join(buf, sizeof(buf), name, ".scores");
    _CHECK(add(context, graph, buf, scores_shape, input->dtype, VKLLM_OP_MATMUL, s_srcs, 2, &sp, sizeof(sp), false,
               &scores));

    vkllm_op_softmax_params smp = {1, params.offsets};
    join(buf, sizeof(buf), name, ".attn_weights");
    _CHECK(add(context, graph, buf, scores_shape, input->dtype, VKLLM_OP_SOFTMAX, &scores, 1, &smp, sizeof(smp),
               false, &probs));

    uint32_t out_shape[4] = {B, H, S, hd};
    vkllm_tensor *o_srcs[] = {probs, Vs};
    vkllm_op_matmul_params op1 = {1.0f, 0};
    // The reference names this node with the block prefix only ("block.N.attn").
    _CHECK(add(context, graph, name, out_shape, input->dtype, VKLLM_OP_MATMUL, o_srcs, 2, &op1, sizeof(op1), false,
               &attn));

    // [B,H,S,hd] -> permute -> [B,S,H,hd] -> COPY (materialise) -> reshape [B,1,S,H*hd].
    vkllm_tensor *attn_ref, *concat, *concat_ref;
    _CHECK(view(context, graph, attn, nullptr, perm, &attn_ref));
    join(buf, sizeof(buf), name, ".concated_heads");
    _CHECK(add(context, graph, buf, attn_ref->shapes, attn_ref->dtype, VKLLM_OP_COPY, &attn_ref, 1, NULL, 0, false,
               &concat));
    uint32_t concat_shape[4] = {B, 1, S, HD};
    _CHECK(view(context, graph, concat, concat_shape, nullptr, &concat_ref));

    uint32_t final_shape[4] = {B, 1, S, hidden};
    vkllm_tensor *f_srcs[] = {concat_ref, params.WO};
    vkllm_tensor *final_out, *final_add;
    join(buf, sizeof(buf), name, ".final_output");
    _CHECK(add(context, graph, buf, final_shape, concat->dtype, VKLLM_OP_MATMUL, f_srcs, 2, &op1, sizeof(op1), false,
               &final_out));
    vkllm_tensor *a_srcs[] = {input, final_out};
    int32_t add_op = 0;
    join(buf, sizeof(buf), name, ".final_output_add");
    _CHECK(add(context, graph, buf, final_out->shapes, final_out->dtype, VKLLM_OP_BIN, a_srcs, 2, &add_op,
               sizeof(add_op), false, &final_add));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_llama2_build_transformer_block(struct vkllm_context *context, struct vkllm_graph *graph,
                                                            struct vkllm_kvcache *kvcache, struct vkllm_tensor *input,
                                                            struct vkllm_llama2_transformer_block_params params,
                                                            uint32_t block_idx)
{
    _CHECK_ARGS(context && graph && input);
    _CHECK(vkllm_llama2_build_self_attn_layer(context, graph, kvcache, input, params.attn, block_idx));
    vkllm_tensor *attn_out = graph->nodes->data[graph->nodes->used_n - 1];
    _CHECK(vkllm_llama2_build_ffn_layer(context, graph, attn_out, params.ffn, block_idx));
    return VKLLM_ERR_OK;
}
