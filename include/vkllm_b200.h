/* B200-specific additions to the vkllm C API. None of these has a counterpart in the reference;
 * they expose what the CUDA backend adds (device-side random init for benchmarks, execution-mode
 * control, the fused decode engine's device-resident loop, tensor parallelism) without changing
 * any reference signature. */
#ifndef VKLLM_B200_H
#define VKLLM_B200_H

#include <stddef.h>
#include <stdint.h>

#include "vkllm_errors.h"

#ifdef __cplusplus
extern "C" {
#endif

struct vkllm_context;
struct vkllm_models_llama2;

/* Library version string. */
extern const char *vkllm_b200_version(void);

/* ---- model construction without a GGUF file ------------------------------------------------ */

struct vkllm_b200_llama2_config
{
    uint32_t block_count;
    uint32_t context_length;
    uint32_t embedding_length;
    uint32_t head_count;
    uint32_t ffn_length; /* SwiGLU hidden size */
    uint32_t vocab_size;
    float rope_freq_base; /* <= 0: 10000 */
    float rms_eps;        /* <= 0: 1e-5 */
    float init_std;       /* <= 0: 0.02 */
};

/* Fills `model` with the tensors vkllm_models_llama2_load would create for a GGUF of this shape
 * (same names, shapes, dtypes), generated on the device: fp16 weights from a counter-based
 * generator (Irwin-Hall sum of 12 uniforms, scaled to init_std; element i of the t-th tensor in
 * GGUF order depends only on (seed, t, i)), f32 norm gains of 1. Used where writing a multi-GB
 * GGUF is impractical (7B/13B benchmarks). */
extern vkllm_err_t vkllm_b200_models_llama2_init_random(struct vkllm_context *context,
                                                        struct vkllm_models_llama2 *model,
                                                        const struct vkllm_b200_llama2_config *cfg, uint64_t seed);

/* Tensor-parallel shard `tp_rank` of `tp_size` (<= 8) of the same random model: Wq, Wk, Wv, Wgate,
 * Wup and the output matrix keep rows [r n/N, (r+1) n/N), Wo and Wdown keep the matching columns
 * (attention heads and FFN columns sharded), the embedding and the
 * norm gains stay whole, and the KV cache holds head_count / tp_size heads. Every shard element has
 * the bits of the same element of the unsharded model. head_count, ffn_length and vocab_size must
 * be multiples of tp_size. Such a model decodes only through the engine entry points
 * (vkllm_b200_engine_*) after vkllm_b200_tp_connect. */
extern vkllm_err_t vkllm_b200_models_llama2_init_random_tp(struct vkllm_context *context,
                                                           struct vkllm_models_llama2 *model,
                                                           const struct vkllm_b200_llama2_config *cfg, uint64_t seed,
                                                           uint32_t tp_rank, uint32_t tp_size);

/* Tensor-parallel shard `tp_rank` of `tp_size` (<= 8) of a GGUF model, read at load time: each rank
 * uploads only its shard of every matrix, with the layout of vkllm_b200_models_llama2_init_random_tp
 * (rows of Wq, Wk, Wv, Wgate, Wup and output; columns of Wo and Wdown; the embedding and the norm
 * gains whole). Metadata and the tokenizer vocabulary are read as vkllm_models_llama2_load
 * (src/models/vkllm_models_llama2.c:67-187) reads them. head_count, vocab_size and the FFN length
 * must be multiples of tp_size (VKLLM_ERR_ARGS otherwise). tp_size 1 is vkllm_models_llama2_load. */
extern vkllm_err_t vkllm_b200_models_llama2_load_tp(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                    const char *file, uint32_t tp_rank, uint32_t tp_size);

/* Host only (no device): the shard of tensor `tensor` of a GGUF file that rank tp_rank of tp_size
 * holds under the layout above, written row-major to dst (dst_bytes at least rows x cols x element
 * size); shape receives {rows, cols}. dst NULL: shape only. */
extern vkllm_err_t vkllm_b200_gguf_read_shard(const char *file, const char *tensor, uint32_t tp_rank,
                                              uint32_t tp_size, void *dst, uint64_t dst_bytes, uint32_t *shape);

/* Tensor parallelism over peer memory (one process per GPU, every rank with its shard from
 * vkllm_b200_models_llama2_init_random_tp or vkllm_b200_models_llama2_load_tp). Each rank calls
 * vkllm_b200_tp_init, which allocates its exchange buffer and writes its 64-byte CUDA IPC handle to
 * handle_out; the caller gathers the
 * handles of all ranks (rank order, 64 bytes each, e.g. with torch.distributed.all_gather_object)
 * and passes them to vkllm_b200_tp_connect, which maps the peers' buffers. Then the engine entry
 * points decode on every rank in lockstep: the Wo and down projections of each layer exchange
 * their partial sums inside the decode kernel (NVLink stores + release flags, bounded waits), and
 * the argmax of the vocabulary shards is combined with the reference tie rule. Every rank must make
 * the same engine calls in the same order. Call both before the first decode. */
extern vkllm_err_t vkllm_b200_tp_init(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                      void *handle_out);
extern vkllm_err_t vkllm_b200_tp_connect(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                         const void *handles);

/* NCCL exchange of a tensor-parallel model (the baseline the peer-memory exchange is measured
 * against): the decode step runs the per-op kernels on the shards, with an ncclAllReduce (sum, fp32)
 * of the Wo and down partial rows after each projection and an ncclAllGather of the argmax class
 * candidates, all captured in one CUDA graph per step. One rank calls vkllm_b200_tp_nccl_unique_id
 * (128 bytes); the caller hands those bytes to every rank, and every rank then calls
 * vkllm_b200_tp_nccl_connect (collective over the ranks; before the first engine call).
 * libnccl.so.2 is loaded at the first call (VKLLM_ERR_VULKAN when it cannot be). With only this
 * exchange connected the engine uses it; with both, VKLLM_B200_TP_EXCHANGE=nccl at engine creation
 * selects it (default: the peer-memory exchange). */
extern vkllm_err_t vkllm_b200_tp_nccl_unique_id(void *id_out);
extern vkllm_err_t vkllm_b200_tp_nccl_connect(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                              const void *id);

/* The shard of a rows x cols matrix held by tensor-parallel rank tp_rank of tp_size: split 1 = rows
 * (Wq, Wk, Wv, Wgate, Wup, output), 2 = columns (Wo, Wdown), 0 = whole (embedding). out = {row0, rows,
 * col0, cols} of the shard in the unsharded matrix. Host only. */
extern vkllm_err_t vkllm_b200_tp_shard(uint32_t rows, uint32_t cols, int split, uint32_t tp_rank, uint32_t tp_size,
                                       uint32_t *out);
/* Host twin of a shard of the device generator: element (i, c) is element (row0 + i) * full_cols +
 * col0 + c of tensor `tensor_id` (what init_random_tp writes on the device). */
extern void vkllm_b200_random_f16_host_shard(uint64_t seed, uint64_t tensor_id, float std_dev, uint64_t full_cols,
                                             uint32_t row0, uint32_t rows, uint32_t col0, uint32_t cols, uint16_t *out);

/* Host-side twin of the device generator: the fp16 bit patterns of elements [first, first + n) of
 * tensor `tensor_id` (for CPU references of randomly initialised models). */
extern void vkllm_b200_random_f16_host(uint64_t seed, uint64_t tensor_id, float std_dev, uint64_t first, uint64_t n,
                                       uint16_t *out);

/* ---- execution control ---------------------------------------------------------------------- */

enum
{
    VKLLM_B200_EXEC_FUSED = 0,  /* llama2 graphs run the fused engine (default) */
    VKLLM_B200_EXEC_STRICT = 1, /* every graph runs one kernel per node, like the reference */
};
extern vkllm_err_t vkllm_b200_set_exec_mode(struct vkllm_context *context, int mode);
extern int vkllm_b200_get_exec_mode(struct vkllm_context *context);

/* Structural graph cache (on by default; VKLLM_B200_GRAPH_CACHE=0 at context creation turns it off).
 * vkllm_graph_free hands the nodes of a graph built by vkllm_models_llama2_build_graph to the
 * context, and the next build for the same model, batch and token count takes them back, rewriting
 * only the fields that follow the position (RoPE and softmax offsets, KV-slice rows, score columns).
 * The graph the caller sees is the one a fresh build makes; node buffers stay attached between
 * tokens. A caller that edits a built graph's nodes in place before freeing it turns the cache off.
 * Turning it off (on = 0) frees the cached nodes; a model's entries go with vkllm_models_llama2_free,
 * and all entries with a change of execution mode. */
extern vkllm_err_t vkllm_b200_set_graph_cache(struct vkllm_context *context, int on);

/* The context's CUDA stream (cudaStream_t); all graph work is enqueued on it. */
extern void *vkllm_b200_context_stream(struct vkllm_context *context);
extern int vkllm_b200_context_device(struct vkllm_context *context);
extern vkllm_err_t vkllm_b200_allocator_stats(struct vkllm_context *context, uint64_t *dev_in_use,
                                              uint64_t *dev_cached, uint64_t *host_in_use);

/* ---- fused decode engine: device-resident token loop ------------------------------------------
 * The engine keeps a device "step state" (current token, position). One decode step reads it,
 * runs the whole model for that token, writes the greedy next token back into it, appends the
 * token to a device ring of generated tokens and advances the position, so steps can be enqueued
 * back to back with no host round trip. */

/* Builds the engine for `model` (workspace, kernel parameters, CUDA Graph of one decode step). */
extern vkllm_err_t vkllm_b200_engine_prepare(struct vkllm_context *context, struct vkllm_models_llama2 *model);
/* Enqueues: state.token = token, state.pos = pos, ring cleared. */
extern vkllm_err_t vkllm_b200_engine_set_state(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                               uint32_t token, uint32_t pos);
/* Enqueues n decode steps (CUDA Graph launches) on the context stream. */
extern vkllm_err_t vkllm_b200_engine_decode_steps(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                  uint32_t n);
/* Waits for the stream, then copies the first n generated tokens since set_state. */
extern vkllm_err_t vkllm_b200_engine_read_tokens(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                 uint32_t *out, uint32_t n);
/* Waits for the stream, then copies the fp16 logits of the last step ([vocab] halves). */
extern vkllm_err_t vkllm_b200_engine_read_logits(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                 uint16_t *out, uint32_t n);
/* Kernel launches per decode step of the engine's current mode: the persistent cooperative
 * kernel (one launch runs up to 64 steps) reports 1; the CUDA-Graph fallback (environment
 * VKLLM_B200_DECODE=graph, or devices without cooperative launch) 2 + 6 * layers. */
extern uint32_t vkllm_b200_engine_kernels_per_step(struct vkllm_context *context, struct vkllm_models_llama2 *model);
/* Kernel launches enqueued by the last vkllm_b200_engine_decode_steps call. */
extern uint32_t vkllm_b200_engine_last_launches(struct vkllm_context *context, struct vkllm_models_llama2 *model);
/* Tracing: with the environment variable VKLLM_B200_TRACE=1 set when the engine is built, the
 * persistent kernel's CTA 0 records %globaltimer (ns) at its start and at every grid barrier
 * arrival and release. Copies up to `cap` entries of the last launch; returns the count copied
 * (0 when tracing is off). Per step the barriers are, per layer: after QKV, scores, probs.V, Wo,
 * up/gate, down; then after the logits and after the argmax. A single mark (no pair) follows each
 * GEMV phase's input staging (before QKV, Wo, up/gate, down and logits). */
extern uint32_t vkllm_b200_engine_read_trace(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                             uint64_t *out, uint32_t cap);
/* Tracing: for each grid barrier of the last persistent launch, %globaltimer (ns) when the last
 * CTA arrived, stored at the index of the barrier's release entry in vkllm_b200_engine_read_trace's
 * layout (other entries undefined). Returns the count copied, 0 when tracing is off. */
extern uint32_t vkllm_b200_engine_read_trace_last(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                  uint64_t *out, uint32_t cap);
/* Tracing: %globaltimer (ns) of every CTA's arrival at each of the first 1023 grid barriers of the
 * last persistent launch, out[barrier * grid + cta] with grid = the SM count; row 1023 holds each
 * CTA's %smid. Returns the count copied, 0 when tracing is off. */
extern uint32_t vkllm_b200_engine_read_cta_trace(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                 uint64_t *out, uint32_t cap);
/* Tracing: CTA 0's per-warp weight-pipeline accounting, in SM cycles, summed over every persistent
 * launch since the engine was built: out[(warp * 5 + kind) * 4 + {0: mbarrier wait, 1: consume
 * (compute + refill issue), 2: chunks, 3: compute}], kind 0..4 = QKV, Wo, up/gate, down, logits.
 * With cap >= 648, out[640..647] adds CTA 0's attention sub-steps in SM cycles: 0 q load, 1 key
 * scores, 2 split statistics, 3 wait for the sibling splits, 4 head statistics, 5 probs . V, 6 the
 * combine of the splits, 7 attention items. Needs cap >= 640; returns 640 or 648, or 0 when tracing
 * is off. */
extern uint32_t vkllm_b200_engine_read_warp_trace(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                  uint64_t *out, uint32_t cap);
/* Tensor-core GEMM (tcgen05 + TMEM, TMA-fed): C = act(scale * A . B^T) for fp16 A [M, K] (row
 * stride lda elements), B [N, K] (row stride ldb), C [M, N] (row stride ldc), fp32 accumulation,
 * act 1 = SiLU. Device pointers, 16-byte aligned; K, lda and ldb multiples of 8. Enqueued on
 * `stream` (a cudaStream_t, NULL = default stream). Returns VKLLM_ERR_ARGS when the shape or the
 * alignment does not fit, VKLLM_ERR_VULKAN on a launch error. It is the kernel behind
 * VKLLM_OP_MATMUL (src/core/vkllm_op_matmul.c:212-315) for fp16 operands with M > 1 and B [N, K]. */
extern vkllm_err_t vkllm_b200_gemm_f16(const void *A, const void *B, void *C, uint32_t M, uint32_t N, uint32_t K,
                                       uint64_t lda, uint64_t ldb, uint64_t ldc, float scale, int act, void *stream);
/* Sticky error word of the tensor-core GEMM on the current device: 0, or bit 0 when one of its
 * bounded waits expired (the results of that launch are not valid). */
extern uint32_t vkllm_b200_gemm_f16_error(void);

/* The reference's token loop (tests/vkllm_test_infer_gguf.c:181-272) as one call, through the public
 * entry points: for each of n_tokens iterations, a mapped u32 input tensor, vkllm_graph_new,
 * vkllm_models_llama2_build_graph at `offset`, vkllm_graph_init, vkllm_commands_upload of the ids,
 * vkllm_graph_run, vkllm_graph_post_run, the last row of the mapped argmax output and
 * vkllm_graph_free. The first iteration feeds the n_prompt ids of `prompt` (the prefill), each later
 * one the previous prediction; out_tokens[i] receives iteration i's prediction. When host_us is not
 * NULL it receives the host time spent outside vkllm_graph_run (microseconds, all iterations). */
extern vkllm_err_t vkllm_b200_token_loop(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                         const uint32_t *prompt, uint32_t n_prompt, uint32_t offset,
                                         uint32_t n_tokens, uint32_t *out_tokens, double *host_us);

/* Batched greedy decode of independent sequences sharing the model's weights (no reference
 * counterpart; the reference decodes one sequence per graph). Each sequence has its own KV cache of
 * `kv_rows` rows per layer and head inside the batch. A step of all sequences runs the reference
 * graph's nodes with S = 1 per sequence: projections as tensor-core GEMMs with M = n_seqs, RoPE /
 * KV rows / attention / argmax per sequence, fp16 at every node.
 *   vkllm_b200_batch_new            allocates the caches and activations (zeroed).
 *   vkllm_b200_batch_load_sequence  copies rows [0, n_rows) of the model's own KV cache (written by a
 *                                   prefill through vkllm_graph_run) into slot `seq`, whose next input
 *                                   token is `next_token` at position n_rows.
 *   vkllm_b200_batch_decode_steps   n greedy steps of every sequence (n <= 1024); VKLLM_ERR_ARGS if a
 *                                   sequence would pass its KV capacity.
 *   vkllm_b200_batch_read_tokens    tokens of the last decode call, [step][seq].
 *   vkllm_b200_batch_read_logits    fp16 logits of the last step, [seq][vocab]. */
struct vkllm_b200_batch;
extern vkllm_err_t vkllm_b200_batch_new(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                        uint32_t n_seqs, uint32_t kv_rows, struct vkllm_b200_batch **out);
extern vkllm_err_t vkllm_b200_batch_load_sequence(struct vkllm_context *context, struct vkllm_b200_batch *batch,
                                                  uint32_t seq, uint32_t next_token, uint32_t n_rows);
extern vkllm_err_t vkllm_b200_batch_decode_steps(struct vkllm_context *context, struct vkllm_b200_batch *batch,
                                                 uint32_t n_steps);
extern vkllm_err_t vkllm_b200_batch_read_tokens(struct vkllm_context *context, struct vkllm_b200_batch *batch,
                                                uint32_t *out, uint32_t n_steps);
extern vkllm_err_t vkllm_b200_batch_read_logits(struct vkllm_context *context, struct vkllm_b200_batch *batch,
                                                uint16_t *out);
extern void vkllm_b200_batch_free(struct vkllm_context *context, struct vkllm_b200_batch *batch);

/* 1 when the engine runs the persistent decode kernel. */
extern int vkllm_b200_engine_is_persistent(struct vkllm_context *context, struct vkllm_models_llama2 *model);

/* Times `iters` launches of one decode kernel of the engine ("qkv", "wo", "upgate", "down", "logits")
 * on the context stream with CUDA events, cycling through the layers so every launch streams its
 * own weights. Returns the mean microseconds per launch and the algorithmic bytes per launch
 * (weights + activations read and written). Clobbers the engine's step state. */
extern vkllm_err_t vkllm_b200_engine_bench_kernel(struct vkllm_context *context, struct vkllm_models_llama2 *model,
                                                  const char *kernel, uint32_t iters, float *us_per_launch,
                                                  uint64_t *bytes_per_launch);

/* Decode attention for one token that allocates nothing. No counterpart in the reference (whose
 * attention is three graph nodes: scores MATMUL, SOFTMAX, probs.V MATMUL); this computes the same
 * result as those nodes for S = 1, in fp16 with fp32 arithmetic, for callers that cannot call
 * cudaMalloc (inside stream capture, under a fixed memory budget, on real-time paths).
 *   q       fp16 [heads, head_dim], the rotated query of the token
 *   kcache  fp16 [heads, cache_rows, head_dim], vcache likewise; keys/values 0 .. n_keys-1 are used
 *   out     fp16 [heads, head_dim]
 *   scale   score scale (1/sqrt(head_dim) for LLaMA-2); stream is a cudaStream_t (NULL = legacy)
 * kcache and vcache must be 8-byte aligned (rows are read 4 halves at a time), q and out 2-byte
 * aligned; other pointers return VKLLM_ERR_ARGS without launching anything.
 * When n_keys == head_dim the result is the reference graph's, not textbook attention: its MATMUL
 * decides "B is transposed" from shapes alone (src/core/vkllm_op_matmul.c:14-30), so at that one key
 * count the probs.V node computes out[w] = sum_k p_k * V[w][k]. This entry point reproduces that.
 * All scratch lives in one static device array of about 1.1 MiB that every GPU loading the library
 * holds until exit. Limits: heads <= 64, head_dim <= 256 and a multiple of 4,
 * heads * cache_rows <= 262144; larger sizes return VKLLM_ERR_ARGS. The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress, with that device current) and should
 * come before any stream capture; the device that is current at each call must be the one that owns
 * `stream` and the buffers. The looked-up address is kept for the life of the process, so calls
 * after a cudaDeviceReset of that device are not supported. The kernels contain no waits: a fault
 * shows up as a CUDA error at the caller's next synchronisation of `stream`. Every call shares the
 * array: calls that overlap on the GPU (two streams, or two host threads) race on it and must be
 * serialised by the caller. */
extern vkllm_err_t vkllm_b200_attention_decode_noalloc(const void *q, const void *kcache, const void *vcache,
                                                       uint32_t heads, uint32_t head_dim, uint32_t cache_rows,
                                                       uint32_t n_keys, float scale, void *out, void *stream);

/* ---- struct layout queries (for FFI bindings that mirror the public structs) --------------- */
extern size_t vkllm_b200_sizeof(const char *struct_name);
extern size_t vkllm_b200_offsetof(const char *struct_name, const char *field);

#ifdef __cplusplus
}
#endif
#endif
