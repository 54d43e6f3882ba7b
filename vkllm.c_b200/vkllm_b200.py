"""ctypes binding of libvkllm_b200.so, the C-ABI library that replaces vkllm.c's LLaMA-2 path.

The functions keep the reference's C names and argument meaning (include/*.h); this module only
declares their signatures, mirrors the public structs (checked against the library's own layout
queries) and adds small conveniences used by the tests and bench.py. Everything that computes
runs inside the library on the GPU; a missing library raises at import-use time.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("VKLLM_B200_LIB_PATH") or os.path.join(HERE, "lib", "libvkllm_b200.so")

OK, ALLOC, VULKAN, DEV_NOT_FOUND, PIPELINE_NOT_FOUND, ARGS = 1, 2, 3, 4, 5, 6
F32, F16, I8, U32 = 1, 2, 3, 4
(OP_NONE, OP_COPY, OP_BIN, OP_EMBEDDING, OP_RMSNORM, OP_MATMUL, OP_ROPE, OP_SOFTMAX, OP_FFN_UP_AND_GATE,
 OP_UPDATE_ROWS, OP_ARG_MAX, OP_REF) = range(12)
EXEC_FUSED, EXEC_STRICT = 0, 1
NP_DTYPE = {F32: np.float32, F16: np.float16, U32: np.uint32, I8: np.int8}


class VkllmError(RuntimeError):
    def __init__(self, err, what):
        super().__init__(f"{what} failed: {err_s(err)} ({err})")
        self.err = err


class TensorData(C.Structure):
    _fields_ = [("dev", C.c_void_p), ("host", C.c_void_p), ("mapped", C.c_bool), ("is_ref", C.c_bool),
                ("capacity", C.c_uint64)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("dtype", C.c_int), ("shapes", C.c_uint32 * 4),
                ("strides", C.c_uint32 * 4), ("bytes", C.c_uint32), ("device", C.c_void_p), ("data", TensorData),
                ("state_flags", C.c_uint32), ("op", C.c_int), ("pipeline", C.c_void_p),
                ("srcs", C.c_void_p * 4)]  # followed by the flexible params[] block


class Array(C.Structure):
    _fields_ = [("alloc_n", C.c_size_t), ("used_n", C.c_size_t), ("data", C.c_void_p)]


class Graph(C.Structure):
    _fields_ = [("nodes", C.POINTER(Array)), ("input_nodes", C.POINTER(Array)), ("output_node", C.POINTER(Tensor)),
                ("commands", C.c_void_p), ("b200_plan", C.c_void_p)]


class Meta(C.Structure):
    _fields_ = [("block_count", C.c_uint32), ("context_length", C.c_uint32), ("embedding_length", C.c_uint32),
                ("rope_freq_base", C.c_float), ("layer_norm_rms_epsilon", C.c_float), ("key_length", C.c_uint32),
                ("value_length", C.c_uint32), ("vocab_size", C.c_uint32), ("head_count", C.c_uint32),
                ("head_count_kv", C.c_uint32), ("bos_token_id", C.c_uint32), ("eos_token_id", C.c_uint32),
                ("padding_token_id", C.c_uint32), ("add_bos_token", C.c_bool), ("add_eos_token", C.c_bool),
                ("tokens", C.c_void_p)]


class Weights(C.Structure):
    _fields_ = [("tok_embed_weights", C.POINTER(Tensor)), ("blocks", C.POINTER(Array)),
                ("output_norm_weight", C.POINTER(Tensor)), ("output_weight", C.POINTER(Tensor)),
                ("kvcache", C.c_void_p)]


class B200Part(C.Structure):
    _fields_ = [("engine", C.c_void_p), ("tp_rank", C.c_uint32), ("tp_size", C.c_uint32), ("tp_comm", C.c_void_p)]


class Llama2(C.Structure):
    _fields_ = [("meta", Meta), ("weights", Weights), ("b200", B200Part)]


class BlockWeights(C.Structure):
    _fields_ = [(n, C.POINTER(Tensor)) for n in
                ("attn_norm_weight", "ffn_norm_weight", "WQ", "WK", "WV", "WO", "WU", "WG", "WD")]


class KVCache(C.Structure):
    _fields_ = [("kcaches", C.POINTER(Array)), ("vcaches", C.POINTER(Array)), ("kcache_shape", C.c_uint32 * 4),
                ("vcache_shape", C.c_uint32 * 4), ("layer_counts", C.c_uint32)]


class Llama2Config(C.Structure):
    _fields_ = [("block_count", C.c_uint32), ("context_length", C.c_uint32), ("embedding_length", C.c_uint32),
                ("head_count", C.c_uint32), ("ffn_length", C.c_uint32), ("vocab_size", C.c_uint32),
                ("rope_freq_base", C.c_float), ("rms_eps", C.c_float), ("init_std", C.c_float)]


class TokenIdArray(C.Structure):
    _fields_ = [("alloc_n", C.c_size_t), ("used_n", C.c_size_t), ("data", C.POINTER(C.c_uint32))]


PT = C.POINTER(Tensor)
_lib = None

# name -> (restype, argtypes)
_SIGS = {
    "vkllm_err_s": (C.c_char_p, [C.c_int]),
    "vkllm_dtype_s": (C.c_char_p, [C.c_int]),
    "vkllm_op_s": (C.c_char_p, [C.c_int]),
    "vkllm_get_dtype_info": (C.c_int, [C.c_int, C.c_void_p]),
    "vkllm_context_new": (C.c_int, [C.c_uint32, C.POINTER(C.c_void_p)]),
    "vkllm_context_free": (None, [C.c_void_p]),
    "vkllm_tensor_new": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32), C.c_int, C.c_int,
                                   C.POINTER(PT), C.c_uint32, C.c_void_p, C.c_size_t, C.c_bool, C.POINTER(PT)]),
    "vkllm_tensor_free": (None, [C.c_void_p, PT]),
    "vkllm_tensor_flush_cache": (C.c_int, [C.c_void_p, PT]),
    "vkllm_tensor_invalid_cache": (C.c_int, [C.c_void_p, PT]),
    "vkllm_tensor_new_staging": (C.c_int, [C.c_void_p, PT, C.POINTER(PT)]),
    "vkllm_tensor_reshape": (C.c_int, [C.c_void_p, PT, C.POINTER(C.c_uint32)]),
    "vkllm_tensor_permute": (C.c_int, [C.c_void_p, PT, C.POINTER(C.c_uint32)]),
    "vkllm_tensor_copy_ref": (C.c_int, [C.c_void_p, PT, C.POINTER(PT)]),
    "vkllm_tensor_slice0": (C.c_int, [C.c_void_p, PT, C.POINTER(C.c_uint32), C.POINTER(PT)]),
    "vkllm_tensor_s": (C.c_int, [C.c_void_p, PT, C.c_char_p, C.c_size_t]),
    "vkllm_commands_new": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "vkllm_commands_free": (None, [C.c_void_p, C.c_void_p]),
    "vkllm_commands_begin": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vkllm_commands_end": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vkllm_commands_upload": (C.c_int, [C.c_void_p, C.c_void_p, PT, C.c_void_p, C.c_size_t]),
    "vkllm_commands_download": (C.c_int, [C.c_void_p, C.c_void_p, PT, C.c_void_p, C.c_size_t]),
    "vkllm_commands_submit": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vkllm_commands_wait_exec": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vkllm_graph_new": (C.c_int, [C.c_void_p, C.POINTER(C.POINTER(Graph))]),
    "vkllm_graph_add_input": (C.c_int, [C.c_void_p, C.POINTER(Graph), PT]),
    "vkllm_graph_add_node": (C.c_int, [C.c_void_p, C.POINTER(Graph), PT]),
    "vkllm_graph_set_output": (C.c_int, [C.c_void_p, C.POINTER(Graph), PT]),
    "vkllm_graph_init": (C.c_int, [C.c_void_p, C.POINTER(Graph)]),
    "vkllm_graph_run": (C.c_int, [C.c_void_p, C.POINTER(Graph)]),
    "vkllm_graph_post_run": (C.c_int, [C.c_void_p, C.POINTER(Graph)]),
    "vkllm_graph_free": (C.c_int, [C.c_void_p, C.POINTER(Graph)]),
    "vkllm_pipeline_query_exec_time": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint64)]),
    "vkllm_models_llama2_load": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_char_p]),
    "vkllm_models_llama2_free": (C.c_int, [C.c_void_p, C.POINTER(Llama2)]),
    "vkllm_models_llama2_build_graph": (C.c_int, [C.c_void_p, C.POINTER(Llama2), PT, C.POINTER(Graph),
                                                  C.c_uint32]),
    "vkllm_models_llama2_tokenize": (C.c_int, [C.POINTER(Llama2), C.c_char_p,
                                               C.POINTER(C.POINTER(TokenIdArray))]),
    "vkllm_kvcache_new": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.c_uint32,
                                    C.POINTER(C.POINTER(KVCache))]),
    "vkllm_kvcache_update": (C.c_int, [C.c_void_p, C.POINTER(KVCache), C.POINTER(PT), C.POINTER(PT), C.c_uint32,
                                       C.c_uint32]),
    "vkllm_kvcache_free": (None, [C.c_void_p, C.POINTER(KVCache)]),
    "vkllm_hashmap_new": (C.c_int, [C.POINTER(C.c_void_p), C.c_size_t]),
    "vkllm_hashmap_free": (None, [C.c_void_p]),
    "vkllm_hashmap_insert": (C.c_int, [C.c_void_p, C.c_char_p, C.c_uint64]),
    "vkllm_hashmap_get": (C.c_bool, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint64)]),
    "vkllm_hashmap_remove": (C.c_int, [C.c_void_p, C.c_char_p]),
    "vkllm_hashmap_size": (C.c_size_t, [C.c_void_p]),
    "vkllm_b200_version": (C.c_char_p, []),
    "vkllm_b200_models_llama2_init_random": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.POINTER(Llama2Config),
                                                       C.c_uint64]),
    "vkllm_b200_random_f16_host": (None, [C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, C.c_uint64, C.c_void_p]),
    "vkllm_b200_set_exec_mode": (C.c_int, [C.c_void_p, C.c_int]),
    "vkllm_b200_set_graph_cache": (C.c_int, [C.c_void_p, C.c_int]),
    "vkllm_b200_get_exec_mode": (C.c_int, [C.c_void_p]),
    "vkllm_b200_context_stream": (C.c_void_p, [C.c_void_p]),
    "vkllm_b200_context_device": (C.c_int, [C.c_void_p]),
    "vkllm_b200_allocator_stats": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                             C.POINTER(C.c_uint64)]),
    "vkllm_b200_engine_prepare": (C.c_int, [C.c_void_p, C.POINTER(Llama2)]),
    "vkllm_b200_engine_set_state": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_uint32, C.c_uint32]),
    "vkllm_b200_engine_decode_steps": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_uint32]),
    "vkllm_b200_engine_read_tokens": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_engine_read_logits": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_engine_kernels_per_step": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2)]),
    "vkllm_b200_engine_last_launches": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2)]),
    "vkllm_b200_engine_is_persistent": (C.c_int, [C.c_void_p, C.POINTER(Llama2)]),
    "vkllm_b200_engine_read_trace": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_engine_read_warp_trace": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_engine_read_trace_last": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_engine_read_cta_trace": (C.c_uint32, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32]),
    "vkllm_b200_gemm_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                      C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_int, C.c_void_p]),
    "vkllm_b200_gemm_f16_error": (C.c_uint32, []),
    "vkllm_b200_token_loop": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                        C.c_void_p, C.POINTER(C.c_double)]),
    "vkllm_b200_batch_new": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_uint32, C.c_uint32, C.POINTER(C.c_void_p)]),
    "vkllm_b200_batch_load_sequence": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32]),
    "vkllm_b200_batch_decode_steps": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "vkllm_b200_batch_read_tokens": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32]),
    "vkllm_b200_batch_read_logits": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "vkllm_b200_batch_free": (None, [C.c_void_p, C.c_void_p]),
    "vkllm_b200_models_llama2_init_random_tp": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.POINTER(Llama2Config),
                                                          C.c_uint64, C.c_uint32, C.c_uint32]),
    "vkllm_b200_tp_init": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p]),
    "vkllm_b200_models_llama2_load_tp": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_char_p, C.c_uint32,
                                                   C.c_uint32]),
    "vkllm_b200_gguf_read_shard": (C.c_int, [C.c_char_p, C.c_char_p, C.c_uint32, C.c_uint32, C.c_void_p,
                                             C.c_uint64, C.c_void_p]),
    "vkllm_b200_tp_shard": (C.c_int, [C.c_uint32, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32, C.c_void_p]),
    "vkllm_b200_random_f16_host_shard": (None, [C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, C.c_uint32, C.c_uint32,
                                                C.c_uint32, C.c_uint32, C.c_void_p]),
    "vkllm_b200_tp_connect": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p]),
    "vkllm_b200_tp_nccl_unique_id": (C.c_int, [C.c_void_p]),
    "vkllm_b200_tp_nccl_connect": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_void_p]),
    "vkllm_b200_engine_bench_kernel": (C.c_int, [C.c_void_p, C.POINTER(Llama2), C.c_char_p, C.c_uint32,
                                                 C.POINTER(C.c_float), C.POINTER(C.c_uint64)]),
    "vkllm_b200_attention_decode_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                                      C.c_uint32, C.c_uint32, C.c_float, C.c_void_p, C.c_void_p]),
    "vkllm_b200_sizeof": (C.c_size_t, [C.c_char_p]),
    "vkllm_b200_offsetof": (C.c_size_t, [C.c_char_p, C.c_char_p]),
}

OPS = ["matmul", "rmsnorm", "rope", "softmax", "update_rows", "bin", "copy", "embedding", "arg_max", "ffn_up_and_gate"]
for _o in OPS:
    for _s in ("init", "run", "post_run"):
        _SIGS[f"vkllm_op_{_o}_{_s}"] = (C.c_int, [C.c_void_p, C.c_void_p, PT])

# Every symbol the binding declares (tests/test_abi.py checks each against include/*.h and the library).
EXPORTED = sorted(_SIGS)


def lib():
    """Loads the library once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `python vkllm.c_b200/build.py` (or __graft_entry__.build())")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name, None)
            if f is None:  # a library older than this binding: calling the entry point raises
                continue
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def err_s(e):
    return lib().vkllm_err_s(e).decode()


def check(e, what):
    if e != OK:
        raise VkllmError(e, what)


def u32x4(vals):
    return (C.c_uint32 * 4)(*vals)


class Context:
    """vkllm_context on CUDA device `dev` (vkllm_context_new / vkllm_context_free)."""

    def __init__(self, dev=0):
        self.ptr = C.c_void_p()
        check(lib().vkllm_context_new(dev, C.byref(self.ptr)), "vkllm_context_new")

    def close(self):
        if self.ptr:
            lib().vkllm_context_free(self.ptr)
            self.ptr = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self):
        return lib().vkllm_b200_context_stream(self.ptr)

    def set_exec_mode(self, mode):
        check(lib().vkllm_b200_set_exec_mode(self.ptr, mode), "vkllm_b200_set_exec_mode")

    def set_graph_cache(self, on):
        check(lib().vkllm_b200_set_graph_cache(self.ptr, int(bool(on))), "vkllm_b200_set_graph_cache")


def tensor_new(ctx, name, shape, dtype, op=OP_NONE, srcs=(), params=None, mapped=False):
    out = PT()
    arr = (PT * 4)(*srcs) if srcs else None
    if params is None:
        pbuf, pbytes = None, 0
    else:
        raw = bytes(params)
        pbuf, pbytes = C.create_string_buffer(raw, len(raw)), len(raw)
    check(lib().vkllm_tensor_new(ctx.ptr, name.encode(), u32x4(shape), dtype, op, arr, len(srcs), pbuf, pbytes,
                                 mapped, C.byref(out)), f"vkllm_tensor_new({name})")
    return out


def tensor_free(ctx, t):
    lib().vkllm_tensor_free(ctx.ptr, t)


def params_of(t, ctype):
    """View of a tensor's trailing params block as `ctype`."""
    addr = C.addressof(t.contents) + C.sizeof(Tensor)
    return ctype.from_address(addr)


def np_of(t, arr_dtype=None):
    dt = NP_DTYPE[t.contents.dtype] if arr_dtype is None else arr_dtype
    return dt


class Commands:
    def __init__(self, ctx):
        self.ctx = ctx
        self.ptr = C.c_void_p()
        check(lib().vkllm_commands_new(ctx.ptr, C.byref(self.ptr)), "vkllm_commands_new")

    def close(self):
        if self.ptr:
            lib().vkllm_commands_free(self.ctx.ptr, self.ptr)
            self.ptr = C.c_void_p()

    def begin(self):
        check(lib().vkllm_commands_begin(self.ctx.ptr, self.ptr), "begin")

    def end(self):
        check(lib().vkllm_commands_end(self.ctx.ptr, self.ptr), "end")

    def upload(self, t, arr):
        a = np.ascontiguousarray(arr)
        check(lib().vkllm_commands_upload(self.ctx.ptr, self.ptr, t, a.ctypes.data, a.nbytes), "upload")

    def download(self, t, nbytes, dtype):
        out = np.empty(nbytes // np.dtype(dtype).itemsize, dtype=dtype)
        check(lib().vkllm_commands_download(self.ctx.ptr, self.ptr, t, out.ctypes.data, out.nbytes), "download")
        return out

    def submit_wait(self):
        check(lib().vkllm_commands_submit(self.ctx.ptr, self.ptr), "submit")
        check(lib().vkllm_commands_wait_exec(self.ctx.ptr, self.ptr), "wait_exec")


def strided_from_dense(t, flat):
    """Scatters a dense [B,C,H,W] array into the byte-strided layout of tensor t (for uploads)."""
    tc = t.contents
    es = np.dtype(NP_DTYPE[tc.dtype]).itemsize
    total = tc.bytes // es
    buf = np.zeros(total, dtype=NP_DTYPE[tc.dtype])
    st = [s // es for s in tc.strides]
    view = np.lib.stride_tricks.as_strided(buf, shape=tuple(tc.shapes), strides=tuple(s * es for s in st))
    view[...] = flat.reshape(tuple(tc.shapes))
    return buf


def dense_from_strided(t, buf):
    tc = t.contents
    view = np.lib.stride_tricks.as_strided(buf, shape=tuple(tc.shapes), strides=tuple(tc.strides))  # byte strides
    return np.array(view)


def run_op(ctx, node, init_fn, run_fn):
    """Runs one op node like the reference op tests: begin, init, run, end, submit, wait."""
    cmd = Commands(ctx)
    try:
        cmd.begin()
        check(getattr(lib(), init_fn)(ctx.ptr, cmd.ptr, node), init_fn)
        check(getattr(lib(), run_fn)(ctx.ptr, cmd.ptr, node), run_fn)
        cmd.end()
        cmd.submit_wait()
    finally:
        cmd.close()


def upload_download_roundtrip(ctx, t, arr):
    cmd = Commands(ctx)
    try:
        cmd.begin()
        cmd.upload(t, arr)
        cmd.end()
        cmd.submit_wait()
    finally:
        cmd.close()


def fetch(ctx, t):
    """Downloads a (non-view or view) tensor's whole buffer and returns its dense [B,C,H,W] values."""
    tc = t.contents
    dt = NP_DTYPE[tc.dtype]
    cmd = Commands(ctx)
    try:
        cmd.begin()
        buf = cmd.download(t, tc.bytes, dt)
        cmd.end()
        cmd.submit_wait()
    finally:
        cmd.close()
    return dense_from_strided(t, buf)


def put(ctx, t, dense):
    """Uploads dense [B,C,H,W] values into tensor t's strided layout."""
    buf = strided_from_dense(t, np.asarray(dense, dtype=NP_DTYPE[t.contents.dtype]))
    cmd = Commands(ctx)
    try:
        cmd.begin()
        cmd.upload(t, buf)
        cmd.end()
        cmd.submit_wait()
    finally:
        cmd.close()


class Model:
    """struct vkllm_models_llama2 owned from Python."""

    def __init__(self, ctx):
        self.ctx = ctx
        self.m = Llama2()
        self.loaded = False

    def load(self, path):
        check(lib().vkllm_models_llama2_load(self.ctx.ptr, C.byref(self.m), path.encode()), "llama2_load")
        self.loaded = True
        return self

    def init_random(self, cfg: dict, seed: int):
        c = Llama2Config(**cfg)
        check(lib().vkllm_b200_models_llama2_init_random(self.ctx.ptr, C.byref(self.m), C.byref(c), seed),
              "llama2_init_random")
        self.loaded = True
        return self

    def init_random_tp(self, cfg: dict, seed: int, rank: int, world: int):
        """Tensor-parallel shard `rank` of `world` of the random model of init_random."""
        c = Llama2Config(**cfg)
        check(lib().vkllm_b200_models_llama2_init_random_tp(self.ctx.ptr, C.byref(self.m), C.byref(c), seed, rank,
                                                             world), "llama2_init_random_tp")
        self.loaded = True
        return self

    def load_tp(self, path, rank: int, world: int):
        """Tensor-parallel shard `rank` of `world` of a GGUF model (only the shard is uploaded)."""
        check(lib().vkllm_b200_models_llama2_load_tp(self.ctx.ptr, C.byref(self.m), path.encode(), rank, world),
              "llama2_load_tp")
        self.loaded = True
        return self

    def tp_connect(self, all_gather):
        """Sets up the peer-memory exchange: `all_gather(bytes) -> list of bytes` (rank order) is the
        caller's collective, e.g. torch.distributed.all_gather_object."""
        h = (C.c_char * 64)()
        check(lib().vkllm_b200_tp_init(self.ctx.ptr, C.byref(self.m), h), "tp_init")
        handles = all_gather(bytes(h))
        buf = (C.c_char * (64 * len(handles))).from_buffer_copy(b"".join(handles))
        check(lib().vkllm_b200_tp_connect(self.ctx.ptr, C.byref(self.m), buf), "tp_connect")

    def tp_connect_nccl(self, all_gather):
        """Sets up the NCCL exchange: rank 0's unique id reaches every rank through `all_gather(bytes)
        -> list of bytes` (the caller's collective); then the communicator is created (collective)."""
        uid = (C.c_char * 128)()
        if self.m.b200.tp_rank == 0:
            check(lib().vkllm_b200_tp_nccl_unique_id(uid), "tp_nccl_unique_id")
        got = all_gather(bytes(uid))
        root = (C.c_char * 128).from_buffer_copy(got[0])
        check(lib().vkllm_b200_tp_nccl_connect(self.ctx.ptr, C.byref(self.m), root), "tp_nccl_connect")

    def free(self):
        if self.loaded:
            check(lib().vkllm_models_llama2_free(self.ctx.ptr, C.byref(self.m)), "llama2_free")
            self.loaded = False

    @property
    def meta(self):
        return self.m.meta

    def block(self, i):
        arr = self.m.weights.blocks.contents
        ptrs = C.cast(arr.data, C.POINTER(C.POINTER(BlockWeights)))
        return ptrs[i].contents

    def step(self, tokens, offset, logits=None):
        """One reference-style token-loop iteration (tests/vkllm_test_infer_gguf.c:181-272): new mapped
        input tensor, new graph, build_graph, init, upload, run, post_run, read the last row of the
        mapped argmax output, free the graph. Returns the predicted token. When `logits` is a list,
        the fp16 logits of the last row are appended to it (read from the "logits" node when the
        graph ran node by node, from the fused engine otherwise)."""
        l = lib()
        toks = np.asarray(tokens, dtype=np.uint32)
        inp = tensor_new(self.ctx, "input_toks", (1, 1, 1, len(toks)), U32, mapped=True)
        g = C.POINTER(Graph)()
        check(l.vkllm_graph_new(self.ctx.ptr, C.byref(g)), "graph_new")
        try:
            check(l.vkllm_models_llama2_build_graph(self.ctx.ptr, C.byref(self.m), inp, g, offset), "build_graph")
            check(l.vkllm_graph_init(self.ctx.ptr, g), "graph_init")
            check(l.vkllm_commands_upload(self.ctx.ptr, g.contents.commands, inp, toks.ctypes.data, toks.nbytes),
                  "upload")
            check(l.vkllm_graph_run(self.ctx.ptr, g), "graph_run")
            check(l.vkllm_graph_post_run(self.ctx.ptr, g), "graph_post_run")
            out = g.contents.output_node
            check(l.vkllm_tensor_invalid_cache(self.ctx.ptr, out), "invalid_cache")
            oc = out.contents
            host = C.cast(oc.data.host, C.POINTER(C.c_uint32))
            st = [s // 4 for s in oc.strides]
            i = (oc.shapes[0] - 1) * st[0] + (oc.shapes[1] - 1) * st[1] + (oc.shapes[2] - 1) * st[2]
            if logits is not None:
                logits.append(self._last_logits(g))
            return int(host[i])
        finally:
            l.vkllm_graph_free(self.ctx.ptr, g)

    def _last_logits(self, g):
        nodes = g.contents.nodes.contents
        arr = C.cast(nodes.data, C.POINTER(PT))
        for i in range(nodes.used_n - 1, -1, -1):
            t = arr[i]
            if t.contents.name == b"logits":
                if t.contents.data.dev:
                    return fetch(self.ctx, t)[0, 0, -1].copy()
                break
        return self.engine_logits().copy()

    def token_loop(self, prompt, offset, n_tokens):
        """The reference token loop in native code (vkllm_b200_token_loop): returns the n_tokens
        predictions and the host microseconds spent outside vkllm_graph_run."""
        p = np.asarray(prompt, dtype=np.uint32)
        out = np.zeros(n_tokens, dtype=np.uint32)
        host = C.c_double(0.0)
        check(lib().vkllm_b200_token_loop(self.ctx.ptr, C.byref(self.m), p.ctypes.data, len(p), offset, n_tokens,
                                          out.ctypes.data, C.byref(host)), "token_loop")
        return [int(t) for t in out], host.value

    def generate(self, prompt, n_tokens, logits=None):
        """Greedy loop: prefill with `prompt`, then feed each prediction back; n_tokens predictions."""
        out, toks, offset = [], list(prompt), 0
        for _ in range(n_tokens):
            t = self.step(toks, offset, logits)
            offset += len(toks)
            out.append(t)
            toks = [t]
        return out

    # fused engine helpers
    def engine_prepare(self):
        check(lib().vkllm_b200_engine_prepare(self.ctx.ptr, C.byref(self.m)), "engine_prepare")

    def engine_logits(self):
        v = self.m.meta.vocab_size
        out = np.empty(v, dtype=np.uint16)
        check(lib().vkllm_b200_engine_read_logits(self.ctx.ptr, C.byref(self.m), out.ctypes.data, v), "read_logits")
        return out.view(np.float16)


def random_f16_host(seed, tensor_id, std, first, n):
    out = np.empty(n, dtype=np.uint16)
    lib().vkllm_b200_random_f16_host(seed, tensor_id, std, first, n, out.ctypes.data)
    return out


class Batch:
    """Batched greedy decode of independent sequences on one model (vkllm_b200_batch_*)."""

    def __init__(self, model, n_seqs, kv_rows):
        self.model, self.ctx, self.n = model, model.ctx, n_seqs
        self.ptr = C.c_void_p()
        check(lib().vkllm_b200_batch_new(self.ctx.ptr, C.byref(model.m), n_seqs, kv_rows, C.byref(self.ptr)),
              "batch_new")

    def add_prompt(self, seq, prompt):
        """Prefills `prompt` through the drop-in graph API (the model's KV cache) and moves its KV rows
        into slot `seq`. Returns the prefill's predicted token (the slot's next input)."""
        first = self.model.step(list(prompt), 0)
        check(lib().vkllm_b200_batch_load_sequence(self.ctx.ptr, self.ptr, seq, first, len(prompt)), "load_sequence")
        return first

    def decode(self, n_steps):
        check(lib().vkllm_b200_batch_decode_steps(self.ctx.ptr, self.ptr, n_steps), "batch_decode_steps")
        out = np.zeros((n_steps, self.n), dtype=np.uint32)
        check(lib().vkllm_b200_batch_read_tokens(self.ctx.ptr, self.ptr, out.ctypes.data, n_steps), "read_tokens")
        return out

    def logits(self):
        V = self.model.meta.vocab_size
        out = np.zeros((self.n, V), dtype=np.uint16)
        check(lib().vkllm_b200_batch_read_logits(self.ctx.ptr, self.ptr, out.ctypes.data), "read_logits")
        return out.view(np.float16)

    def free(self):
        if self.ptr:
            lib().vkllm_b200_batch_free(self.ctx.ptr, self.ptr)
            self.ptr = C.c_void_p()
