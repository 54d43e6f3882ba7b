"""TEST INFRASTRUCTURE ONLY: Python binding of the parity oracle (oracle/vkllm_oracle.cpp).

A CPU restatement of the reference vkllm.c shader math (see the C++ header comment for the
reference file:line each function follows). Used by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker; the product never imports it.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
_lib = None

F32, F16, U32 = 1, 2, 4
_CODE = {np.dtype(np.float32): F32, np.dtype(np.float16): F16, np.dtype(np.uint32): U32}


class _View(C.Structure):
    _fields_ = [("dtype", C.c_int), ("shape", C.c_uint32 * 4), ("stride", C.c_uint32 * 4), ("data", C.c_void_p)]


class _Cfg(C.Structure):
    _fields_ = [("D", C.c_uint32), ("H", C.c_uint32), ("F", C.c_uint32), ("V", C.c_uint32), ("L", C.c_uint32),
                ("ctx", C.c_uint32), ("unk", C.c_uint32), ("eps", C.c_float), ("rope_base", C.c_float)]


def build():
    """Compiles liboracle.so with the committed Makefile (a few seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        try:
            l = C.CDLL(LIB_PATH)
        except OSError:
            build()
            l = C.CDLL(LIB_PATH)
        V = C.POINTER(_View)
        sig = {
            "oracle_threads": (C.c_int, [C.c_int]),
            "oracle_set_arith": (C.c_int, [C.c_int]),
            "oracle_op_matmul": (C.c_int, [V, V, V, C.c_float, C.c_int]),
            "oracle_op_rmsnorm": (C.c_int, [V, C.c_void_p, V, C.c_float]),
            "oracle_op_rope": (C.c_int, [V, V, C.c_uint32, C.c_float, C.c_int]),
            "oracle_op_softmax": (C.c_int, [V, V, C.c_int, C.c_uint32]),
            "oracle_op_update_rows": (C.c_int, [V, V, C.c_uint32, C.c_int]),
            "oracle_op_copy": (C.c_int, [V, V, C.c_int]),
            "oracle_op_bin": (C.c_int, [V, V, V, C.c_int]),
            "oracle_op_embedding": (C.c_int, [V, V, V, C.c_uint32, C.c_int]),
            "oracle_op_arg_max": (C.c_int, [V, C.c_void_p, C.POINTER(C.c_uint32)]),
            "oracle_op_ffn_up_gate": (C.c_int, [V, V, V, V]),
            "oracle_round16": (None, [C.c_void_p, C.c_void_p, C.c_uint64]),
            "oracle_f32_to_f16": (None, [C.c_void_p, C.c_void_p, C.c_uint64]),
            "oracle_f16_to_f32": (None, [C.c_void_p, C.c_void_p, C.c_uint64]),
            "oracle_random_f16": (None, [C.c_uint64, C.c_uint64, C.c_float, C.c_uint64, C.c_uint64, C.c_void_p]),
            "oracle_llama2_new": (C.c_void_p, [C.POINTER(_Cfg), C.c_void_p, C.c_void_p, C.c_void_p,
                                               C.POINTER(C.c_void_p)]),
            "oracle_llama2_free": (None, [C.c_void_p]),
            "oracle_llama2_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p,
                                             C.c_void_p]),
        }
        for n, (r, a) in sig.items():
            f = getattr(l, n)
            f.restype, f.argtypes = r, a
        _lib = l
    return _lib


def threads(n=0):
    return lib().oracle_threads(n)


def set_arith(mode):
    """"fp32" (default): the f16f32 shader variants, the parity target. "fp16": the variants a device
    with shaderFloat16 selects (fp16 GEMV accumulation, fp16 dot pairs in the GEMM, fp16 softmax and
    RoPE). Returns the previous mode."""
    return "fp16" if lib().oracle_set_arith(1 if mode == "fp16" else 0) else "fp32"


def _view(arr):
    """A [B,C,H,W] numpy array (possibly a strided view) as an oracle view."""
    assert arr.ndim == 4
    it = arr.dtype.itemsize
    v = _View()
    v.dtype = _CODE[arr.dtype]
    for i in range(4):
        v.shape[i] = arr.shape[i]
        v.stride[i] = arr.strides[i] // it
    v.data = arr.ctypes.data
    return v


def matmul(a, b, out_shape, scale=1.0, act=0):
    out = np.zeros(out_shape, dtype=a.dtype)
    lib().oracle_op_matmul(C.byref(_view(a)), C.byref(_view(b)), C.byref(_view(out)), scale, act)
    return out


def rmsnorm(x, g, eps):
    y = np.zeros(x.shape, dtype=np.float16)
    g = np.ascontiguousarray(g, dtype=np.float32)
    lib().oracle_op_rmsnorm(C.byref(_view(x)), g.ctypes.data, C.byref(_view(y)), eps)
    return y


def rope(x, offset, base, neox=False):
    y = np.zeros(x.shape, dtype=x.dtype)
    lib().oracle_op_rope(C.byref(_view(x)), C.byref(_view(y)), offset, base, int(neox))
    return y


def softmax(x, seq_mask, offsets):
    x = np.ascontiguousarray(x)
    y = np.zeros(x.shape, dtype=x.dtype)
    lib().oracle_op_softmax(C.byref(_view(x)), C.byref(_view(y)), seq_mask, offsets)
    return y


def update_rows(src, cache, offset_rows):
    out = np.array(cache, copy=True)
    lib().oracle_op_update_rows(C.byref(_view(src)), C.byref(_view(out)), offset_rows, src.dtype.itemsize)
    return out


def copy(x):
    y = np.zeros(x.shape, dtype=x.dtype)
    lib().oracle_op_copy(C.byref(_view(x)), C.byref(_view(y)), x.dtype.itemsize)
    return y


def bin_op(a, b, op, out_dtype):
    out = np.zeros(a.shape, dtype=out_dtype)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    lib().oracle_op_bin(C.byref(_view(a)), C.byref(_view(b)), C.byref(_view(out)), op)
    return out


def embedding(ids, table, out_shape, unk):
    out = np.zeros(out_shape, dtype=table.dtype)
    lib().oracle_op_embedding(C.byref(_view(ids)), C.byref(_view(table)), C.byref(_view(out)), unk,
                              table.dtype.itemsize)
    return out


def arg_max(x):
    out = np.zeros(x.shape[:3] + (1,), dtype=np.uint32)
    st = (C.c_uint32 * 4)(*[s // 4 for s in out.strides])
    lib().oracle_op_arg_max(C.byref(_view(x)), out.ctypes.data, st)
    return out


def ffn_up_gate(x, wu, wg, out_dtype):
    out = np.zeros(x.shape[:3] + (wu.shape[2],), dtype=out_dtype)
    lib().oracle_op_ffn_up_gate(C.byref(_view(x)), C.byref(_view(wu)), C.byref(_view(wg)), C.byref(_view(out)))
    return out


def round16(x):
    """One fp16 rounding of each fp32 value, as the fp16 arithmetic mode applies it after every op."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_round16(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f32_to_f16_bits(x):
    """The oracle's software fp32 -> fp16 conversion (storage rounding), as raw bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16(x.ctypes.data, out.ctypes.data, x.size)
    return out


def random_f16(seed, tensor_id, std, first, n):
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_random_f16(seed, tensor_id, std, first, n, out.ctypes.data)
    return out.view(np.float16)


class Llama2:
    """The reference LLaMA-2 token step on the CPU. `weights` maps GGUF tensor names to numpy arrays
    (fp16 matrices as [rows, cols], f32 norm gains as [n]); they must stay alive with this object."""

    def __init__(self, cfg, weights, ctx=None):
        self.cfg = cfg
        self.w = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        c = _Cfg(D=cfg["D"], H=cfg["H"], F=cfg["F"], V=cfg["V"], L=cfg["L"], ctx=ctx or cfg["ctx"],
                 unk=cfg.get("unk", 0), eps=cfg["eps"], rope_base=cfg["rope_base"])
        names = []
        for l in range(cfg["L"]):
            names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight", f"blk.{l}.attn_q.weight",
                      f"blk.{l}.attn_k.weight", f"blk.{l}.attn_v.weight", f"blk.{l}.attn_output.weight",
                      f"blk.{l}.ffn_gate.weight", f"blk.{l}.ffn_up.weight", f"blk.{l}.ffn_down.weight"]
        ptrs = (C.c_void_p * len(names))(*[self.w[n].ctypes.data for n in names])
        self.h = lib().oracle_llama2_new(C.byref(c), self.w["token_embd.weight"].ctypes.data,
                                         self.w["output_norm.weight"].ctypes.data,
                                         self.w["output.weight"].ctypes.data, ptrs)

    def step(self, tokens, offset):
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        S = len(toks)
        logits = np.zeros((S, self.cfg["V"]), dtype=np.float16)
        out = np.zeros(S, dtype=np.uint32)
        r = lib().oracle_llama2_step(self.h, toks.ctypes.data, S, offset, logits.ctypes.data, out.ctypes.data)
        if r != 0:
            raise RuntimeError("oracle step past the context")
        return logits, out

    def generate(self, prompt, n_tokens):
        """Returns (tokens, last-row logits per step) of the reference greedy loop."""
        toks, offset, out, lg = list(prompt), 0, [], []
        for _ in range(n_tokens):
            logits, am = self.step(toks, offset)
            offset += len(toks)
            out.append(int(am[-1]))
            lg.append(logits[-1].copy())
            toks = [out[-1]]
        return out, lg

    def close(self):
        if self.h:
            lib().oracle_llama2_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
