"""Generates tests/golden/ref_ops.npz: seeded inputs and the outputs of the reference's OWN test-side
CPU reference functions, compiled from the reference checkout where they lie.

vkllm.c stores no golden vectors: each op test in its tests/ directory draws random inputs and
compares the Vulkan result with an in-file CPU function. oracle/refpin/Makefile compiles those
test files unchanged (with stub headers for the Vulkan/VMA/log.c/libcheck names they mention) into
oracle/_ref/librefpin.so, exporting these functions; this script calls them through ctypes:

  refpin_matmul       matmul_op_host       tests/vkllm_test_op_matmul.c:33-165
  refpin_rmsnorm      rmsnorm_op_host      tests/vkllm_test_op_rmsnorm.c:14-106
  refpin_rope         rope_op_host         tests/vkllm_test_op_rope.c:17-94
  refpin_softmax      softmax_op_host      tests/vkllm_test_op_softmax.c:14-119
  refpin_arg_max      arg_max_op_host      tests/vkllm_test_op_arg_max.c:12-71
  refpin_update_rows  update_rows_op_host  tests/vkllm_test_op_update_rows.c:75-122
  refpin_embedding    embedding_op_host    tests/vkllm_test_op_embedding.c:32-94
  refpin_copy         copy_op_host         tests/vkllm_test_op_copy.c:16-68
  refpin_bin          bin_op_host          tests/vkllm_test_op_bin.c:24-114
  refpin_fp32_to_fp16 vkllm_fp32_to_fp16   src/core/vkllm_common.h:157-186 (truncating)

Every fp16 output is therefore rounded the way the reference's tests round it. One key is not
from reference code: `am_out_shader`, the shader's argmax tie rule (src/shaders/vkllm_arg_max.comp:
54-90), restated below because no CPU function of the reference implements it (its test uses the
first maximum, and the two differ on ties: quirk Q8).

Inputs come from numpy.random.default_rng with fixed seeds (the reference's tests use unseeded
rand()). Run where the reference checkout exists, after `make -C oracle/refpin REF=<checkout>`:

    python tests/golden/make_golden.py            # rewrites ref_ops.npz next to this file
    python tests/golden/make_golden.py --check    # regenerates in memory, compares with the file
"""
import argparse
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REFPIN = os.path.join(ROOT, "oracle", "_ref", "librefpin.so")
OUT = os.path.join(HERE, "ref_ops.npz")

F32, F16, U32 = 1, 2, 4  # vkllm_dtype_t: src/core/vkllm_dtypes.inc:5-8

U4 = C.c_uint32 * 4


def refpin():
    if not os.path.exists(REFPIN):
        raise FileNotFoundError(f"{REFPIN} missing: run make -C oracle/refpin REF=<reference checkout>")
    lib = C.CDLL(REFPIN)
    lib.refpin_fp32_to_fp16.restype = C.c_uint16
    lib.refpin_fp32_to_fp16.argtypes = [C.c_float]
    lib.refpin_rope.argtypes = [C.c_void_p, C.c_void_p, U4, U4, U4, U4, C.c_uint32, C.c_float, C.c_int]
    return lib


def _u4(v):
    return U4(*[int(x) for x in v])


def _bstrides(a):
    """Byte strides of a 4-D numpy array (the reference passes strides in bytes)."""
    return _u4(a.strides)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _dt(a):
    return {np.dtype(np.float16): F16, np.dtype(np.float32): F32, np.dtype(np.uint32): U32}[a.dtype]


def ref_matmul(lib, a, b, transposed_b, act):
    B, Cc = max(a.shape[0], b.shape[0]), max(a.shape[1], b.shape[1])
    M, K = a.shape[2], a.shape[3]
    N = b.shape[2] if transposed_b else b.shape[3]
    out = np.zeros((B, Cc, M, N), dtype=a.dtype)
    lib.refpin_matmul(_p(a), _p(b), _p(out), a.shape[0], a.shape[1], b.shape[0], b.shape[1], M, K, N,
                      _bstrides(a), _bstrides(b), _bstrides(out), _dt(a), int(transposed_b), int(act))
    return out


def ref_rmsnorm(lib, x, g):
    """The reference test's eps is fixed at 1e-6 (tests/vkllm_test_op_rmsnorm.c:36)."""
    out = np.zeros_like(x)
    g4 = g.reshape(1, 1, 1, -1)
    lib.refpin_rmsnorm(_p(x), _p(g4), _p(out), _u4(x.shape), _bstrides(x), _bstrides(g4), _dt(x), _dt(g4),
                       _dt(out))
    return out


def ref_rope(lib, x, offset, base):
    """x may be a strided view; the output is contiguous of the same shape."""
    out = np.zeros(x.shape, dtype=x.dtype)
    # The reference function reads through the view's byte strides from the view's base pointer.
    lib.refpin_rope(x.__array_interface__["data"][0], _p(out), _u4(x.shape), _bstrides(x), _u4(out.shape),
                    _bstrides(out), offset, base, _dt(x))
    return out


def ref_softmax(lib, x, seq_mask, offsets):
    out = np.zeros_like(x)
    lib.refpin_softmax(_p(x), _p(out), _u4(x.shape), _bstrides(x), _dt(x), C.c_int32(seq_mask),
                       C.c_uint32(offsets))
    return out


def ref_arg_max(lib, x):
    out = np.zeros(x.shape[:3] + (1,), dtype=np.uint32)
    lib.refpin_arg_max(_p(x), _p(out), _u4(x.shape), _bstrides(x), _u4(out.shape), _bstrides(out), _dt(x))
    return out


def ref_update_rows(lib, src, cache, off):
    out = cache.copy()
    lib.refpin_update_rows(_p(src), _p(out), _u4(src.shape), _bstrides(src), _u4(out.shape), _bstrides(out), off,
                           _dt(src))
    return out


def ref_embedding(lib, ids, table):
    """Out-of-range ids map to row 0 in the test's function (tests/vkllm_test_op_embedding.c:58-61)."""
    out = np.zeros((1, 1, ids.shape[3], table.shape[3]), dtype=table.dtype)
    lib.refpin_embedding(ids.ctypes.data_as(C.POINTER(C.c_uint32)), _p(table), _p(out), _u4(ids.shape),
                         _u4(table.shape), _u4(out.shape), _bstrides(ids), _bstrides(table), _bstrides(out),
                         _dt(table))
    return out


def ref_copy(lib, x):
    """x may be a strided view; the output is contiguous of the same shape."""
    out = np.zeros(x.shape, dtype=x.dtype)
    lib.refpin_copy(x.__array_interface__["data"][0], _p(out), _u4(x.shape), _bstrides(x), _bstrides(out), _dt(x))
    return out


def ref_bin(lib, a, b, op):
    out = np.zeros(a.shape, dtype=a.dtype)
    lib.refpin_bin(_p(a), _p(b), _p(out), _u4(a.shape), _bstrides(a), _bstrides(b), _bstrides(out), _dt(a), _dt(b),
                   _dt(out), C.c_int32(op))
    return out


def ref_arg_max_shader(x):
    """src/shaders/vkllm_arg_max.comp:54-90: lane l scans w = l, l+32, ... keeping the first strict
    maximum (an empty lane keeps -FLT_MAX and its own index), then a 16/8/4/2/1 tree keeps the left
    operand unless the right one is strictly greater. It differs from the test's first maximum only
    on ties (quirk Q8)."""
    xf = x.astype(np.float32)
    B, Cc, H, W = x.shape
    out = np.zeros((B, Cc, H, 1), dtype=np.uint32)
    fmax = np.float32(np.finfo(np.float32).max)
    for b in range(B):
        for c in range(Cc):
            for h in range(H):
                vals = [(-fmax, l) if l >= W else (xf[b, c, h, l], l) for l in range(32)]
                for l in range(32):
                    for i in range(l + 32, W, 32):
                        if xf[b, c, h, i] > vals[l][0]:
                            vals[l] = (xf[b, c, h, i], i)
                step = 16
                while step > 0:
                    for l in range(step):
                        if vals[l + step][0] > vals[l][0]:
                            vals[l] = vals[l + step]
                    step //= 2
                out[b, c, h, 0] = vals[0][1]
    return out


def f16(rng, shape, lo=-1.0, hi=1.0):
    return rng.uniform(lo, hi, size=shape).astype(np.float32).astype(np.float16)


def generate(lib):
    rng = np.random.default_rng(20240611)
    g = {}
    # matmul families of tests/vkllm_test_op_matmul.c:166-286 at reduced sizes
    mm = [("gemv", (1, 1), (1, 1), 1, 1024, 256, True, 0),
          ("odd_t", (1, 1), (1, 1), 33, 259, 65, True, 0),
          ("odd_n", (1, 1), (1, 1), 33, 259, 65, False, 0),
          ("batch_t", (2, 2), (2, 2), 16, 64, 32, True, 0),
          ("batch_n", (2, 2), (2, 2), 16, 64, 32, False, 0),
          ("bcast_a", (1, 1), (4, 1), 8, 32, 16, True, 0),
          ("bcast_b", (1, 4), (1, 1), 8, 32, 16, False, 0),
          ("silu_t", (1, 1), (1, 1), 12, 96, 40, True, 1)]
    for name, (Ba, Ca), (Bb, Cb), M, K, N, tb, act in mm:
        a = f16(rng, (Ba, Ca, M, K))
        b = f16(rng, (Bb, Cb, N, K) if tb else (Bb, Cb, K, N))
        g[f"mm_{name}_a"], g[f"mm_{name}_b"] = a, b
        g[f"mm_{name}_meta"] = np.array([M, K, N, int(tb), act], dtype=np.int64)
        g[f"mm_{name}_out"] = ref_matmul(lib, a, b, tb, act)
    # rmsnorm: fp16 input, fp32 gains (the model path)
    x = f16(rng, (1, 1, 11, 320), -2.0, 2.0)
    gw = rng.uniform(0.5, 1.5, size=320).astype(np.float32)
    g["rms_x"], g["rms_g"], g["rms_out"] = x, gw, ref_rmsnorm(lib, x, gw)
    # rope on a contiguous [1, 4, 11, 32] and on the strided head view of [1, 1, 11, 128]
    x = f16(rng, (1, 4, 11, 32))
    g["rope_x"], g["rope_out"] = x, ref_rope(lib, x, 5, 10000.0)
    flat = f16(rng, (1, 1, 11, 128))
    g["rope_flat"] = flat
    g["rope_view_out"] = ref_rope(lib, flat.reshape(1, 11, 4, 32).transpose(0, 2, 1, 3), 3, 10000.0)
    # softmax widths of tests/vkllm_test_op_softmax.c:121-145, masked and unmasked
    for W, mask, off in ((64, 0, 0), (130, 1, 0), (96, 1, 40)):
        x = f16(rng, (1, 2, 4, W), -4.0, 4.0)
        g[f"sm_{W}_{mask}_{off}_x"] = x
        g[f"sm_{W}_{mask}_{off}_out"] = ref_softmax(lib, x, mask, off)
    # arg_max with planted ties (the test's function keeps the first maximum)
    x = f16(rng, (1, 1, 3, 1000))
    x[0, 0, 0, 17] = x[0, 0, 0, 900] = np.float16(3.0)
    x[0, 0, 1, 5] = x[0, 0, 1, 6] = np.float16(2.5)
    g["am_x"], g["am_out"], g["am_out_shader"] = x, ref_arg_max(lib, x), ref_arg_max_shader(x)
    # update_rows with an offset, into a zeroed cache
    src = f16(rng, (1, 4, 3, 16))
    cache = np.zeros((1, 4, 32, 16), dtype=np.float16)
    g["ur_src"], g["ur_cache"], g["ur_out"] = src, cache, ref_update_rows(lib, src, cache, 7)
    # embedding with out-of-vocabulary ids (the test's function maps them to row 0)
    table = f16(rng, (1, 1, 50, 32))
    ids = np.array([3, 0, 49, 50, 12, 77, 3, 1], dtype=np.uint32).reshape(1, 1, 1, 8)
    g["emb_table"], g["emb_ids"], g["emb_out"] = table, ids, ref_embedding(lib, ids, table)
    # copy of a permuted view [1, S, H, hd] -> contiguous (the attention output path)
    x = f16(rng, (1, 4, 6, 16)).transpose(0, 2, 1, 3)
    g["copy_x"], g["copy_out"] = np.ascontiguousarray(x.transpose(0, 2, 1, 3)), ref_copy(lib, x)
    # bin: add, sub, mul, div on fp16 and fp32
    for op in range(4):
        for dt in (np.float16, np.float32):
            a = rng.uniform(-2, 2, size=(2, 3, 8, 24)).astype(dt)
            b = rng.uniform(0.5, 2, size=(2, 3, 8, 24)).astype(dt)
            key = f"bin_{op}_{np.dtype(dt).name}"
            g[f"{key}_a"], g[f"{key}_b"], g[f"{key}_out"] = a, b, ref_bin(lib, a, b, op)
    # the reference's truncating fp32 -> fp16 helper on special and random values
    vals = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 1e6, -1e6, 6.1e-5, 6.0e-5, 5.96e-8, 1e-9,
                  np.inf, -np.inf, np.nan, 0.1, 1.0 / 3.0], dtype=np.float32),
        rng.standard_normal(2000).astype(np.float32) * np.float32(30.0)])
    g["f16_vals"] = vals
    g["f16_bits"] = np.array([lib.refpin_fp32_to_fp16(float(v)) for v in vals], dtype=np.uint16)
    return g


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--check", action="store_true", help="compare a fresh generation with the committed file")
    a = ap.parse_args()
    g = generate(refpin())
    if a.check:
        old = np.load(OUT)
        bad = [k for k in g if k not in old or old[k].tobytes() != g[k].tobytes()]
        assert not bad, f"differs from the committed fixture: {bad}"
        print("fixture matches the reference functions")
        return
    np.savez_compressed(OUT, **g)
    print("wrote", OUT, sum(v.nbytes for v in g.values()), "bytes")


if __name__ == "__main__":
    main()
