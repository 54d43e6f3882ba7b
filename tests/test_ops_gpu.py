"""Per-operator parity: the CUDA path, called through the C-ABI exactly like the reference op tests
(tests/vkllm_test_op_*.c: tensor_new -> upload -> op init/run -> submit/wait -> download), against
the CPU oracle on the same seeded inputs. Shapes: the reference tests' own cases plus BASELINE's
operator microbenchmark shapes.

Tolerance for fp16 results: |gpu - oracle| <= 2e-3 * |oracle| + 2e-3 * max|oracle| (a couple of fp16
ulps; both sides accumulate in fp32 but in different orders), and the reference test's MSE bound as
a floor. Gathers, copies and argmax indices are bit-exact."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(20261201)


def rand(shape, dtype, lo=-1.0, hi=1.0):
    return RNG.uniform(lo, hi, size=shape).astype(dtype)


def close(gpu, ref, rel=2e-3, mse_bound=None):
    g = np.asarray(gpu, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert g.shape == r.shape
    scale = max(np.abs(r).max(), 1e-6)
    bad = np.abs(g - r) > rel * np.abs(r) + rel * scale
    assert not bad.any(), f"{bad.sum()} of {bad.size} mismatches; max abs diff {np.abs(g - r).max()} (scale {scale})"
    if mse_bound is not None:
        assert float(np.mean((g - r) ** 2)) <= mse_bound


def mk(vk, ctx, name, arr, dtype):
    t = vk.tensor_new(ctx, name, arr.shape, dtype)
    vk.put(ctx, t, arr)
    return t


def op_node(vk, ctx, name, shape, dtype, op, srcs, params):
    return vk.tensor_new(ctx, name, shape, dtype, op=op, srcs=srcs, params=params)


# ---------------------------------------------------------------------------------------------
# MATMUL: reference cases (tests/vkllm_test_op_matmul.c:179-286) and BASELINE microbench shapes.
MATMUL_CASES = [
    # B_a, C_a, B_b, C_b, M, K, N, dtype, transposed_b, act
    (1, 1, 1, 1, 1, 1024, 2048, "f32", True, 0),
    (1, 1, 1, 1, 1, 1024, 2048, "f16", True, 0),
    (1, 1, 1, 1, 512, 1024, 2048, "f16", True, 0),
    (1, 1, 1, 1, 333, 1259, 365, "f16", True, 0),
    (1, 1, 1, 1, 333, 1259, 365, "f32", True, 0),
    (1, 1, 1, 1, 512, 1024, 2048, "f16", False, 0),
    (1, 1, 1, 1, 333, 1259, 365, "f16", False, 0),
    (4, 1, 4, 1, 256, 512, 1024, "f16", True, 0),
    (2, 4, 2, 4, 128, 256, 512, "f16", False, 0),
    (1, 1, 4, 1, 128, 256, 512, "f16", True, 0),
    (4, 1, 1, 1, 128, 256, 512, "f16", False, 0),
    (1, 4, 4, 1, 64, 128, 256, "f16", True, 1),
    (1, 1, 1, 1, 512, 1024, 2048, "f16", True, 1),
    (1, 1, 1, 1, 1, 4096, 4096, "f16", True, 0),
    (1, 1, 1, 1, 1, 4096, 11008, "f16", True, 1),
    (1, 1, 1, 1, 1, 11008, 4096, "f16", True, 0),
    (1, 1, 1, 1, 8, 4096, 4096, "f16", True, 0),
    (1, 1, 1, 1, 64, 4096, 4096, "f16", True, 0),
    (1, 1, 1, 1, 512, 4096, 4096, "f16", True, 0),
    (1, 1, 1, 1, 1, 288, 32000, "f16", True, 0),
]


@pytest.mark.parametrize("case", MATMUL_CASES, ids=lambda c: "x".join(map(str, c)))
def test_matmul(vk, ctx, orc, case):
    Ba, Ca, Bb, Cb, M, K, N, dts, tb, act = case
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    a = rand((Ba, Ca, M, K), npdt)
    b = rand((Bb, Cb, N, K) if tb else (Bb, Cb, K, N), npdt)
    if not tb and K == N:
        pytest.skip("shape-only predicate would read B as transposed")
    A = mk(vk, ctx, "A", a, dt)
    B = mk(vk, ctx, "B", b, dt)
    out_shape = (max(Ba, Bb), max(Ca, Cb), M, N)
    params = bytes(C.c_float(1.0)) + bytes(C.c_int32(act))
    node = op_node(vk, ctx, "C", out_shape, dt, vk.OP_MATMUL, [A, B], params)
    vk.run_op(ctx, node, "vkllm_op_matmul_init", "vkllm_op_matmul_run")
    got = vk.fetch(ctx, node)
    ref = orc.matmul(a, b, out_shape, 1.0, act)
    close(got, ref, rel=2e-3 if dts == "f16" else 1e-4, mse_bound=1e-2 if dts == "f16" else 1e-3)
    for t in (node, A, B):
        vk.tensor_free(ctx, t)


def test_matmul_scale_and_batched_gemv(vk, ctx, orc):
    """Decode attention scores: GEMV batched over heads with scale 1/sqrt(hd) on a cache slice view."""
    H, L, hd, ctxlen = 6, 37, 48, 64
    q = rand((1, H, 1, hd), np.float16)
    cache = rand((1, H, ctxlen, hd), np.float16)
    Q = mk(vk, ctx, "q", q, vk.F16)
    K = mk(vk, ctx, "k", cache, vk.F16)
    ext = (C.c_uint32 * 4)(1, H, L, hd)
    Ks = vk.PT()
    vk.check(vk.lib().vkllm_tensor_slice0(ctx.ptr, K, ext, C.byref(Ks)), "slice0")
    scale = 1.0 / np.sqrt(hd)
    node = op_node(vk, ctx, "scores", (1, H, 1, L), vk.F16, vk.OP_MATMUL, [Q, Ks],
                   bytes(C.c_float(scale)) + bytes(C.c_int32(0)))
    vk.run_op(ctx, node, "vkllm_op_matmul_init", "vkllm_op_matmul_run")
    got = vk.fetch(ctx, node)
    ref = orc.matmul(q, cache[:, :, :L, :], (1, H, 1, L), scale, 0)
    close(got, ref)
    for t in (node, Ks, Q, K):
        vk.tensor_free(ctx, t)


# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("shape", [(1, 1, 10, 128), (2, 1, 5, 256), (1, 2, 8, 512), (3, 4, 6, 64), (1, 1, 512, 4096),
                                   (1, 1, 1, 288), (1, 1, 32, 288)])
def test_rmsnorm(vk, ctx, orc, shape):
    x = rand(shape, np.float16, -1, 1)
    g = rand((1, 1, 1, shape[3]), np.float32, 0.5, 1.5)
    X = mk(vk, ctx, "x", x, vk.F16)
    G = mk(vk, ctx, "g", g, vk.F32)
    eps = 1e-5
    node = op_node(vk, ctx, "y", shape, vk.F16, vk.OP_RMSNORM, [X, G], bytes(C.c_float(2.0)) + bytes(C.c_float(eps)))
    vk.run_op(ctx, node, "vkllm_op_rmsnorm_init", "vkllm_op_rmsnorm_run")
    close(vk.fetch(ctx, node), orc.rmsnorm(x, g.reshape(-1), eps), mse_bound=1e-2)
    for t in (node, X, G):
        vk.tensor_free(ctx, t)


class RopeParams(C.Structure):
    _fields_ = [("offset", C.c_uint32), ("base", C.c_float), ("neox_style", C.c_bool)]


@pytest.mark.parametrize("shape,offset,dts", [((1, 1, 10, 128), 0, "f32"), ((2, 1, 5, 64), 0, "f16"),
                                              ((1, 2, 8, 256), 5, "f16"), ((3, 4, 6, 32), 10, "f16"),
                                              ((8, 32, 32, 128), 0, "f16"), ((1, 32, 512, 128), 0, "f16"),
                                              ((1, 6, 1, 48), 200, "f16")])
@pytest.mark.parametrize("neox", [False, True])
def test_rope(vk, ctx, orc, shape, offset, dts, neox):
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    x = rand(shape, npdt)
    X = mk(vk, ctx, "x", x, dt)
    p = RopeParams(offset, 10000.0, neox)
    node = op_node(vk, ctx, "r", shape, dt, vk.OP_ROPE, [X], bytes(p))
    vk.run_op(ctx, node, "vkllm_op_rope_init", "vkllm_op_rope_run")
    close(vk.fetch(ctx, node), orc.rope(x, offset, 10000.0, neox), rel=2e-3 if dts == "f16" else 1e-4)
    for t in (node, X):
        vk.tensor_free(ctx, t)


def test_rope_strided_view(vk, ctx, orc):
    """The reference test's view case: [1,1,11,3200] reshaped to [1,11,32,100] and permuted to [1,32,11,100]
    (tests/vkllm_test_op_rope.c:126-132)."""
    base = rand((1, 1, 11, 3200), np.float16)
    Bt = mk(vk, ctx, "q", base, vk.F16)
    ref_t = vk.PT()
    vk.check(vk.lib().vkllm_tensor_copy_ref(ctx.ptr, Bt, C.byref(ref_t)), "copy_ref")
    vk.check(vk.lib().vkllm_tensor_reshape(ctx.ptr, ref_t, vk.u32x4((1, 11, 32, 100))), "reshape")
    vk.check(vk.lib().vkllm_tensor_permute(ctx.ptr, ref_t, vk.u32x4((0, 2, 1, 3))), "permute")
    node = op_node(vk, ctx, "rq", (1, 32, 11, 100), vk.F16, vk.OP_ROPE, [ref_t], bytes(RopeParams(3, 10000.0, False)))
    vk.run_op(ctx, node, "vkllm_op_rope_init", "vkllm_op_rope_run")
    view = base.reshape(1, 11, 32, 100).transpose(0, 2, 1, 3)
    close(vk.fetch(ctx, node), orc.rope(view, 3, 10000.0, False))
    for t in (node, ref_t, Bt):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("shape,mask,offsets,dts", [((1, 1, 10, 128), 0, 0, "f32"), ((2, 1, 5, 256), 1, 0, "f32"),
                                                    ((1, 1, 10, 128), 0, 0, "f16"), ((1, 2, 8, 512), 0, 0, "f16"),
                                                    ((1, 1, 10, 128), 1, 0, "f16"), ((1, 32, 1, 4096), 1, 4095, "f16"),
                                                    ((1, 6, 32, 32), 1, 0, "f16"), ((1, 6, 4, 40), 1, 36, "f16")])
def test_softmax(vk, ctx, orc, shape, mask, offsets, dts):
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    x = rand(shape, npdt, -4, 4)
    X = mk(vk, ctx, "x", x, dt)
    node = op_node(vk, ctx, "p", shape, dt, vk.OP_SOFTMAX, [X], bytes(C.c_int32(mask)) + bytes(C.c_uint32(offsets)))
    vk.run_op(ctx, node, "vkllm_op_softmax_init", "vkllm_op_softmax_run")
    close(vk.fetch(ctx, node), orc.softmax(x, mask, offsets), rel=2e-3 if dts == "f16" else 1e-5)
    for t in (node, X):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("src_shape,dst_shape,off,dts", [((1, 1, 5, 32), (1, 1, 10, 32), 5, "f32"),
                                                         ((2, 3, 4, 64), (2, 3, 10, 64), 2, "f16"),
                                                         ((1, 2, 8, 128), (1, 2, 16, 128), 4, "f16"),
                                                         ((1, 32, 1, 128), (1, 32, 4096, 128), 4095, "f16")])
def test_update_rows_bit_exact(vk, ctx, orc, src_shape, dst_shape, off, dts):
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    src = rand(src_shape, npdt)
    cache = rand(dst_shape, npdt)
    S = mk(vk, ctx, "src", src, dt)
    node = vk.tensor_new(ctx, "cache", dst_shape, dt, op=vk.OP_UPDATE_ROWS, srcs=[S], params=bytes(C.c_uint32(off)))
    vk.put(ctx, node, cache)
    vk.run_op(ctx, node, "vkllm_op_update_rows_init", "vkllm_op_update_rows_run")
    got = vk.fetch(ctx, node)
    assert np.array_equal(got.view(np.uint8), orc.update_rows(src, cache, off).view(np.uint8))
    for t in (node, S):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("dts", ["f16", "f32"])
def test_bin(vk, ctx, orc, op, dts):
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    shape = (2, 3, 7, 301)
    a = rand(shape, npdt)
    b = rand(shape, npdt, 0.5, 2.0)
    A, B = mk(vk, ctx, "a", a, dt), mk(vk, ctx, "b", b, dt)
    node = op_node(vk, ctx, "o", shape, dt, vk.OP_BIN, [A, B], bytes(C.c_int32(op)))
    vk.run_op(ctx, node, "vkllm_op_bin_init", "vkllm_op_bin_run")
    got = vk.fetch(ctx, node)
    ref = orc.bin_op(a, b, op, npdt)
    assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), "elementwise op must be bit-exact"
    for t in (node, A, B):
        vk.tensor_free(ctx, t)


def test_copy_permuted_bit_exact(vk, ctx, orc):
    x = rand((1, 6, 5, 48), np.float16)
    X = mk(vk, ctx, "x", x, vk.F16)
    r = vk.PT()
    vk.check(vk.lib().vkllm_tensor_copy_ref(ctx.ptr, X, C.byref(r)), "copy_ref")
    vk.check(vk.lib().vkllm_tensor_permute(ctx.ptr, r, vk.u32x4((0, 2, 1, 3))), "permute")
    node = op_node(vk, ctx, "c", (1, 5, 6, 48), vk.F16, vk.OP_COPY, [r], None)
    vk.run_op(ctx, node, "vkllm_op_copy_init", "vkllm_op_copy_run")
    got = vk.fetch(ctx, node)
    assert np.array_equal(got, x.transpose(0, 2, 1, 3))
    for t in (node, r, X):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("n_ids,V,D", [(1, 32000, 288), (32, 32000, 288), (512, 32000, 4096)])
def test_embedding_bit_exact(vk, ctx, orc, n_ids, V, D):
    table = rand((1, 1, V, D), np.float16)
    ids = RNG.integers(0, V + 50, size=(1, 1, 1, n_ids)).astype(np.uint32)  # some ids >= V -> unk
    T = mk(vk, ctx, "E", table, vk.F16)
    I = mk(vk, ctx, "ids", ids, vk.U32)
    node = op_node(vk, ctx, "emb", (1, 1, n_ids, D), vk.F16, vk.OP_EMBEDDING, [I, T], bytes(C.c_uint32(0)))
    vk.run_op(ctx, node, "vkllm_op_embedding_init", "vkllm_op_embedding_run")
    got = vk.fetch(ctx, node)
    ref = orc.embedding(ids, table, (1, 1, n_ids, D), 0)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    for t in (node, T, I):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("shape,dts", [((1, 1, 10, 128), "f32"), ((2, 4, 8, 64), "f16"), ((1, 12, 16, 512), "f16"),
                                       ((1, 1, 1, 10), "f32"), ((1, 1, 1, 32000), "f32"), ((1, 1, 3, 32000), "f16")])
def test_arg_max_exact(vk, ctx, orc, shape, dts):
    npdt = np.float16 if dts == "f16" else np.float32
    dt = vk.F16 if dts == "f16" else vk.F32
    x = rand(shape, npdt, -8, 8)
    X = mk(vk, ctx, "x", x, dt)
    node = op_node(vk, ctx, "am", shape[:3] + (1,), vk.U32, vk.OP_ARG_MAX, [X], None)
    vk.run_op(ctx, node, "vkllm_op_arg_max_init", "vkllm_op_arg_max_run")
    assert np.array_equal(vk.fetch(ctx, node), orc.arg_max(x))
    for t in (node, X):
        vk.tensor_free(ctx, t)


@pytest.mark.parametrize("dts", ["f32", "f16"])
def test_arg_max_long_rows_tie_rule(vk, ctx, orc, dts):
    """Rows of >= 1024 entries take the block-per-row kernel: the same lane/tree tie rule (maxima in
    several classes, repeated maxima inside one class far apart, all-equal rows) and the shader's
    NaN behaviour (a class whose first element is NaN keeps it; later NaNs never win)."""
    W = 32000
    npdt = np.float16 if dts == "f16" else np.float32
    x = rand((1, 1, 6, W), npdt, -4, 4)
    x[0, 0, 0, [5, 37, 100, 31999]] = 7.0      # classes 5, 5, 4, 31: the reference's tree decides
    x[0, 0, 1, [40 + 32 * 900, 8]] = 7.0        # class 8 twice, far apart: its first strict max wins
    x[0, 0, 2, :] = 1.0                         # all equal
    x[0, 0, 3, 3] = np.nan                      # class 3 starts with NaN and keeps it
    x[0, 0, 3, [3 + 32 * 10, 70]] = 7.0
    x[0, 0, 4, [900, 17 + 32 * 500]] = np.nan   # later NaNs never win
    x[0, 0, 4, 12345] = 7.0
    X = mk(vk, ctx, "x", x, vk.F16 if dts == "f16" else vk.F32)
    node = op_node(vk, ctx, "am", (1, 1, 6, 1), vk.U32, vk.OP_ARG_MAX, [X], None)
    vk.run_op(ctx, node, "vkllm_op_arg_max_init", "vkllm_op_arg_max_run")
    got = vk.fetch(ctx, node).reshape(-1)
    ref = orc.arg_max(x).reshape(-1)
    assert np.array_equal(got, ref), (got, ref)
    for t in (node, X):
        vk.tensor_free(ctx, t)


def test_arg_max_tie_rule(vk, ctx, orc):
    """Equal maxima: the winner follows the reference's lane/tree rule, not the lowest index."""
    W = 1000
    x = np.zeros((1, 1, 4, W), dtype=np.float32)
    x[0, 0, 0, [5, 37, 100, 999]] = 3.0     # lanes 5, 5, 4, 7
    x[0, 0, 1, [40, 8]] = 2.0                # lane 8 twice: first strict max (index 8) wins the lane
    x[0, 0, 2, [31, 63, 1]] = 1.0            # lane 31 vs lane 1
    x[0, 0, 3, :] = -1.0                     # all equal
    X = mk(vk, ctx, "x", x, vk.F32)
    node = op_node(vk, ctx, "am", (1, 1, 4, 1), vk.U32, vk.OP_ARG_MAX, [X], None)
    vk.run_op(ctx, node, "vkllm_op_arg_max_init", "vkllm_op_arg_max_run")
    got = vk.fetch(ctx, node).reshape(-1)
    ref = orc.arg_max(x).reshape(-1)
    assert np.array_equal(got, ref)
    for t in (node, X):
        vk.tensor_free(ctx, t)


def test_ffn_up_and_gate(vk, ctx, orc):
    x = rand((1, 1, 4, 256), np.float16)
    wu = rand((1, 1, 512, 256), np.float16, -0.1, 0.1)
    wg = rand((1, 1, 512, 256), np.float16, -0.1, 0.1)
    X, U, G = mk(vk, ctx, "x", x, vk.F16), mk(vk, ctx, "wu", wu, vk.F16), mk(vk, ctx, "wg", wg, vk.F16)
    node = op_node(vk, ctx, "y", (1, 1, 4, 512), vk.F16, vk.OP_FFN_UP_AND_GATE, [X, U, G], None)
    vk.run_op(ctx, node, "vkllm_op_ffn_up_and_gate_init", "vkllm_op_ffn_up_and_gate_run")
    close(vk.fetch(ctx, node), orc.ffn_up_gate(x, wu, wg, np.float16))
    for t in (node, X, U, G):
        vk.tensor_free(ctx, t)


def test_invalid_shapes_are_rejected(vk, ctx):
    a = vk.tensor_new(ctx, "a", (1, 1, 4, 64), vk.F16)
    b = vk.tensor_new(ctx, "b", (1, 1, 32, 65), vk.F16)
    node = op_node(vk, ctx, "c", (1, 1, 4, 32), vk.F16, vk.OP_MATMUL, [a, b], bytes(C.c_float(1.0)) + bytes(C.c_int32(0)))
    cmd = vk.Commands(ctx)
    assert vk.lib().vkllm_op_matmul_init(ctx.ptr, cmd.ptr, node) == vk.ARGS
    cmd.close()
    bad = vk.PT()
    assert vk.lib().vkllm_tensor_new(ctx.ptr, b"z", vk.u32x4((1, 0, 1, 1)), vk.F16, 0, None, 0, None, 0, False,
                                     C.byref(bad)) == vk.ARGS
    for t in (node, a, b):
        vk.tensor_free(ctx, t)
