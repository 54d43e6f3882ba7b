"""Pins the oracle (oracle/, the CPU restatement of the reference's shaders) to the reference's own
test-side CPU references: tests/golden/ref_ops.npz holds seeded inputs and the outputs of those
functions, compiled from the reference's test files and called by tests/golden/make_golden.py
(oracle/refpin/Makefile builds them). CPU only.

Bars: bit-exact for gather / row copies / argmax; for floating point, the reference tests' own
mean-squared-error thresholds (matmul 1e-2, rope 1e-2 for fp16; tests/vkllm_test_op_matmul.c:382,
tests/vkllm_test_op_rope.c:184) and, tighter, an element bound of two fp16 ulps of the element plus
1e-3 of the tensor's largest magnitude (the oracle rounds to nearest where the tests truncate, and
sums in the shaders' order).
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_ops.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLD)


def close(got, ref, mse_tol):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    mse = float(np.mean((got - ref) ** 2))
    assert mse <= mse_tol, f"mse {mse}"
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    bound = 2 * ulp + 1e-3 * max(np.abs(ref).max(), 1e-6)
    bad = np.abs(got - ref) > bound
    assert not bad.any(), f"{bad.sum()} elements off; max abs diff {np.abs(got - ref).max()}"


@pytest.mark.parametrize("name", ["gemv", "odd_t", "odd_n", "batch_t", "batch_n", "bcast_a", "bcast_b", "silu_t"])
def test_matmul_matches_reference_test_formula(orc, g, name):
    a, b = g[f"mm_{name}_a"], g[f"mm_{name}_b"]
    M, K, N, tb, act = (int(v) for v in g[f"mm_{name}_meta"])
    ref = g[f"mm_{name}_out"]
    got = orc.matmul(a, b, ref.shape, 1.0, act)
    close(got, ref, 1e-2)


def test_rmsnorm_matches_reference_test_formula(orc, g):
    close(orc.rmsnorm(g["rms_x"], g["rms_g"], 1e-6), g["rms_out"], 1e-3)


def test_rope_matches_reference_test_formula(orc, g):
    close(orc.rope(g["rope_x"], 5, 10000.0), g["rope_out"], 1e-2)


def test_rope_on_strided_head_view(orc, g):
    view = g["rope_flat"].reshape(1, 11, 4, 32).transpose(0, 2, 1, 3)
    close(orc.rope(view, 3, 10000.0), g["rope_view_out"], 1e-2)


@pytest.mark.parametrize("W,mask,off", [(64, 0, 0), (130, 1, 0), (96, 1, 40)])
def test_softmax_matches_reference_test_formula(orc, g, W, mask, off):
    x = g[f"sm_{W}_{mask}_{off}_x"]
    close(orc.softmax(x, mask, off), g[f"sm_{W}_{mask}_{off}_out"], 1e-3)


def test_arg_max_is_exact_and_follows_the_shader_tie_rule(orc, g):
    """Rows 0 and 1 hold planted ties: the shader's lane/tree rule (kept by the oracle and the CUDA
    kernels) and the reference test's first-maximum formula disagree there (quirk Q8); row 2 has no
    tie and all three agree."""
    got = orc.arg_max(g["am_x"])
    np.testing.assert_array_equal(got, g["am_out_shader"])
    np.testing.assert_array_equal(got[:, :, 2], g["am_out"][:, :, 2])
    assert (g["am_out_shader"][:, :, :2] != g["am_out"][:, :, :2]).all()


def test_update_rows_is_exact(orc, g):
    out = orc.update_rows(g["ur_src"], g["ur_cache"], 7)
    assert out.tobytes() == g["ur_out"].tobytes()


def test_embedding_is_exact_with_unk(orc, g):
    """The reference test's function maps out-of-range ids to row 0 (the shader's unk parameter,
    which the model sets to padding_token_id, defaults to 0)."""
    ids = g["emb_ids"]
    out = orc.embedding(ids, g["emb_table"], (1, 1, ids.shape[3], g["emb_table"].shape[3]), 0)
    assert out.tobytes() == g["emb_out"].tobytes()


def test_copy_of_permuted_view_is_exact(orc, g):
    x = g["copy_x"].transpose(0, 2, 1, 3)
    assert orc.copy(x).tobytes() == g["copy_out"].tobytes()


@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("dt", ["float16", "float32"])
def test_bin_matches_reference_test_formula(orc, g, op, dt):
    key = f"bin_{op}_{dt}"
    a, b, ref = g[f"{key}_a"], g[f"{key}_b"], g[f"{key}_out"]
    got = orc.bin_op(a, b, op, ref.dtype)
    if dt == "float32":
        np.testing.assert_array_equal(got, ref)
    else:
        close(got, ref, 1e-4)


def test_header_fp16_helper_is_the_reference_helper(tmp_path, g):
    """include/vkllm_common.h's vkllm_fp32_to_fp16 (which reference-style callers use to fill
    tensors) gives the reference helper's bits on every value, NaN, infinities and denormals
    included."""
    import ctypes as C
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "h.c"
    src.write_text('#include "vkllm_common.h"\n'
                   "unsigned short conv(float v) { return vkllm_fp32_to_fp16(v).bits; }\n"
                   "float back(unsigned short b) { vkllm_fp16_pack p = {b}; return vkllm_fp16_to_fp32(p); }\n")
    so = tmp_path / "h.so"
    subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-I", os.path.join(root, "include"), str(src), "-o", str(so)],
                   check=True)
    lib = C.CDLL(str(so))
    lib.conv.restype, lib.conv.argtypes = C.c_ushort, [C.c_float]
    got = np.array([lib.conv(float(v)) for v in g["f16_vals"]], dtype=np.uint16)
    np.testing.assert_array_equal(got, g["f16_bits"])


def test_fixture_is_reproduced_by_the_reference_functions():
    """Where the reference's test functions were compiled here (oracle/_ref/librefpin.so), every
    stored array is regenerated from them and compared byte for byte."""
    import make_golden

    if not os.path.exists(make_golden.REFPIN):
        pytest.skip("oracle/_ref/librefpin.so not built (needs the reference checkout)")
    fresh = make_golden.generate(make_golden.refpin())
    stored = np.load(GOLD)
    assert sorted(fresh) == sorted(stored.files)
    for k in fresh:
        assert fresh[k].tobytes() == stored[k].tobytes(), k


def test_planted_error_is_caught(orc, g):
    """The check is not vacuous: a one-ulp-per-element shift of the oracle's matmul is detected."""
    a, b = g["mm_odd_t_a"], g["mm_odd_t_b"]
    ref = g["mm_odd_t_out"]
    got = orc.matmul(a, b, ref.shape, 1.0, 0).astype(np.float32) * np.float32(1.01)
    with pytest.raises(AssertionError):
        close(got, ref, 1e-2)


def test_fp16_arithmetic_rounding_is_round_to_nearest_even(orc):
    """The fp16 arithmetic mode rounds after every operation with the F16C conversion; the storage
    conversion is the software f2h. Both must be IEEE round-to-nearest-even: compared with numpy's
    float32 -> float16 cast on every fp32 value next to each fp16 number and halfway point (ties),
    the subnormal range, the overflow edge, signed zeros, infinities and a random sweep."""
    h = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)  # every finite positive fp16
    mids = ((h[:-1].astype(np.float64) + h[1:]) / 2).astype(np.float32)  # exact ties in fp32
    near = np.concatenate([np.nextafter(v, np.float32(np.inf)) for v in (h, mids)] +
                          [np.nextafter(v, np.float32(0)) for v in (h, mids)])
    edge = np.array([65504, 65519.996, 65520, 65536, 1e30, np.inf, 0.0, 2.0 ** -25, 2.0 ** -25 * 1.0001,
                     2.0 ** -24, 3 * 2.0 ** -26, 1e-40, 5.96e-8], dtype=np.float32)
    rnd = np.random.default_rng(1).standard_normal(1 << 20).astype(np.float32) * np.float32(100)
    x = np.concatenate([h, mids, near, edge, rnd])
    x = np.concatenate([x, -x])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16)
    got = orc.round16(x)
    np.testing.assert_array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))
    np.testing.assert_array_equal(orc.f32_to_f16_bits(x), want.view(np.uint16))
