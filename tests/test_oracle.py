"""Pins the oracle (oracle/, the CPU restatement of the reference's shaders) to the reference's own
test-side CPU references: tests/golden/ref_ops.npz holds seeded inputs and the outputs of those
functions (restated by tests/golden/make_golden.py). CPU only.

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
    ids = g["emb_ids"]
    out = orc.embedding(ids, g["emb_table"], (1, 1, ids.shape[3], g["emb_table"].shape[3]), 2)
    assert out.tobytes() == g["emb_out"].tobytes()


def test_planted_error_is_caught(orc, g):
    """The check is not vacuous: a one-ulp-per-element shift of the oracle's matmul is detected."""
    a, b = g["mm_odd_t_a"], g["mm_odd_t_b"]
    ref = g["mm_odd_t_out"]
    got = orc.matmul(a, b, ref.shape, 1.0, 0).astype(np.float32) * np.float32(1.01)
    with pytest.raises(AssertionError):
        close(got, ref, 1e-2)
