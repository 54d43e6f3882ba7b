"""The oracle's second arithmetic mode: the shader variants a Vulkan device reporting shaderFloat16
selects (fp16 GEMV accumulation, fp16 dot pairs in the GEMM, fp16 softmax and RoPE;
src/shaders/BUILD:69-108, src/core/vkllm_op_matmul.c:92-102). The reference's numbers depend on that
device bit, so its divergence from the default f16f32 arithmetic (the parity target) is measured
here on the BASELINE tiny config: per decode step, the max-abs and mean-abs difference of the fp16
logits and whether the greedy tokens agree. CPU only.

The bars below only check that the mode is live and stays a small perturbation of the same model;
the numbers themselves are the report (pytest -s prints them)."""
import numpy as np
import pytest

N_PROMPT, N_STEPS = 32, 33


@pytest.fixture(scope="module")
def runs(orc):
    import gen_gguf

    w = gen_gguf.make_weights(gen_gguf.TINY, 1234)
    prompt = gen_gguf.prompt(7, N_PROMPT)
    out = {}
    for mode in ("fp32", "fp16"):
        prev = orc.set_arith(mode)
        try:
            m = orc.Llama2(dict(gen_gguf.TINY), w)
            out[mode] = m.generate(prompt, N_STEPS)
            m.close()
        finally:
            orc.set_arith(prev)
    return out


def test_fp16arith_divergence_from_fp32arith(runs):
    t32, l32 = runs["fp32"]
    t16, l16 = runs["fp16"]
    first = next((i for i in range(N_STEPS) if t32[i] != t16[i]), N_STEPS)
    rows = []
    for i in range(min(first + 1, N_STEPS)):  # steps whose inputs agree
        d = np.abs(l16[i].astype(np.float32) - l32[i].astype(np.float32))
        rows.append((i, float(d.max()), float(d.mean())))
    print("\nfp16arith vs fp32arith, tiny config: step, max-abs, mean-abs of the fp16 logits")
    for r in rows:
        print("  %2d  %.5f  %.6f" % r)
    print("greedy tokens agree for the first %d of %d steps" % (first, N_STEPS))
    assert any(r[1] > 0 for r in rows), "fp16 mode changed nothing"
    assert all(r[2] < 5e-2 for r in rows)
    assert first >= 1


def test_mode_switch_restores_fp32(orc, runs):
    """After the fp16 run the default mode is back: a fresh fp32 run repeats the first one exactly."""
    import gen_gguf

    assert orc.set_arith("fp32") == "fp32"
    w = gen_gguf.make_weights(gen_gguf.TINY, 1234)
    m = orc.Llama2(dict(gen_gguf.TINY), w)
    toks, lg = m.generate(gen_gguf.prompt(7, N_PROMPT), 3)
    m.close()
    assert toks == runs["fp32"][0][:3]
    assert all(a.tobytes() == b.tobytes() for a, b in zip(lg, runs["fp32"][1][:3]))
