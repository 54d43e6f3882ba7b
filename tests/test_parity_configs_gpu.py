"""Parity at the shapes the benchmark runs: the persistent decode kernel at the LLaMA-2-7B geometry
(dim 4096, 32 heads of 128, SwiGLU 11008, vocab 32000) and the 13B geometry
(configs[4]: dim 5120, 40 heads, SwiGLU 13824), against the CPU oracle on the same weights.

The kernel's tile counts, row splits per phase, attention key splits and logits partition all depend
on these dimensions, so the tiny-model tests do not cover them. Weights come from the library's
random initialiser (the same generator as bench.py) and are downloaded for the oracle.

Bar. north_star states max-abs 2e-2 / mean-abs 2e-3 on the fp16 logits, quoted on the tiny config. At
the 7B depth the reference's own result is not defined that finely: the oracle's two arithmetic
modes, which restate the shader variants the reference picks by the device's shaderFloat16 bit,
differ from each other by max-abs 0.04-0.07 and mean-abs 0.008-0.014 on these logits, and their
greedy tokens part within a few steps. So each step's bar is the larger of the north_star numbers
and that reference-internal spread (fp16arith vs fp32arith, computed here on the same weights and
prompt, at the steps whose inputs agree in both modes; later steps keep the largest spread seen);
the comparison is against fp32arith, the parity target. Greedy tokens must be identical
except at a reference tie at fp16 resolution, which tests/parity.py reports as a warning. The
decode must have run on the persistent kernel."""
import ctypes as C

import numpy as np
import pytest

from parity import compare_greedy, download_weights

pytestmark = pytest.mark.gpu

CFG_7B = dict(block_count=32, context_length=4096, embedding_length=4096, head_count=32, ffn_length=11008,
              vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
CFG_13B = dict(block_count=40, context_length=4096, embedding_length=5120, head_count=40, ffn_length=13824,
               vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)


def oracle_with_bars(orc, cfg, weights, prompt, n_tokens, oracle_ctx):
    """The oracle's greedy run in both arithmetic modes. Returns the fp32arith tokens and logits (the
    parity target) and per-step max-abs / mean-abs bars: north_star's, widened to the fp16arith vs
    fp32arith spread. The spread is measured at the steps whose inputs agree in both modes; a later
    step (after the two modes' greedy tokens parted) takes the largest spread measured before it."""
    ocfg = dict(D=cfg["embedding_length"], H=cfg["head_count"], F=cfg["ffn_length"], V=cfg["vocab_size"],
                L=cfg["block_count"], ctx=oracle_ctx, eps=cfg["rms_eps"], rope_base=cfg["rope_freq_base"])
    orc.threads(0)
    runs = {}
    for mode in ("fp16", "fp32"):
        prev = orc.set_arith(mode)
        try:
            m = orc.Llama2(ocfg, weights, ctx=oracle_ctx)
            runs[mode] = m.generate(list(prompt), n_tokens)
            m.close()
        finally:
            orc.set_arith(prev)
    ref_toks, ref_logits = runs["fp32"]
    t16, l16 = runs["fp16"]
    max_bar, mean_bar, seen_max, seen_mean = [], [], 2e-2, 2e-3
    for i in range(n_tokens):
        if t16[:i] == ref_toks[:i]:
            spread = np.abs(l16[i].astype(np.float32) - ref_logits[i].astype(np.float32))
            seen_max, seen_mean = max(seen_max, float(spread.max())), max(seen_mean, float(spread.mean()))
        max_bar.append(seen_max)
        mean_bar.append(seen_mean)
    return ref_toks, ref_logits, max_bar, mean_bar


def run_pair(vk, ctx, orc, cfg, seed, prompt_len, n_tokens, oracle_ctx):
    prompt = list(np.random.default_rng(seed).integers(3, cfg["vocab_size"], size=prompt_len, dtype=np.uint32))
    model = vk.Model(ctx).init_random(cfg, seed)
    try:
        logits = []
        toks = model.generate(prompt, n_tokens, logits)
        persistent = vk.lib().vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m))
        weights = download_weights(vk, ctx, model, cfg)
    finally:
        model.free()
    ref_toks, ref_logits, max_bar, mean_bar = oracle_with_bars(orc, cfg, weights, prompt, n_tokens, oracle_ctx)
    return toks, logits, ref_toks, ref_logits, persistent, max_bar, mean_bar


def test_7b_decode_parity(vk, ctx, orc):
    """All 32 layers of the 7B geometry: a 4-token prefill then 4 decode steps on the persistent
    kernel (one launch per token)."""
    toks, logits, ref_toks, ref_logits, persistent, mb, ab = run_pair(vk, ctx, orc, CFG_7B, 31, 4, 5, 64)
    assert persistent
    compare_greedy(toks, logits, ref_toks, ref_logits, mb, ab, "7b")


def test_7b_geometry_decode_at_bench_positions(vk, ctx, orc):
    """Two layers of the 7B geometry decoding at positions 512..515 after a 512-token prefill: the
    attention phase splits each head's 513+ keys over several CTAs as in the benchmark."""
    cfg = dict(CFG_7B, block_count=2, context_length=1024)
    toks, logits, ref_toks, ref_logits, persistent, mb, ab = run_pair(vk, ctx, orc, cfg, 32, 512, 5, 1024)
    assert persistent
    compare_greedy(toks, logits, ref_toks, ref_logits, mb, ab, "7b geometry, 2 layers")


def test_13b_geometry_decode_parity(vk, ctx, orc):
    """Two layers of the 13B geometry (40 heads, SwiGLU 13824, dim 5120) after a 40-token prefill."""
    cfg = dict(CFG_13B, block_count=2, context_length=512)
    toks, logits, ref_toks, ref_logits, persistent, mb, ab = run_pair(vk, ctx, orc, cfg, 33, 40, 5, 512)
    assert persistent
    compare_greedy(toks, logits, ref_toks, ref_logits, mb, ab, "13b geometry, 2 layers")


def test_7b_geometry_batched_decode_at_bench_shape(vk, ctx, orc):
    """The batched decode at the benchmark's own shape: 64 sequences in one batch,
    each with its own 128-token prompt, KV rows for 384 positions, decoding positions 128..131 on two
    layers of the 7B geometry. M = 64 selects the benchmark's GEMM tiles and K splits and the staged
    attention at the same key counts. Eight slots spread over the batch (first, last and six between)
    are checked against the oracle run on that sequence alone, with the per-step bars of the other
    tests here (north_star's, widened to the reference-internal spread on that sequence)."""
    cfg = dict(CFG_7B, block_count=2, context_length=512)
    n_seqs, P, cap, n_steps = 64, 128, 384, 4
    rng = np.random.default_rng(34)
    prompts = [rng.integers(3, cfg["vocab_size"], size=P, dtype=np.uint32) for _ in range(n_seqs)]
    model = vk.Model(ctx).init_random(cfg, 34)
    batch = None
    try:
        batch = vk.Batch(model, n_seqs, cap)
        firsts = [batch.add_prompt(i, p) for i, p in enumerate(prompts)]
        toks, logits = [], []
        for _ in range(n_steps):
            toks.append(batch.decode(1)[0].copy())
            logits.append(batch.logits().copy())
        toks = np.stack(toks)
        weights = download_weights(vk, ctx, model, cfg)
    finally:
        if batch is not None:
            batch.free()
        model.free()
    for i in (0, 9, 18, 27, 36, 45, 54, 63):
        ref_toks, ref_logits, mb, ab = oracle_with_bars(orc, cfg, weights, prompts[i], n_steps + 1, cap)
        assert firsts[i] == ref_toks[0], f"sequence {i}: prefill token"
        compare_greedy([int(t) for t in toks[:, i]], [logits[s][i] for s in range(n_steps)], ref_toks[1:],
                       ref_logits[1:], mb[1:], ab[1:], f"batched 7b geometry, sequence {i}")
