"""Batched greedy decode of independent sequences (BASELINE configs[3] shape, here on the tiny
model): every sequence of the batch must decode exactly what it decodes alone. Each sequence is
prefilled through the drop-in graph API, moved into its batch slot, then all decode together on the
tensor-core GEMM path (M = number of sequences). Reference: the CPU oracle run on each sequence
separately (prefill + the same number of greedy steps). Bar: fp16 logits
within max-abs 2e-2 / mean-abs 2e-3 at every compared step, and identical greedy token ids for 32
steps of every sequence, except at a reference tie at fp16 resolution (its top two logits within one
fp16 ulp), which tests/parity.py reports as a warning with both tokens' logits; the comparison of
that sequence stops there, since later inputs differ."""
import numpy as np
import pytest

from parity import compare_greedy

pytestmark = pytest.mark.gpu

# (seed, prompt length); the last sequence passes Lk == hd (48 on the tiny model), where the
# reference reads V transposed
PROMPTS = [(11, 8), (12, 12), (13, 5), (14, 1), (15, 40)]
N_STEPS = 32

# the batch's kernel choices (read when the batch is created): the default (bulk-copy staged
# attention, tile-order GEMM operands), the register-loading attention kernel, the staged kernel
# with 128 threads, row-major GEMM operands, and GEMM tiles that stage all 128 rows of A (up to 8
# sequences the default tiles stage 64)
VARIANTS = {"default": {}, "att_registers": {"VKLLM_B200_BATCH_ATT_STAGED": "0"},
            "att_staged_128": {"VKLLM_B200_BATCH_ATT_STAGED": "128"}, "rowmajor_b": {"VKLLM_B200_BATCH_TILED": "0"},
            "full_a_tiles": {"VKLLM_B200_BATCH_GEMM": "3,3,4,1,1,0"}}


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_batched_decode_matches_each_sequence_alone(vk, ctx, tiny_gguf, orc, variant, monkeypatch):
    import gen_gguf

    for k, v in VARIANTS[variant].items():
        monkeypatch.setenv(k, v)
    path, weights = tiny_gguf
    cfg = dict(gen_gguf.TINY)
    prompts = [gen_gguf.prompt(seed, n) for seed, n in PROMPTS]
    model = vk.Model(ctx).load(path)
    batch = None
    try:
        batch = vk.Batch(model, len(prompts), 96)
        firsts = [batch.add_prompt(i, p) for i, p in enumerate(prompts)]
        toks, logits = [], []
        for _ in range(N_STEPS):  # step by step to compare every step's logits
            toks.append(batch.decode(1)[0])
            logits.append(batch.logits())
        toks = np.stack(toks)
    finally:
        if batch is not None:
            batch.free()
        model.free()
    for i, p in enumerate(prompts):
        m = orc.Llama2(cfg, weights)
        ref_toks, ref_logits = m.generate(p, N_STEPS + 1)
        m.close()
        assert firsts[i] == ref_toks[0]
        ours = [int(t) for t in toks[:, i]]
        ref = ref_toks[1:N_STEPS + 1]
        compare_greedy(ours, [logits[st][i] for st in range(N_STEPS)], ref, ref_logits[1:N_STEPS + 1], 2e-2, 2e-3,
                       f"{variant} sequence {i}")


def test_batch_rejects_a_sequence_past_its_capacity(vk, ctx, tiny_gguf):
    import gen_gguf

    path, _ = tiny_gguf
    model = vk.Model(ctx).load(path)
    batch = None
    try:
        batch = vk.Batch(model, 2, 16)
        batch.add_prompt(0, gen_gguf.prompt(3, 10))
        batch.add_prompt(1, gen_gguf.prompt(4, 4))
        batch.decode(5)  # positions 10..14 fit in 16 rows
        with pytest.raises(RuntimeError):
            batch.decode(4)  # sequence 0 would write rows 15..18
    finally:
        if batch is not None:
            batch.free()
        model.free()


def test_in_place_weights_match_tile_copies(vk, ctx, monkeypatch):
    """VKLLM_B200_BATCH_TILED=2 reads the model's own matrices as grouped GEMM operands instead of the
    batch's tile-order copies: the same GEMM tiles and K splits over the same values, so tokens and
    logits are bit-identical. A random model whose Q/K/V and FFN row counts are multiples of 256, so
    that whole B tiles lie in one matrix."""
    cfg = dict(block_count=2, context_length=256, embedding_length=512, head_count=4, ffn_length=1280,
               vocab_size=4096, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(3, 4096, size=n, dtype=np.uint32) for n in (9, 3, 17, 1, 30, 6)]
    runs = []
    for tiled in ("1", "2"):
        monkeypatch.setenv("VKLLM_B200_BATCH_TILED", tiled)
        model = vk.Model(ctx).init_random(cfg, 77)
        batch = None
        try:
            batch = vk.Batch(model, len(prompts), 64)
            firsts = [batch.add_prompt(i, p) for i, p in enumerate(prompts)]
            toks, logits = [], []
            for _ in range(16):
                toks.append(batch.decode(1)[0].copy())
                logits.append(batch.logits().copy())
        finally:
            if batch is not None:
                batch.free()
            model.free()
        runs.append((firsts, np.stack(toks), np.stack(logits)))
    (f1, t1, l1), (f2, t2, l2) = runs
    assert f1 == f2
    assert np.array_equal(t1, t2)
    assert np.array_equal(l1.view(np.uint16), l2.view(np.uint16))


# (head size, heads, prompt lengths): ragged key counts (tails of 1..15 rows past a 16-key block),
# a one-token prompt, and one sequence that passes Lk == hd (quirk Q1) during the steps
TC_MODELS = {64: (8, (1, 17, 40, 56, 9, 33)), 128: (4, (1, 17, 120, 70, 9, 100))}
# chunk rows : ring buffers : threads per CTA of the tensor-core attention (read when the batch is
# created); threads 0 runs the FMA staged kernel on the same models
TC_CHUNKS = ["48:2:128", "64:2:256", "16:4:128", "128:2:256", "48:3:128", "32:2:128", "64:2:0"]


@pytest.mark.parametrize("chunk", TC_CHUNKS)
@pytest.mark.parametrize("hd", sorted(TC_MODELS))
def test_tensor_core_attention_matches_each_sequence_alone(vk, ctx, orc, hd, chunk, monkeypatch):
    """k_b_attention_tc (mma.sync over TMA-swizzled K/V chunks) at head sizes 64 and 128, 4 and 8
    warps per CTA and several chunk / ring shapes: every sequence of a batch of 6 decodes what the oracle decodes on it alone
    (logits within north_star's bar at every step, greedy ids identical except at a reference tie).
    Prompts of 1 to 120 tokens put the last key block's tail at every remainder; one sequence per
    model crosses Lk == hd, where the kernel runs the reference's transposed-V reading."""
    from parity import download_weights

    c, r, t = chunk.split(":")
    monkeypatch.setenv("VKLLM_B200_BATCH_ATT_CHUNK", c)
    monkeypatch.setenv("VKLLM_B200_BATCH_ATT_RING", r)
    monkeypatch.setenv("VKLLM_B200_BATCH_ATT_TC", t)
    H, lens = TC_MODELS[hd]
    cfg = dict(block_count=2, context_length=256, embedding_length=H * hd, head_count=H, ffn_length=1280,
               vocab_size=4096, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
    rng = np.random.default_rng(hd)
    prompts = [rng.integers(3, cfg["vocab_size"], size=n, dtype=np.uint32) for n in lens]
    n_steps, cap = 24, 192
    model = vk.Model(ctx).init_random(cfg, 40 + hd)
    batch = None
    try:
        batch = vk.Batch(model, len(prompts), cap)
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
    ocfg = dict(D=cfg["embedding_length"], H=H, F=cfg["ffn_length"], V=cfg["vocab_size"], L=cfg["block_count"],
                ctx=cap, eps=cfg["rms_eps"], rope_base=cfg["rope_freq_base"])
    orc.threads(0)
    for i, p in enumerate(prompts):
        m = orc.Llama2(ocfg, weights, ctx=cap)
        ref_toks, ref_logits = m.generate(list(p), n_steps + 1)
        m.close()
        assert firsts[i] == ref_toks[0]
        compare_greedy([int(t) for t in toks[:, i]], [logits[s][i] for s in range(n_steps)], ref_toks[1:],
                       ref_logits[1:], 2e-2, 2e-3, f"hd {hd} chunk {chunk} sequence {i}")
