"""Batched greedy decode of independent sequences (BASELINE configs[3] shape, here on the tiny
model): every sequence of the batch must decode exactly what it decodes alone. Each sequence is
prefilled through the drop-in graph API, moved into its batch slot, then all decode together on the
tensor-core GEMM path (M = number of sequences). Reference: the CPU oracle run on each sequence
separately (prefill + the same number of greedy steps). Bar: identical
greedy token ids for the first 32 steps of every sequence, and fp16 logits within max-abs 2e-2 /
mean-abs 2e-3 at every step. A token mismatch fails with the reference's logits of both tokens and
its top two, so a tie broken the other way by a different fp32 summation order is visible as such."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (seed, prompt length); the last sequence passes Lk == hd (48 on the tiny model), where the
# reference reads V transposed
PROMPTS = [(11, 8), (12, 12), (13, 5), (14, 1), (15, 40)]
N_STEPS = 32

# the batch's kernel choices (read when the batch is created): the default (bulk-copy staged
# attention, tile-order GEMM operands), the register-loading attention kernel, the staged kernel
# with 128 threads, and row-major GEMM operands
VARIANTS = {"default": {}, "att_registers": {"VKLLM_B200_BATCH_ATT_STAGED": "0"},
            "att_staged_128": {"VKLLM_B200_BATCH_ATT_STAGED": "128"}, "rowmajor_b": {"VKLLM_B200_BATCH_TILED": "0"}}


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
        for s in range(N_STEPS):
            r = np.asarray(ref_logits[s + 1], dtype=np.float32)
            d = np.abs(logits[s][i].astype(np.float32) - r)
            assert d.max() <= 2e-2 and d.mean() <= 2e-3, (i, s, d.max(), d.mean())
            if ours[s] != ref[s]:
                raise AssertionError(f"sequence {i} step {s}: token {ours[s]} vs reference {ref[s]}; reference "
                                     f"logits {r[ref[s]]} (its choice) / {r[ours[s]]} (ours), its top two "
                                     f"{np.sort(r)[-2:]}; our logits {logits[s][i][ref[s]]} / {logits[s][i][ours[s]]}")


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
