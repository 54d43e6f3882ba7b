"""The fused prefill step (a llama2 graph of S > 1 tokens run by the engine: RMSNORM, tensor-core
projections, RoPE with the KV-cache rows, one attention kernel for scores / causal softmax / probs.V,
Wo, the FFN and the logits) against the CPU oracle's restatement of the reference graph, on the
BASELINE tiny config (head_dim 48).

Cases: prompt lengths below, at and above one 64-key block; S = 48 = head_dim, where the
reference's shape-only MATMUL predicate reads V transposed (quirk Q1,
src/core/vkllm_op_matmul.c:14-30); and a prompt prefilled in two chunks, the second at a nonzero
position over the cache the first wrote. Compared: the argmax of EVERY row of the graph's output
(the reference computes all S rows, src/models/vkllm_models_llama2.c:569-587) and the last row's
fp16 logits, within the north_star bar (max-abs 2e-2, mean-abs 2e-3); the attention kernel's single-CTA
form (VKLLM_B200_PF_ATT_PAIR=0; the default splits the key blocks over a cluster of two CTAs) and the
node-by-node path (VKLLM_B200_PREFILL=0) must agree with the oracle the same way."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run_graph(vk, ctx, model, toks, offset):
    """One graph run over `toks` at `offset`; returns (argmax of every row, last-row logits)."""
    l = vk.lib()
    toks = np.asarray(toks, dtype=np.uint32)
    inp = vk.tensor_new(ctx, "input_toks", (1, 1, 1, len(toks)), vk.U32, mapped=True)
    g = C.POINTER(vk.Graph)()
    vk.check(l.vkllm_graph_new(ctx.ptr, C.byref(g)), "graph_new")
    try:
        vk.check(l.vkllm_models_llama2_build_graph(ctx.ptr, C.byref(model.m), inp, g, offset), "build_graph")
        vk.check(l.vkllm_graph_init(ctx.ptr, g), "graph_init")
        vk.check(l.vkllm_commands_upload(ctx.ptr, g.contents.commands, inp, toks.ctypes.data, toks.nbytes), "upload")
        vk.check(l.vkllm_graph_run(ctx.ptr, g), "graph_run")
        vk.check(l.vkllm_graph_post_run(ctx.ptr, g), "graph_post_run")
        out = g.contents.output_node
        vk.check(l.vkllm_tensor_invalid_cache(ctx.ptr, out), "invalid_cache")
        host = C.cast(out.contents.data.host, C.POINTER(C.c_uint32))
        ids = [int(host[i]) for i in range(len(toks))]
        return ids, model._last_logits(g)
    finally:
        l.vkllm_graph_free(ctx.ptr, g)


def check_rows(ids, logits, ref_ids, ref_all):
    """Every row's argmax equals the reference's, except at a reference tie at fp16 resolution (its
    top two logits within one fp16 ulp), reported as a warning; last-row logits within the bar."""
    import warnings

    from parity import ulp16

    for i, (a, b) in enumerate(zip(ids, ref_ids)):
        if a != int(b):
            r = ref_all[i].astype(np.float32)
            gap = float(r[int(b)] - r[a])
            assert gap <= ulp16(r[int(b)]), f"row {i}: {a} vs reference {int(b)}, gap {gap}"
            warnings.warn(f"prefill row {i}: argmax {a} vs reference {int(b)} at a reference tie (gap {gap})")
    d = np.abs(logits.astype(np.float32) - ref_all[-1].astype(np.float32))
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (d.max(), d.mean())


@pytest.mark.parametrize("n", [5, 47, 48, 49, 130])
@pytest.mark.parametrize("path", ["fused", "fused_single_cta", "nodes"])
def test_prefill_matches_oracle(vk, ctx, orc, tiny_gguf, n, path, monkeypatch):
    import gen_gguf

    if path == "nodes":
        monkeypatch.setenv("VKLLM_B200_PREFILL", "0")
    if path == "fused_single_cta":  # attention without the CTA-pair key split
        monkeypatch.setenv("VKLLM_B200_PF_ATT_PAIR", "0")
    path_, weights = tiny_gguf
    prompt = gen_gguf.prompt(100 + n, n)
    model = vk.Model(ctx).load(path_)
    try:
        ids, logits = run_graph(vk, ctx, model, prompt, 0)
    finally:
        model.free()
    m = orc.Llama2(dict(gen_gguf.TINY), weights)
    ref_logits, ref_ids = m.step(prompt, 0)
    m.close()
    check_rows(ids, logits, ref_ids, ref_logits)


def test_chunked_prefill_matches_oracle(vk, ctx, orc, tiny_gguf):
    """Two prefill chunks (20 tokens, then 70 at position 20) and one decode step, against the oracle
    run the same way."""
    import gen_gguf

    path_, weights = tiny_gguf
    prompt = gen_gguf.prompt(77, 90)
    model = vk.Model(ctx).load(path_)
    m = orc.Llama2(dict(gen_gguf.TINY), weights)
    try:
        for toks, off in ((prompt[:20], 0), (prompt[20:], 20)):
            ids, logits = run_graph(vk, ctx, model, toks, off)
            ref_logits, ref_ids = m.step(toks, off)
            check_rows(ids, logits, ref_ids, ref_logits)
        ids, logits = run_graph(vk, ctx, model, [ids[-1]], 90)
        ref_logits, ref_ids = m.step([int(ref_ids[-1])], 90)
        check_rows(ids, logits, ref_ids, ref_logits)
    finally:
        m.close()
        model.free()


@pytest.mark.parametrize("tile", ["256x192", "256x160", "256x224", "128x256"])
def test_grouped_prefill_gemm_tiles(vk, ctx, monkeypatch, tile):
    """Fused prefill of a model whose Q/K/V and FFN row counts are multiples of 256, so that the Q/K/V
    and up/gate projections run as grouped GEMMs over the model's own matrices. With the tile forced
    to one whose width does not divide the group (4096 / 192, 1280 / 192, ...), B tiles straddle two
    matrices and load in 32-row pieces. Every forced tile must give the prefill's tokens and, within
    the logit bar, its logits with the tuner's own choices."""
    import ctypes as C

    cfg = dict(block_count=2, context_length=512, embedding_length=512, head_count=4, ffn_length=1280,
               vocab_size=4096, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
    rng = np.random.default_rng(3)
    prompt = [int(t) for t in rng.integers(3, 4096, size=200)]
    runs = []
    for forced in (None, tile):
        if forced:
            monkeypatch.setenv("VKLLM_B200_GEMM_TILE", forced)
        else:
            monkeypatch.delenv("VKLLM_B200_GEMM_TILE", raising=False)
        model = vk.Model(ctx).init_random(cfg, 21)
        try:
            tok = model.step(prompt, 0)
            buf = np.zeros(cfg["vocab_size"], dtype=np.uint16)
            vk.check(vk.lib().vkllm_b200_engine_read_logits(ctx.ptr, C.byref(model.m), buf.ctypes.data,
                                                           cfg["vocab_size"]), "logits")
            runs.append((tok, buf.view(np.float16).astype(np.float32)))
        finally:
            model.free()
    (t0, l0), (t1, l1) = runs
    d = np.abs(l0 - l1)
    assert d.max() <= 2e-2 and d.mean() <= 2e-3, (tile, d.max(), d.mean())
    assert t0 == t1 or abs(l0[t0] - l0[t1]) <= 2e-3, (tile, t0, t1)
