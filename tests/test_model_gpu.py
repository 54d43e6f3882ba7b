"""End-to-end LLaMA-2 parity on the BASELINE tiny config (dim 288, 6 layers, 6 heads of 48, SwiGLU
768, vocab 32000, context 256): a seeded synthetic GGUF loaded through vkllm_models_llama2_load and
driven by the reference token loop (tests/vkllm_test_infer_gguf.c:181-272) through the C-ABI, against
the CPU oracle's restatement of the reference graph on the same weights and prompt.

Bar: greedy token ids identical for the first 32 steps; fp16 logits within
max-abs 2e-2 and mean-abs 2e-3 at every step whose inputs agree. Every execution path is checked:
node by node (STRICT, the reference's own DAG), the persistent decode kernel (FUSED, the default, its row partition calibrated at engine creation),
the CUDA-graph decode path that runs when cooperative launch is unavailable (VKLLM_B200_DECODE=graph),
the persistent kernel with equal row shares (VKLLM_B200_PERSIST_BALANCE=0), and the persistent
kernel whose Wo and down tiles wait per input segment for its producers instead of at grid barriers
(VKLLM_B200_PERSIST_FINE=1)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PROMPT, N_STEPS = 32, 65  # prefill + 64 greedy decode steps


@pytest.fixture(scope="module")
def reference_run(tiny_gguf, orc):
    import gen_gguf

    _, weights = tiny_gguf
    cfg = dict(gen_gguf.TINY)
    m = orc.Llama2(cfg, weights)
    prompt = gen_gguf.prompt(7, N_PROMPT)
    toks, logits = m.generate(prompt, N_STEPS)
    m.close()
    return prompt, toks, logits


MODES = {"strict": {}, "fused": {}, "fused_graph": {"VKLLM_B200_DECODE": "graph"},
         "fused_equal_shares": {"VKLLM_B200_PERSIST_BALANCE": "0"}, "fused_fine": {"VKLLM_B200_PERSIST_FINE": "1"}}


@pytest.mark.parametrize("mode", list(MODES))
def test_tiny_token_loop_parity(vk, ctx, tiny_gguf, reference_run, mode, monkeypatch):
    import ctypes as C

    for k, v in MODES[mode].items():  # read when the model's decode engine is created
        monkeypatch.setenv(k, v)
    path, _ = tiny_gguf
    prompt, ref_toks, ref_logits = reference_run
    ctx.set_exec_mode(vk.EXEC_STRICT if mode == "strict" else vk.EXEC_FUSED)
    model = vk.Model(ctx).load(path)
    try:
        assert model.meta.embedding_length == 288 and model.meta.block_count == 6
        logits = []
        toks = model.generate(prompt, N_STEPS, logits)
        if mode != "strict":
            persistent = vk.lib().vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m))
            assert bool(persistent) == (mode != "fused_graph"), (mode, persistent)
    finally:
        model.free()
        ctx.set_exec_mode(vk.EXEC_FUSED)
    assert toks[:32] == ref_toks[:32], f"first divergence at {next(i for i in range(32) if toks[i] != ref_toks[i])}"
    n_same = next((i for i in range(N_STEPS) if toks[i] != ref_toks[i]), N_STEPS)
    for i in range(min(n_same + 1, N_STEPS)):
        d = np.abs(logits[i].astype(np.float32) - ref_logits[i].astype(np.float32))
        assert d.max() <= 2e-2, f"step {i}: max-abs {d.max()}"
        assert d.mean() <= 2e-3, f"step {i}: mean-abs {d.mean()}"


# Long-context shape for the persistent kernel's attention phase: 8 heads of 128 split 18 ways, 24
# key groups per split (F = 6144 sizes the shared scratch for them), so a decode at position ~1800
# reduces ~100 keys per split in 5 rounds, past its 4-round load window (the tiny model needs 1).
LONG = dict(D=1024, L=1, H=8, F=6144, V=512, ctx=2048, eps=1e-5, rope_base=10000.0)
LONG_PROMPT, LONG_STEPS = 1800, 9


def test_long_context_decode_parity(vk, ctx, orc, tmp_path):
    import ctypes as C

    import gen_gguf

    path = str(tmp_path / "long.gguf")
    weights = gen_gguf.write_gguf(path, LONG, seed=99)
    prompt = gen_gguf.prompt(5, LONG_PROMPT, vocab=LONG["V"])
    model = vk.Model(ctx).load(path)
    try:
        logits = []
        toks = model.generate(prompt, LONG_STEPS, logits)
        assert vk.lib().vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m))
    finally:
        model.free()
    m = orc.Llama2(dict(LONG), weights)
    ref_toks, ref_logits = m.generate(prompt, LONG_STEPS)
    m.close()
    from parity import compare_greedy

    compare_greedy(toks, logits, ref_toks, ref_logits, 2e-2, 2e-3, "long context")


def test_tokenizer_and_metadata(vk, ctx, tiny_gguf):
    import ctypes as C

    path, _ = tiny_gguf
    model = vk.Model(ctx).load(path)
    try:
        m = model.meta
        assert (m.vocab_size, m.head_count, m.context_length) == (32000, 6, 256)
        assert abs(m.layer_norm_rms_epsilon - 1e-5) < 1e-12 and m.bos_token_id == 1
        arr = C.POINTER(vk.TokenIdArray)()
        vk.check(vk.lib().vkllm_models_llama2_tokenize(C.byref(model.m), b"<t5><t6> <t7>", C.byref(arr)), "tokenize")
        ids = [arr.contents.data[i] for i in range(arr.contents.used_n)]
        assert ids[0] == 1 and ids[-1] == 2  # add_bos / add_eos defaults
    finally:
        model.free()


def test_device_loop_matches_api_loop(vk, ctx, tiny_gguf, reference_run):
    """The device-resident loop used by bench.py (engine set_state + decode_steps) produces the same
    greedy tokens as the reference-style API loop."""
    import ctypes as C

    path, _ = tiny_gguf
    prompt, ref_toks, _ = reference_run
    model = vk.Model(ctx).load(path)
    try:
        first = model.step(list(prompt), 0)  # prefill through the API
        assert first == ref_toks[0]
        model.engine_prepare()
        l = vk.lib()
        vk.check(l.vkllm_b200_engine_set_state(ctx.ptr, C.byref(model.m), first, N_PROMPT), "set_state")
        vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(model.m), 40), "decode_steps")
        out = np.zeros(40, dtype=np.uint32)
        vk.check(l.vkllm_b200_engine_read_tokens(ctx.ptr, C.byref(model.m), out.ctypes.data, 40), "read_tokens")
        assert list(out) == ref_toks[1:41]
        kps = l.vkllm_b200_engine_kernels_per_step(ctx.ptr, C.byref(model.m))
        if l.vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m)):
            assert kps == 1 and l.vkllm_b200_engine_last_launches(ctx.ptr, C.byref(model.m)) == 1  # 40 steps, 1 launch
        else:
            assert kps == 2 + 6 * 6
    finally:
        model.free()


def test_random_init_matches_host_generator(vk, ctx):
    """vkllm_b200_models_llama2_init_random fills weights with the documented generator."""
    cfg = dict(block_count=1, context_length=64, embedding_length=256, head_count=4, ffn_length=512,
               vocab_size=1000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
    model = vk.Model(ctx).init_random(cfg, seed=99)
    try:
        got = vk.fetch(ctx, model.m.weights.tok_embed_weights).reshape(-1).view(np.uint16)
        ref = vk.random_f16_host(99, 0, 0.02, 0, got.size)
        assert np.array_equal(got, ref)
        wq = vk.fetch(ctx, model.block(0).WQ).reshape(-1).view(np.uint16)
        assert np.array_equal(wq, vk.random_f16_host(99, 3, 0.02, 0, wq.size))
    finally:
        model.free()


def test_gguf_loader_matches_the_gguf_reader(vk, ctx, tiny_gguf):
    """The C++ GGUF loader (the gguf-tools call sites of src/models/vkllm_models_llama2.c:185-392)
    against the `gguf` package's reader on the same file: every tensor's bytes, after upload and
    download, are identical."""
    import gguf

    path, _ = tiny_gguf
    rd = gguf.GGUFReader(path)
    want = {t.name: np.asarray(t.data).reshape(-1) for t in rd.tensors}
    model = vk.Model(ctx).load(path)
    try:
        w = model.m.weights
        got = {"token_embd.weight": vk.fetch(ctx, w.tok_embed_weights), "output.weight": vk.fetch(ctx, w.output_weight),
               "output_norm.weight": vk.fetch(ctx, w.output_norm_weight)}
        names = {"attn_norm_weight": "attn_norm", "ffn_norm_weight": "ffn_norm", "WQ": "attn_q", "WK": "attn_k",
                 "WV": "attn_v", "WO": "attn_output", "WG": "ffn_gate", "WU": "ffn_up", "WD": "ffn_down"}
        for l in range(model.meta.block_count):
            bw = model.block(l)
            for f, n in names.items():
                got[f"blk.{l}.{n}.weight"] = vk.fetch(ctx, getattr(bw, f))
    finally:
        model.free()
    assert set(got) == set(want)
    for n, a in want.items():
        assert got[n].reshape(-1).tobytes() == a.tobytes(), n
