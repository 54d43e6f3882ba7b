"""Parity at the shapes the benchmark runs: the persistent decode kernel at the LLaMA-2-7B geometry
(dim 4096, 32 heads of 128, SwiGLU 11008, vocab 32000) and the 13B geometry
(configs[4]: dim 5120, 40 heads, SwiGLU 13824), against the CPU oracle on the same weights.

The kernel's tile counts, row splits per phase, attention key splits and logits partition all depend
on these dimensions, so the tiny-model tests do not cover them. Weights come from the library's
random initialiser (the same generator as bench.py) and are downloaded for the oracle.

Bar: identical greedy token ids, fp16 logits within max-abs 2e-2 and
mean-abs 2e-3 at every step, and the decode ran on the persistent kernel."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG_7B = dict(block_count=32, context_length=4096, embedding_length=4096, head_count=32, ffn_length=11008,
              vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
CFG_13B = dict(block_count=40, context_length=4096, embedding_length=5120, head_count=40, ffn_length=13824,
               vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)


def download_weights(vk, ctx, model, cfg):
    w = {}
    m = model.m.weights
    w["token_embd.weight"] = vk.fetch(ctx, m.tok_embed_weights).reshape(cfg["vocab_size"], -1)
    w["output.weight"] = vk.fetch(ctx, m.output_weight).reshape(cfg["vocab_size"], -1)
    w["output_norm.weight"] = vk.fetch(ctx, m.output_norm_weight).reshape(-1)
    names = {"attn_norm_weight": "attn_norm", "ffn_norm_weight": "ffn_norm", "WQ": "attn_q", "WK": "attn_k",
             "WV": "attn_v", "WO": "attn_output", "WG": "ffn_gate", "WU": "ffn_up", "WD": "ffn_down"}
    for l in range(cfg["block_count"]):
        bw = model.block(l)
        for f, n in names.items():
            a = vk.fetch(ctx, getattr(bw, f))
            w[f"blk.{l}.{n}.weight"] = a.reshape(-1) if "norm" in n else a.reshape(a.shape[2], a.shape[3])
    return w


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
    ocfg = dict(D=cfg["embedding_length"], H=cfg["head_count"], F=cfg["ffn_length"], V=cfg["vocab_size"],
                L=cfg["block_count"], ctx=oracle_ctx, eps=cfg["rms_eps"], rope_base=cfg["rope_freq_base"])
    orc.threads(0)
    m = orc.Llama2(ocfg, weights, ctx=oracle_ctx)
    ref_toks, ref_logits = m.generate(prompt, n_tokens)
    m.close()
    return toks, logits, ref_toks, ref_logits, persistent


def assert_parity(toks, logits, ref_toks, ref_logits):
    for i in range(len(ref_toks)):
        r = np.asarray(ref_logits[i], dtype=np.float32)
        d = np.abs(np.asarray(logits[i], dtype=np.float32) - r)
        assert d.max() <= 2e-2 and d.mean() <= 2e-3, f"step {i}: max-abs {d.max()} mean-abs {d.mean()}"
        if toks[i] != ref_toks[i]:
            top2 = np.sort(r)[-2:]
            raise AssertionError(f"step {i}: token {toks[i]} vs reference {ref_toks[i]} (reference logits "
                                 f"{r[ref_toks[i]]} / {r[toks[i]]}, its top two {top2})")


def test_7b_decode_parity(vk, ctx, orc):
    """All 32 layers of the 7B geometry: a 4-token prefill then 4 decode steps on the persistent
    kernel (one launch per token)."""
    toks, logits, ref_toks, ref_logits, persistent = run_pair(vk, ctx, orc, CFG_7B, 31, 4, 5, 64)
    assert persistent
    assert_parity(toks, logits, ref_toks, ref_logits)


def test_7b_geometry_decode_at_bench_positions(vk, ctx, orc):
    """Two layers of the 7B geometry decoding at positions 512..515 after a 512-token prefill: the
    attention phase splits each head's 513+ keys over several CTAs as in the benchmark."""
    cfg = dict(CFG_7B, block_count=2, context_length=1024)
    toks, logits, ref_toks, ref_logits, persistent = run_pair(vk, ctx, orc, cfg, 32, 512, 5, 1024)
    assert persistent
    assert_parity(toks, logits, ref_toks, ref_logits)


def test_13b_geometry_decode_parity(vk, ctx, orc):
    """Two layers of the 13B geometry (40 heads, SwiGLU 13824, dim 5120) after a 40-token prefill."""
    cfg = dict(CFG_13B, block_count=2, context_length=512)
    toks, logits, ref_toks, ref_logits, persistent = run_pair(vk, ctx, orc, cfg, 33, 40, 5, 512)
    assert persistent
    assert_parity(toks, logits, ref_toks, ref_logits)
