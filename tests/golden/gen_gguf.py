"""Writes a synthetic LLaMA-2 GGUF (the BASELINE "tiny" config by default) with seeded weights.

Tensor names and metadata keys follow what vkllm.c's loader reads
(src/models/vkllm_models_llama2.c:67-187, 303-387): fp16 linear/embedding weights ~ N(0, std) from
numpy.random.default_rng(seed), f32 RMSNorm gains of 1, llama.vocab_size written explicitly, and a
placeholder tokenizer vocabulary so the reference-style loop can print tokens.

    python tests/golden/gen_gguf.py out.gguf [--seed 1234]
"""
import argparse

import numpy as np

TINY = dict(D=288, L=6, H=6, F=768, V=32000, ctx=256, eps=1e-5, rope_base=10000.0)


def make_weights(cfg, seed, std=0.02):
    rng = np.random.default_rng(seed)
    D, F, V, L = cfg["D"], cfg["F"], cfg["V"], cfg["L"]

    def w(rows, cols):
        return (rng.standard_normal((rows, cols), dtype=np.float32) * std).astype(np.float16)

    out = {"token_embd.weight": w(V, D)}
    for l in range(L):
        out[f"blk.{l}.attn_norm.weight"] = np.ones(D, dtype=np.float32)
        out[f"blk.{l}.ffn_norm.weight"] = np.ones(D, dtype=np.float32)
        out[f"blk.{l}.attn_q.weight"] = w(D, D)
        out[f"blk.{l}.attn_k.weight"] = w(D, D)
        out[f"blk.{l}.attn_v.weight"] = w(D, D)
        out[f"blk.{l}.attn_output.weight"] = w(D, D)
        out[f"blk.{l}.ffn_gate.weight"] = w(F, D)
        out[f"blk.{l}.ffn_up.weight"] = w(F, D)
        out[f"blk.{l}.ffn_down.weight"] = w(D, F)
    out["output_norm.weight"] = np.ones(D, dtype=np.float32)
    out["output.weight"] = w(V, D)
    return out


def write_gguf(path, cfg=TINY, seed=1234, weights=None):
    import gguf

    weights = weights if weights is not None else make_weights(cfg, seed)
    wr = gguf.GGUFWriter(path, "llama")
    wr.add_block_count(cfg["L"])
    wr.add_context_length(cfg["ctx"])
    wr.add_embedding_length(cfg["D"])
    wr.add_feed_forward_length(cfg["F"])
    wr.add_head_count(cfg["H"])
    wr.add_head_count_kv(cfg["H"])
    wr.add_rope_freq_base(cfg["rope_base"])
    wr.add_layer_norm_rms_eps(cfg["eps"])
    wr.add_key_length(cfg["D"] // cfg["H"])
    wr.add_value_length(cfg["D"] // cfg["H"])
    wr.add_uint32("llama.vocab_size", cfg["V"])
    wr.add_bos_token_id(1)
    wr.add_eos_token_id(2)
    wr.add_pad_token_id(0)
    toks = ["<unk>", "<s>", "</s>"] + [f"<t{i}>" for i in range(3, cfg["V"])]
    wr.add_array("tokenizer.ggml.tokens", toks)
    wr.add_array("tokenizer.ggml.scores", [float(-i) for i in range(cfg["V"])])
    for name, arr in weights.items():
        wr.add_tensor(name, arr)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return weights


def prompt(seed, n, vocab=32000):
    """Seeded uniform prompt ids in [3, vocab)."""
    return np.random.default_rng(seed).integers(3, vocab, size=n, dtype=np.uint32)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args()
    write_gguf(a.out, TINY, a.seed)
    print(a.out)
