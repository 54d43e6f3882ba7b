"""Shared checks of greedy decoding against the CPU oracle (imported by the GPU parity tests).

Greedy tokens: identical step by step. The one exception is a step where the reference's own top
two fp16 logits are within one fp16 ulp of each other (a tie at fp16 resolution): a different fp32
summation order, which any implementation other than the reference shader itself has, can break
it either way. Such a step is reported as a warning with both tokens' logits, and the comparison
stops there because the inputs of later steps differ.

Logits: within max-abs `max_bar` and mean-abs `mean_bar` at every compared step."""
import warnings

import numpy as np


def ulp16(v):
    """Spacing of fp16 numbers at |v| (normal range)."""
    return float(2.0 ** (np.floor(np.log2(max(abs(float(v)), 2.0 ** -14))) - 10))


def compare_greedy(toks, logits, ref_toks, ref_logits, max_bar, mean_bar, what=""):
    """Returns the number of steps compared. `max_bar` / `mean_bar` are floats or per-step lists."""
    n = min(len(toks), len(ref_toks))
    for i in range(n):
        mb = max_bar[i] if isinstance(max_bar, (list, tuple, np.ndarray)) else max_bar
        ab = mean_bar[i] if isinstance(mean_bar, (list, tuple, np.ndarray)) else mean_bar
        r = np.asarray(ref_logits[i], dtype=np.float32)
        d = np.abs(np.asarray(logits[i], dtype=np.float32) - r)
        assert d.max() <= mb and d.mean() <= ab, (f"{what} step {i}: max-abs {d.max():.5f} (bar {mb:.5f}), "
                                                  f"mean-abs {d.mean():.6f} (bar {ab:.6f})")
        if toks[i] != ref_toks[i]:
            top = float(r[ref_toks[i]])
            ours = float(r[toks[i]])
            gap = top - ours
            msg = (f"{what} step {i}: token {toks[i]} vs reference {ref_toks[i]}; reference logits {top} (its "
                   f"choice) / {ours} (ours), gap {gap:.6g} = {gap / ulp16(top):.2f} fp16 ulp; our logits "
                   f"{float(logits[i][ref_toks[i]])} / {float(logits[i][toks[i]])}")
            assert gap <= ulp16(top), "not a tie at fp16 resolution: " + msg
            warnings.warn("greedy divergence at a reference tie: " + msg)
            return i + 1
    return n


def download_weights(vk, ctx, model, cfg):
    """A random-initialised model's weights as the oracle's GGUF-named numpy arrays."""
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
