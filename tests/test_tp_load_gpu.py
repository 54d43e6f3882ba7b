"""B200: load-time tensor-parallel sharding of a GGUF model (vkllm_b200_models_llama2_load_tp). On one
GPU, the model of each rank of 2 (loaded one after the other; no peer exchange is set up) must hold
on the device exactly its shard of every tensor of the tiny GGUF (bit-exact), under the layout of
the random TP models, and a KV cache of head_count / 2 heads."""
import ctypes as C

import numpy as np
import pytest

from test_gguf_shard import split_of

pytestmark = pytest.mark.gpu

FIELDS = (("WQ", "attn_q"), ("WK", "attn_k"), ("WV", "attn_v"), ("WO", "attn_output"), ("WG", "ffn_gate"),
          ("WU", "ffn_up"), ("WD", "ffn_down"), ("attn_norm_weight", "attn_norm"), ("ffn_norm_weight", "ffn_norm"))


def shard(full, name, rank, world):
    if full.ndim == 1:
        return full
    split = split_of(name)
    if split == 1:
        n = full.shape[0] // world
        return full[rank * n:(rank + 1) * n]
    if split == 2:
        n = full.shape[1] // world
        return full[:, rank * n:(rank + 1) * n]
    return full


def test_load_tp_uploads_each_ranks_shard(vk, ctx, tiny_gguf):
    import gen_gguf

    path, weights = tiny_gguf
    world = 2
    for rank in range(world):
        model = vk.Model(ctx).load_tp(path, rank, world)
        try:
            m = model.m
            assert (m.b200.tp_rank, m.b200.tp_size) == (rank, world)
            assert m.meta.head_count == gen_gguf.TINY["H"] and m.meta.block_count == gen_gguf.TINY["L"]

            def check(t, name):
                want = np.ascontiguousarray(shard(weights[name], name, rank, world))
                got = vk.fetch(ctx, t)
                assert got.size == want.size, (name, got.shape, want.shape)
                assert np.array_equal(got.reshape(want.shape).view(np.uint8), want.view(np.uint8)), (name, rank)

            check(m.weights.tok_embed_weights, "token_embd.weight")
            check(m.weights.output_norm_weight, "output_norm.weight")
            check(m.weights.output_weight, "output.weight")
            blocks = C.cast(m.weights.blocks.contents.data, C.POINTER(C.POINTER(vk.BlockWeights)))
            for layer in range(m.meta.block_count):
                bw = blocks[layer].contents
                for field, leaf in FIELDS:
                    check(getattr(bw, field), f"blk.{layer}.{leaf}.weight")
            kv = C.cast(m.weights.kvcache, C.POINTER(vk.KVCache)).contents
            hd = gen_gguf.TINY["D"] // gen_gguf.TINY["H"]
            assert tuple(kv.kcache_shape) == (1, gen_gguf.TINY["H"] // world, gen_gguf.TINY["ctx"], hd)
        finally:
            model.free()
