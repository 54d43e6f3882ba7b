"""CPU: load-time tensor-parallel sharding of a GGUF model (host side of
vkllm_b200_models_llama2_load_tp). For every tensor of the tiny synthetic GGUF, the shard that
vkllm_b200_gguf_read_shard extracts for each rank must be the rank's slice of the unsharded matrix
under the layout the random TP models use (rows of Wq/Wk/Wv/Wgate/Wup/output, columns of
Wo/Wdown, the embedding and norm gains whole), and the shards of all ranks must tile the matrix."""
import ctypes as C

import numpy as np
import pytest

ROWS = ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up")
COLS = ("attn_output", "ffn_down")


def split_of(name):
    if name == "output.weight":
        return 1
    if name.startswith("blk."):
        leaf = name.split(".")[2]
        if leaf in ROWS:
            return 1
        if leaf in COLS:
            return 2
    return 0


def read_shard(vk, path, name, rank, world, ref):
    shape = (C.c_uint32 * 2)()
    out = np.empty(ref.size, dtype=ref.dtype)
    rc = vk.lib().vkllm_b200_gguf_read_shard(path.encode(), name.encode(), rank, world, out.ctypes.data,
                                              out.nbytes, shape)
    return rc, (shape[0], shape[1]), out


@pytest.mark.parametrize("world", [2, 3])
def test_shards_are_the_ranks_slices_and_tile_each_tensor(vk, tiny_gguf, world):
    path, weights = tiny_gguf
    for name, full in weights.items():
        full2 = full.reshape(1, -1) if full.ndim == 1 else full
        split = split_of(name) if full.ndim == 2 else 0
        dim = full2.shape[0] if split == 1 else full2.shape[1] if split == 2 else 0
        if split and dim % world:
            # the split does not divide this tensor (vocab 32000 over 3 ranks): refused
            rc, _, _ = read_shard(vk, path, name, 0, world, full2)
            assert rc == vk.ARGS, name
            continue
        parts = []
        for rank in range(world):
            rc, shape, out = read_shard(vk, path, name, rank, world, full2)
            assert rc == vk.OK, (name, rank)
            if split == 1:
                n = full2.shape[0] // world
                want = full2[rank * n:(rank + 1) * n]
            elif split == 2:
                n = full2.shape[1] // world
                want = full2[:, rank * n:(rank + 1) * n]
            else:
                want = full2
            assert shape == want.shape, (name, rank, shape, want.shape)
            got = out[:want.size].reshape(want.shape)
            assert np.array_equal(got.view(np.uint8), np.ascontiguousarray(want).view(np.uint8)), (name, rank)
            parts.append(got)
        if split:
            assert np.array_equal(np.concatenate(parts, axis=split - 1), full2), name


def test_shard_shape_query_and_bad_arguments(vk, tiny_gguf):
    path, weights = tiny_gguf
    lib = vk.lib()
    shape = (C.c_uint32 * 2)()
    assert lib.vkllm_b200_gguf_read_shard(path.encode(), b"blk.0.ffn_down.weight", 1, 2, None, 0, shape) == vk.OK
    D, F = weights["blk.0.ffn_down.weight"].shape
    assert (shape[0], shape[1]) == (D, F // 2)
    small = np.empty(4, dtype=np.float16)
    assert lib.vkllm_b200_gguf_read_shard(path.encode(), b"blk.0.ffn_down.weight", 0, 2, small.ctypes.data,
                                          small.nbytes, shape) == vk.ARGS
    assert lib.vkllm_b200_gguf_read_shard(path.encode(), b"no.such.tensor", 0, 2, None, 0, shape) == vk.ARGS
    assert lib.vkllm_b200_gguf_read_shard(path.encode(), b"output.weight", 2, 2, None, 0, shape) == vk.ARGS
