"""CPU: the GGUF reader behind vkllm_models_llama2_load / load_tp refuses malformed files with
VKLLM_ERR_ARGS instead of reading past the mapping or allocating without bound. A hand-built minimal
GGUF (one fp16 tensor) reads back exactly; each corruption of it is refused. The reader is reached
through the host-only vkllm_b200_gguf_read_shard."""
import ctypes as C
import struct

import numpy as np
import pytest

F16, F32 = 1, 0
ARR, STR, U32 = 9, 8, 4


def gstr(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def kv_u32(key, v):
    return gstr(key) + struct.pack("<II", U32, v)


def kv_arr(key, elem_type, count, payload=b""):
    return gstr(key) + struct.pack("<IIQ", ARR, elem_type, count) + payload


def desc(name, dims, typ=F16, off=0):
    return gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", typ, off)


def mini(kvs=(), descs=None, data=None, version=3, n_tensors=None, n_kv=None, align=32, magic=b"GGUF"):
    vals = np.arange(32, dtype=np.float16)
    descs = [desc("token_embd.weight", [8, 4])] if descs is None else descs
    data = vals.tobytes() if data is None else data
    head = magic + struct.pack("<IQQ", version, len(descs) if n_tensors is None else n_tensors,
                               len(kvs) if n_kv is None else n_kv)
    body = head + b"".join(kvs) + b"".join(descs)
    return body + b"\0" * ((-len(body)) % align) + data


def read(vk, path, name="token_embd.weight"):
    out = np.zeros(64, dtype=np.float16)
    shape = (C.c_uint32 * 2)()
    rc = vk.lib().vkllm_b200_gguf_read_shard(str(path).encode(), name.encode(), 0, 1, out.ctypes.data, out.nbytes,
                                              shape)
    return rc, (shape[0], shape[1]), out


def test_minimal_file_reads_back(vk, tmp_path):
    p = tmp_path / "ok.gguf"
    p.write_bytes(mini(kvs=[kv_u32("general.alignment", 64)], align=64))
    rc, shape, out = read(vk, p)
    assert rc == vk.OK and shape == (4, 8)
    assert np.array_equal(out[:32], np.arange(32, dtype=np.float16))


BAD = {
    "too_small": lambda: b"GGUF\x03\x00",
    "bad_magic": lambda: mini(magic=b"GGUX"),
    "version_1": lambda: mini(version=1),
    "version_4": lambda: mini(version=4),
    "huge_kv_count": lambda: mini(n_kv=1 << 40),
    "more_kvs_than_bytes": lambda: mini(n_kv=3),
    "huge_key_length": lambda: mini(kvs=[struct.pack("<Q", 1 << 62) + b"k"]),
    "huge_string_array": lambda: mini(kvs=[kv_arr("tokenizer.ggml.tokens", STR, 1 << 40)]),
    "huge_u32_array": lambda: mini(kvs=[kv_arr("tokenizer.ggml.scores", U32, 1 << 40)]),
    "nested_array": lambda: mini(kvs=[kv_arr("x", ARR, 1)]),
    "unknown_value_type": lambda: mini(kvs=[gstr("x") + struct.pack("<I", 77)]),
    "alignment_not_multiple_of_8": lambda: mini(kvs=[kv_u32("general.alignment", 12)], align=12),
    "alignment_huge": lambda: mini(kvs=[kv_u32("general.alignment", 1 << 30)]),
    "five_dims": lambda: mini(descs=[desc("token_embd.weight", [2, 2, 2, 2, 2])]),
    "dims_overflow": lambda: mini(descs=[desc("token_embd.weight", [1 << 33, 1 << 33])]),
    "dims_past_file": lambda: mini(descs=[desc("token_embd.weight", [1 << 31, 1 << 31])]),
    "offset_wraps": lambda: mini(descs=[desc("token_embd.weight", [8, 4], off=(1 << 64) - 16)]),
    "offset_past_end": lambda: mini(descs=[desc("token_embd.weight", [8, 4], off=1 << 20)]),
    "data_truncated": lambda: mini()[:-2],
    "more_tensors_than_described": lambda: mini(n_tensors=2),
}


@pytest.mark.parametrize("case", list(BAD))
def test_malformed_file_is_refused(vk, tmp_path, case):
    p = tmp_path / f"{case}.gguf"
    p.write_bytes(BAD[case]())
    rc, _, _ = read(vk, p)
    assert rc == vk.ARGS, case
