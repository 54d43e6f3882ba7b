"""The C-ABI library: builds, loads without a GPU, exports every function include/*.h declares,
and its public struct layouts match the ctypes mirrors."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"\b(vkllm_[a-z0-9_]+)\s*\(", src):
            name = m.group(1)
            # skip macro-generated inline array helpers and the logger macros
            if name.startswith("vkllm_array_") or name.endswith("_t") or name in ("vkllm_fp16_to_fp32", "vkllm_fp32_to_fp16"):
                continue
            names.add(name)
    return names


def test_library_exports_every_declared_symbol(vk):
    lib = vk.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", vk.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = sorted(n for n in declared_functions() if n not in exported)
    assert not missing, f"declared but not exported: {missing}"
    for n in declared_functions():
        getattr(lib, n)


def test_binding_covers_exports(vk):
    declared = declared_functions()
    for n in vk.EXPORTED:
        assert n in declared, n


def test_error_and_enum_strings(vk):
    lib = vk.lib()
    assert lib.vkllm_err_s(1) == b"VKLLM_ERR_OK"
    assert lib.vkllm_err_s(6) == b"VKLLM_ERR_ARGS"
    assert lib.vkllm_dtype_s(2) == b"float16"
    assert lib.vkllm_op_s(5) == b"VKLLM_OP_MATMUL"
    assert lib.vkllm_op_s(11) == b"VKLLM_OP_REF"


def test_dtype_info(vk):
    class Info(C.Structure):
        _fields_ = [("dtype", C.c_int), ("bytes", C.c_uint32), ("ipb", C.c_uint32), ("bpb", C.c_uint32)]

    lib = vk.lib()
    for dt, b in ((1, 4), (2, 2), (3, 1), (4, 4)):
        i = Info()
        assert lib.vkllm_get_dtype_info(dt, C.byref(i)) == vk.OK
        assert i.bytes == b
    assert lib.vkllm_get_dtype_info(9, C.byref(Info())) == vk.ARGS


@pytest.mark.parametrize("name,mirror", [("vkllm_tensor", "Tensor"), ("vkllm_graph", "Graph"),
                                         ("vkllm_models_llama2", "Llama2"), ("vkllm_kvcache", "KVCache"),
                                         ("block_weights", "BlockWeights")])
def test_struct_layouts(vk, name, mirror):
    lib = vk.lib()
    size = lib.vkllm_b200_sizeof(name.encode())
    assert size == C.sizeof(getattr(vk, mirror)), name
    if name == "vkllm_tensor":
        for f in ("name", "dtype", "shapes", "strides", "bytes", "data", "op", "pipeline", "srcs"):
            assert lib.vkllm_b200_offsetof(b"vkllm_tensor", f.encode()) == getattr(vk.Tensor, f).offset, f
        assert lib.vkllm_b200_offsetof(b"vkllm_tensor", b"params") == C.sizeof(vk.Tensor)


def test_context_without_gpu_reports_no_device(vk):
    from conftest import gpu_available

    if gpu_available():
        pytest.skip("a GPU is present")
    p = C.c_void_p()
    assert vk.lib().vkllm_context_new(0, C.byref(p)) == vk.DEV_NOT_FOUND


def test_hashmap(vk):
    lib = vk.lib()
    m = C.c_void_p()
    assert lib.vkllm_hashmap_new(C.byref(m), 4) == vk.OK
    for i in range(100):
        assert lib.vkllm_hashmap_insert(m, f"node.{i}".encode(), i * 7) == vk.OK
    v = C.c_uint64()
    assert lib.vkllm_hashmap_get(m, b"node.42", C.byref(v)) and v.value == 294
    assert lib.vkllm_hashmap_remove(m, b"node.42") == vk.OK
    assert not lib.vkllm_hashmap_get(m, b"node.42", C.byref(v))
    assert lib.vkllm_hashmap_size(m) == 99
    lib.vkllm_hashmap_free(m)


def test_random_generator_host_twin_matches_oracle(vk, orc):
    import numpy as np

    a = vk.random_f16_host(1234, 5, 0.02, 1000, 4096)
    b = orc.random_f16(1234, 5, 0.02, 1000, 4096).view(np.uint16)
    assert np.array_equal(a, b)
    f = a.view(np.float16).astype(np.float32)
    assert abs(f.mean()) < 2e-3 and 0.017 < f.std() < 0.023
