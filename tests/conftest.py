import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "vkllm.c_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden"),
          ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA path through the C-ABI")


def gpu_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def vk():
    import vkllm_b200

    vkllm_b200.lib()
    return vkllm_b200


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ctx(vk):
    if not gpu_available():
        pytest.skip("no CUDA device")
    c = vk.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory):
    import gen_gguf

    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    weights = gen_gguf.write_gguf(path, gen_gguf.TINY, seed=1234)
    return path, weights
