import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-infer-llama.cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_DIR = os.environ.get("MI_B200_MODEL_DIR", "/tmp/mi_b200_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libmi_cuda.so")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def bits(a) -> np.ndarray:
    """uint32 view for bit-exact float comparison."""
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(scope="session")
def model_path():
    """Path of a seeded random-init Qwen2 GGUF of the given shape (cached)."""
    import mi_gguf

    def make(shape_name: str, seed: int, fast: bool = False) -> str:
        shape = getattr(mi_gguf, shape_name)
        tag = "_fast" if fast else ""
        path = os.path.join(MODEL_DIR, f"{shape_name.lower()}_seed{seed}{tag}.gguf")
        return mi_gguf.ensure_qwen2_gguf(path, shape, seed, fast=fast)

    return make


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import mi_cuda
    mi_cuda.init(0)
    return torch
