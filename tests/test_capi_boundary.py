"""The C-ABI library: loads without a GPU, exports every symbol include/*.h
declares, and rejects bad arguments with a status code and a message (the
reference aborts or asserts in the same places; a library must not)."""
import ctypes as C
import glob
import os
import re

import pytest

import mi_cuda
from conftest import ROOT


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        names |= set(re.findall(r"\b(mi_cuda_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(mi_cuda.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 39
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_symbols()) == set(mi_cuda._SIGS)


def test_pure_host_entry_points_without_gpu():
    L = mi_cuda.lib()
    assert L.mi_cuda_q8_0_packed_bytes(896, 896) == 896 * 896 * 34 // 32
    assert L.mi_cuda_q8_0_packed_bytes(896, 4) == 8 * 896 * 34 // 32  # rows padded to 8
    assert L.mi_cuda_q8_0_packed_bytes(33, 4) == 0
    assert L.mi_cuda_attention_decode_scratch_bytes(14, 128) == 14 * 128 * 4
    # split mode: 32768 positions over 2 KV heads -> 256 splits of 128 positions,
    # each (maximum, denominator, 64 value sums) per query head
    assert L.mi_cuda_attention_decode_split_scratch_bytes(14, 2, 32768, 64) == 14 * 256 * 66 * 4
    assert L.mi_cuda_attention_decode_split_scratch_bytes(14, 2, 1, 64) == 14 * 1 * 66 * 4
    assert L.mi_cuda_attention_decode_split_scratch_bytes(0, 2, 1, 64) == 0
    import numpy as np
    logits = np.array([1.0, 3.0, 3.0, -1.0], dtype=np.float32)
    assert mi_cuda.sample_greedy(logits) == 1  # first index of the maximum


def test_errors_are_status_codes_not_aborts():
    L = mi_cuda.lib()
    # Null arguments are rejected before any device work.
    rc = L.mi_cuda_qwen2_model_load(None, 0, None)
    assert rc == mi_cuda.ERR_ARG
    assert b"null" in L.mi_cuda_last_error()
    rc = L.mi_cuda_kv_cache_init(None, 16, None)
    assert rc == mi_cuda.ERR_ARG
    # the fast-mode switch: no KV cache, or a value other than 0 / 1
    assert L.mi_cuda_qwen2_set_fast_mode(None, 1) == mi_cuda.ERR_ARG
    assert L.mi_cuda_qwen2_fast_mode(None) == 0


def test_device_required_for_compute():
    import torch
    if torch.cuda.is_available():
        pytest.skip("this check is for machines without a GPU")
    L = mi_cuda.lib()
    assert L.mi_cuda_init(0) == mi_cuda.ERR_CUDA
    assert L.mi_cuda_last_error() != b""
