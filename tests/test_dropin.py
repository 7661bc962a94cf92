"""The drop-in boundary: the reference's own model code with the ops_cuda
backend plugged under its executor (mini-infer-llama.cpp_b200/integration).

libmi_ref_cuda.so is the reference's sources compiled unchanged -- GGUF
load, graph build, gallocr reserve and per-step plan, mi_kv_cache_init,
mi_qwen2_forward -- linked with ops_cuda, whose executor takes over
mi_graph_compute (src/graph.cpp:75-83) once a backend is attached: gallocr's
arena becomes one device allocation used at the planned offsets, the weights
and the KV cache live in HBM, and every step's exec nodes run as one
recorded CUDA graph of the backend's per-op calls. The GPU tests compare the
logits of that path with the reference's own CPU run (the separately built
oracle/_ref/libmi_ref.so) bit for bit, prompt and 20+ decode steps.
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import PKG, bits

LIB = os.path.join(PKG, "lib", "libmi_ref_cuda.so")
STATS = ("steps", "nodes", "views_skipped", "arena_bytes", "arena_tensors", "instantiations", "updates",
         "weight_bytes")


def _lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is missing: build it with `make -C mini-infer-llama.cpp_b200/integration "
                    "REF=<reference tree>` (the build entry point does this when the reference is present)")
    L = C.CDLL(LIB)
    L.mirc_open.restype = C.c_void_p
    L.mirc_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
    L.mirc_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    L.mirc_n_vocab.argtypes = [C.c_void_p]
    L.mirc_arena_size.argtypes = [C.c_void_p]
    L.mirc_arena_size.restype = C.c_int64
    L.mirc_stats.argtypes = [C.c_void_p]
    L.mirc_close.argtypes = [C.c_void_p]
    L.mirc_last_error.restype = C.c_char_p
    return L


class Session:
    """mi_qwen2_model_load + mi_kv_cache_init (+ mi_ops_cuda_attach when
    device >= 0) through the drop-in library; forward = mi_qwen2_forward."""

    def __init__(self, L, path, n_ctx, device, n_threads=1):
        self.L = L
        err = C.create_string_buffer(512)
        self.h = L.mirc_open(path.encode(), n_ctx, n_threads, device, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self.n_vocab = L.mirc_n_vocab(self.h)

    def forward(self, tokens, n_past, last_logits_only=False):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((1 if last_logits_only else t.size, self.n_vocab), dtype=np.float32)
        self.L.mirc_forward(self.h, t.ctypes.data, t.size, n_past, int(last_logits_only), out.ctypes.data)
        return out

    @property
    def arena_size(self):
        return int(self.L.mirc_arena_size(self.h))

    def stats(self):
        v = (C.c_int64 * 8)()
        self.L.mirc_stats(v)
        return dict(zip(STATS, list(v)))

    def close(self):
        if self.h:
            self.L.mirc_close(self.h)
            self.h = None


def test_dropin_library_exports_and_cpu_passthrough(model_path):
    """Without an attached backend the wrapped executor is the reference's own
    threadpool walk: the library's CPU forward equals the reference's."""
    import mi_oracle
    L = _lib()
    for name in ("mirc_open", "mirc_forward", "mirc_stats", "mirc_close", "mirc_arena_size",
                 "__wrap__Z16mi_graph_computeP9mi_cgraphP13mi_threadpool"):
        assert hasattr(L, name), name
    path = model_path("TINY", 1)
    s = Session(L, path, 64, device=-1)
    ref = mi_oracle.ReferenceModel(path, n_ctx=64)
    prompt = np.array([5, 7, 9, 200], dtype=np.int32)
    assert np.array_equal(bits(s.forward(prompt, 0)), bits(ref.forward(prompt, 0)))
    assert s.stats()["steps"] == 0  # nothing ran on a device
    s.close()
    ref.close()


@pytest.mark.gpu
@pytest.mark.parametrize("shape,seed,n_ctx", [("TINY", 1, 64), ("SMALL", 4, 256)])
def test_reference_graph_on_device_bitexact(torch_cuda, model_path, shape, seed, n_ctx):
    """The reference's graph and gallocr plan, executed by the device backend:
    prompt logits and 24 decode steps bit-identical to the reference's CPU
    forward; one device arena of exactly gallocr's reserved size; decode steps
    replay one executable CUDA graph updated in place."""
    import mi_oracle
    L = _lib()
    path = model_path(shape, seed)
    dev = Session(L, path, n_ctx, device=0)
    ref = mi_oracle.ReferenceModel(path, n_ctx=n_ctx)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, ref.n_vocab, 9).astype(np.int32)
    want = ref.forward(prompt, 0)
    got = dev.forward(prompt, 0)
    assert np.array_equal(bits(got), bits(want))
    st0 = dev.stats()
    assert st0["arena_bytes"] == dev.arena_size > 0
    assert st0["arena_tensors"] > 0 and st0["views_skipped"] > 0
    tok = int(np.argmax(want[-1]))
    n_steps = 24
    for step in range(n_steps):
        w = ref.forward([tok], prompt.size + step)
        g = dev.forward([tok], prompt.size + step)
        assert np.array_equal(bits(g), bits(w)), f"decode step {step}"
        tok = int(np.argmax(w[0]))
    st = dev.stats()
    assert st["steps"] == 1 + n_steps
    # every decode step records the same kernels: the executable graph is
    # updated, not re-instantiated
    assert st["instantiations"] <= 3 and st["updates"] >= n_steps - 2
    dev.close()
    ref.close()


@pytest.mark.gpu
def test_reference_graph_on_device_last_logits_and_generation(torch_cuda, model_path):
    """last_logits_only (the lm_head over a view of the last column) and a
    greedy generation through the drop-in path equal the reference's."""
    import mi_oracle
    L = _lib()
    path = model_path("SMALL", 5)
    dev = Session(L, path, 128, device=0)
    ref = mi_oracle.ReferenceModel(path, n_ctx=128)
    prompt = np.random.default_rng(3).integers(0, ref.n_vocab, 17).astype(np.int32)
    got = dev.forward(prompt, 0, last_logits_only=True)
    want_tok, _, _ = ref.generate(prompt, 24)
    assert int(np.argmax(got[0])) == want_tok[0]
    toks = [int(np.argmax(got[0]))]
    for i in range(23):
        toks.append(int(np.argmax(dev.forward([toks[-1]], prompt.size + i)[0])))
    assert np.array_equal(np.array(toks, dtype=np.int32), want_tok)
    dev.close()
    ref.close()
