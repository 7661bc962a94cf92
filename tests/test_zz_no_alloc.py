"""The allocation-free decode-attention entry point.

mi_cuda_attention_decode_noalloc serves callers that may not allocate device
memory on their call path (a runtime that allocates nothing after start-up, a
caller recording its own CUDA graph, a plugin host that owns all device memory):
it takes only inputs and outputs and keeps its score scratch in a fixed 4 MiB
array inside the library. This test calls it through the C-ABI several times in a
row with n_kv above 8192 (up to 8192 positions the kernel keeps its scores in
shared memory and never touches the scratch array), so every call goes through
the library's array and the later calls run over the earlier calls' leftover
contents; each result is checked bit for bit against the existing caller-scratch
entry point (zero tolerance, as every parity test here). The largest size the
array allows is one of the calls. It also checks the size limit and argument
errors. The file sorts last so a run that stops at the first
failure has run every other test before it; it passes alone in a fresh process
too (it only needs mi_cuda_init, which the torch_cuda fixture calls).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import bits


def _inputs(n_kv, seed, H=14, HKV=2, D=64):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((H, D), dtype=np.float32),
            rng.standard_normal((n_kv, HKV, D), dtype=np.float32),
            rng.standard_normal((n_kv, HKV, D), dtype=np.float32))


@pytest.mark.gpu
def test_noalloc_attention_matches_caller_scratch_entry_point(torch_cuda):
    import mi_cuda
    torch = torch_cuda
    lib = mi_cuda.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # calls in a row through the static scratch: larger, smaller, then the
    # largest n_kv whose 14 score rows fit the 1,048,576-float array
    for n_kv, seed in ((20000, 1), (9000, 2), ((1 << 20) // 14, 3)):
        q, k, v = (torch.from_numpy(a).cuda() for a in _inputs(n_kv, seed))
        want = mi_cuda.attention_decode(q, k, v, 2, n_kv, 0.125).cpu().numpy()
        out = torch.empty((14, 64), dtype=torch.float32, device="cuda")
        rc = lib.mi_cuda_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 64, 14, 2,
                                                  n_kv, C.c_float(0.125), out.data_ptr(), stream)
        assert rc == mi_cuda.OK, lib.mi_cuda_last_error()
        torch.cuda.synchronize()
        assert np.array_equal(bits(out.cpu().numpy()), bits(want))


@pytest.mark.gpu
def test_noalloc_attention_rejects_sizes_beyond_its_scratch(torch_cuda):
    import mi_cuda
    torch = torch_cuda
    lib = mi_cuda.lib()
    q = torch.zeros((14, 64), dtype=torch.float32, device="cuda")
    kv = torch.zeros((8, 2, 64), dtype=torch.float32, device="cuda")
    n_kv = (1 << 20) // 14 + 1  # 14 * n_kv > 1,048,576
    rc = lib.mi_cuda_attention_decode_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), 64, 14, 2,
                                              n_kv, C.c_float(0.125), q.data_ptr(), None)
    assert rc == mi_cuda.ERR_ARG
    assert b"exceeds the static scratch" in lib.mi_cuda_last_error()


def test_noalloc_attention_rejects_bad_head_counts():
    """Argument errors come back as MI_CUDA_ERR_ARG before any device work (no GPU
    needed): a zero or negative head count would otherwise reach the launch."""
    import mi_cuda
    lib = mi_cuda.lib()
    fake = 256  # never dereferenced: the arguments are rejected first
    for n_head, n_head_kv in ((0, 2), (-2, 2), (14, 0), (14, 3)):
        rc = lib.mi_cuda_attention_decode_noalloc(fake, fake, fake, 64, n_head, n_head_kv, 128,
                                                  C.c_float(0.125), fake, None)
        assert rc == mi_cuda.ERR_ARG, (n_head, n_head_kv)
