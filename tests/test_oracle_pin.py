"""Pins the CPU oracle restatement (oracle/mi_oracle.c) to the reference.

Two kinds of evidence, both on the CPU:
  * the reference's own code, compiled from its sources into
    oracle/_ref/libmi_ref.so, run on the same seeded inputs: bit-exact;
  * the known-answer cases of the reference's tests (tests/test_quant.cpp,
    tests/test_ops_cpu.cpp), restated here.
"""
import math

import numpy as np
import pytest

import mi_gguf
import mi_oracle
from conftest import bits


@pytest.fixture(scope="module")
def R():
    return mi_oracle.Reference()


@pytest.fixture(scope="module")
def S():
    return mi_oracle.Restatement()


def q8_rows(rng, n, k, std=0.02):
    return mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)).view(np.uint8)


# ---- known answers (reference tests/test_quant.cpp) ------------------------

def test_fp16_known_values(S):
    # test_quant.cpp:59-83
    cases = {0x0000: 0.0, 0x8000: -0.0, 0x3C00: 1.0, 0xBC00: -1.0, 0x4000: 2.0, 0x3800: 0.5,
             0x4200: 3.0, 0x0001: 5.9604645e-8, 0x03FF: 6.09755516e-5}
    for h, v in cases.items():
        got = S.lib.mio_fp16_to_fp32(h)
        assert got == np.float32(v)
    assert math.isinf(S.lib.mio_fp16_to_fp32(0x7C00))
    assert math.isnan(S.lib.mio_fp16_to_fp32(0x7E00))


def test_fp16_conversion_matches_reference_all_halves(R, S):
    for h in range(0, 65536, 7):
        a, b = R.lib.mi_ref_fp16_to_fp32(h), S.lib.mio_fp16_to_fp32(h)
        assert (math.isnan(a) and math.isnan(b)) or np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_block_isum_boundaries(R, S):
    # test_quant.cpp:164-198: +-127, zeros, alternating, and random blocks
    full = lambda v: np.full(32, v, dtype=np.int8)
    mixed = np.array([127 if j % 2 == 0 else -127 for j in range(32)], dtype=np.int8)
    pairs = [(full(127), full(127)), (full(127), full(-127)), (full(-127), full(-127)),
             (full(0), full(0)), (full(0), full(127)), (mixed, full(127)), (mixed, mixed)]
    rng = np.random.default_rng(123)
    for _ in range(200):
        pairs.append((rng.integers(-127, 128, 32).astype(np.int8), rng.integers(-127, 128, 32).astype(np.int8)))
    for x, y in pairs:
        want = int(np.dot(x.astype(np.int64), y.astype(np.int64)))
        assert R.lib.mi_ref_block_isum_scalar(x.ctypes.data, y.ctypes.data) == want
        assert R.lib.mi_ref_block_isum_avx2(x.ctypes.data, y.ctypes.data) == want
        assert S.lib.mio_block_isum(x.ctypes.data, y.ctypes.data) == want
        assert int(S.block_lanes(x, y).sum()) == want
    assert int(np.dot(full(127).astype(np.int64), full(127).astype(np.int64))) == 516128


def test_quantize_all_zero_block(R, S):
    # test_quant.cpp:144-162: an all-zero block has d = 0 and q = 0
    x = np.zeros(32, dtype=np.float32)
    a, b = R.quantize_act(x), S.quantize_act(x)
    assert np.array_equal(a, b)
    assert np.all(a == 0)


def test_q8_0_act_layout_and_qs_match_q8_0(R):
    # test_quant.cpp:228-264: 36-byte blocks, qs identical to the Q8_0 quantizer's
    rng = np.random.default_rng(999)
    x = rng.uniform(-5, 5, 32 * 6).astype(np.float32)
    act = R.quantize_act(x).reshape(6, 36)
    q8 = mi_gguf.quantize_q8_0(x.reshape(1, -1)).reshape(-1)
    assert np.array_equal(act[:, 4:].view(np.int8), q8["qs"])


# ---- bit-exact against the compiled reference -------------------------------

@pytest.mark.parametrize("k", [32, 64, 896, 4864])
def test_quantize_act_bitexact(R, S, k):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal((3, k)) * rng.uniform(0.01, 10)).astype(np.float32)
    x[0, :32] = 0.0
    assert np.array_equal(R.quantize_act(x), S.quantize_act(x))


def test_numpy_weight_quantizer_matches_reference(R):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(896 * 4, dtype=np.float32) * np.float32(0.02)
    ref = np.empty(896 * 4 // 32 * 34, dtype=np.uint8)
    R.lib.mi_ref_quantize_row_q8_0(x.ctypes.data, ref.ctypes.data, x.size)
    assert np.array_equal(ref, mi_gguf.quantize_q8_0(x.reshape(1, -1)).view(np.uint8).reshape(-1))


@pytest.mark.parametrize("n,k", [(896, 896), (128, 896), (512, 4864), (64, 64)])
def test_mul_mat_bitexact(R, S, n, k):
    rng = np.random.default_rng(n * 7 + k)
    w = q8_rows(rng, n, k)
    x = rng.standard_normal((2, k), dtype=np.float32)
    act, out = R.mul_mat(w, k, n, x)
    assert np.array_equal(act, S.quantize_act(x))
    assert np.array_equal(bits(out), bits(S.mul_mat(w, k, n, act, 2)))


def test_vec_dot_avx2_vs_scalar_within_reference_tolerance(R, S):
    # test_quant.cpp:266-290: the scalar and AVX2 orders agree within 1e-5
    rng = np.random.default_rng(4242)
    w = q8_rows(rng, 1, 256, std=1.0)
    a = S.quantize_act(rng.uniform(-2, 2, 256).astype(np.float32))
    r_avx = R.lib.mi_ref_vec_dot_q8_0_wact(w.ctypes.data, a.ctypes.data, 256)
    r_sc = R.lib.mi_ref_vec_dot_q8_0_wact_scalar(w.ctypes.data, a.ctypes.data, 256)
    assert np.float32(S.lib.mio_vec_dot_q8_0_wact(w.ctypes.data, a.ctypes.data, 256)) == np.float32(r_avx)
    assert np.float32(S.lib.mio_vec_dot_q8_0_wact_scalar(w.ctypes.data, a.ctypes.data, 256)) == np.float32(r_sc)
    assert abs(r_avx - r_sc) / max(abs(r_sc), 1e-6) < 1e-5


def test_rms_norm_known_and_bitexact(R, S):
    # test_ops_cpu.cpp:65-83: [1, 2, 3, 4] with eps 1e-6
    x = np.array([[1, 2, 3, 4]], dtype=np.float32)
    y = S.rms_norm(x, 1e-6)
    inv = 1.0 / math.sqrt(30.0 / 4 + 1e-6)
    assert np.allclose(y, x * inv, rtol=1e-6)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 896), dtype=np.float32)
    assert np.array_equal(bits(R.op("rms_norm", x, params=(1e-6,))), bits(S.rms_norm(x, 1e-6)))


def test_rope_identity_at_pos0_and_bitexact(R, S):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, 2, 64), dtype=np.float32)
    assert np.array_equal(S.rope(x, 0, 64, 1e6), x)
    x = rng.standard_normal((3, 14, 64), dtype=np.float32)
    for n_past in (0, 1, 37, 2047):
        ref = R.op("rope", x, params=(n_past, 64, 1e6))
        assert np.array_equal(bits(ref), bits(S.rope(x, n_past, 64, 1e6)))


def test_silu_and_softmax_bitexact(R, S):
    rng = np.random.default_rng(17)
    x = (rng.standard_normal(4864) * 4).astype(np.float32)
    assert np.array_equal(bits(R.op("silu", x)), bits(S.silu(x)))
    s = (rng.standard_normal((14, 3, 40)) * 5).astype(np.float32)
    ref = R.op("softmax", s, params=(37, 0.125))
    got = np.empty_like(s)
    S.lib.mio_softmax(s.ctypes.data, 40, 3, 14, 37, 0.125, got.ctypes.data)
    assert np.array_equal(bits(ref), bits(got))
    # causal mask (test_ops_cpu.cpp:181-241): row j sees columns [0, n_past + j]
    assert np.all(got[:, 0, 38:] == 0) and np.all(got[:, 1, 39:] == 0) and np.all(got[:, 2, :] > 0)


@pytest.mark.parametrize("n_kv,n_tokens", [(128, 1), (37, 5), (1024, 1)])
def test_attention_bitexact(R, S, n_kv, n_tokens):
    rng = np.random.default_rng(n_kv)
    H, HKV, D = 14, 2, 64
    n_ctx = n_kv + 3
    q = rng.standard_normal((n_tokens, H, D), dtype=np.float32)
    k = rng.standard_normal((n_ctx, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_ctx, HKV, D), dtype=np.float32)
    n_past = n_kv - n_tokens
    a = R.attention(q, k, v, HKV, n_past, n_tokens, 0.125)
    b = S.attention(q, k, v, HKV, n_past, n_tokens, 0.125)
    for x, y in zip(a, b):
        assert np.array_equal(bits(x), bits(y))


def test_tiny_model_forward_bitexact(model_path):
    import mi_gguf as G
    path = model_path("TINY", 1)
    ref = mi_oracle.ReferenceModel(path, n_ctx=64)
    rs = mi_oracle.RestatedModel(G.GGUFFile(path), n_ctx=64)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 256, 8).astype(np.int32)
    a, b = ref.forward(prompt, 0), rs.forward(prompt, 0)
    assert np.array_equal(bits(a), bits(b))
    tok = int(np.argmax(a[-1]))
    for step in range(12):
        a, b = ref.forward([tok], 8 + step), rs.forward([tok], 8 + step)
        assert np.array_equal(bits(a), bits(b))
        assert mi_oracle.Reference().lib.mi_ref_sample_greedy(a.ctypes.data, a.shape[1]) == int(np.argmax(a[0]))
        tok = int(np.argmax(a[0]))


def test_batch_prefill_equals_incremental(model_path):
    # test_model_qwen2.cpp:186-288: batched prefill == token-by-token decode
    path = model_path("TINY", 2)
    ref_b = mi_oracle.ReferenceModel(path, n_ctx=64)
    ref_i = mi_oracle.ReferenceModel(path, n_ctx=64)
    prompt = np.arange(3, 3 + 9, dtype=np.int32) * 7 % 256
    batch = ref_b.forward(prompt, 0)
    for t in range(prompt.size):
        inc = ref_i.forward(prompt[t:t + 1], t)
        assert np.array_equal(bits(batch[t]), bits(inc[0]))
