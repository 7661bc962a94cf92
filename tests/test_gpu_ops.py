"""Per-op parity on the GPU: each CUDA entry point against the CPU oracle on
the same seeded inputs. Integer work (quantization bytes, block int32 sums,
argmax) and every float output are compared bit for bit: the kernels follow the
reference's IEEE operation order, so the tolerance is zero.

Shapes follow the benchmark configs: the Q8_0 GEMV sweep [N x K] = 896x896,
128x896, 4864x896, 896x4864, 151936x896 (config 1), and decode attention with
14 query / 2 KV heads, head_dim 64, n_kv = 128 / 1024 / 4096 / 32768 (config 2).
"""
import numpy as np
import pytest

import mi_gguf
import mi_oracle
from conftest import bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def S():
    return mi_oracle.Restatement()


@pytest.fixture(scope="module")
def R():
    return mi_oracle.Reference()


@pytest.fixture(scope="module")
def mc(torch_cuda):
    import mi_cuda
    return mi_cuda


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_expf_matches_host_libm_on_every_float(mc, torch_cuda):
    # All 2^32 inputs: the device expf (double core + exception table) against
    # this host's libm expf, which the reference's softmax and SiLU call.
    assert mc.expf_verify(0, 1 << 32) == 0


def test_expf_special_values(mc, torch_cuda):
    torch = torch_cuda
    x = np.array([0.0, -0.0, 1.0, -1.0, 88.7, 88.8, -87.3, -103.9, -104.0, -200.0, 300.0,
                  np.inf, -np.inf, 1e-30, -1e-30], dtype=np.float32)
    y = mc.expf(dev(torch, x)).cpu().numpy()
    want = np.array([mi_oracle.Restatement().expf(float(v)) for v in x], dtype=np.float32)
    assert np.array_equal(bits(y), bits(want))


@pytest.mark.parametrize("k,m", [(896, 1), (896, 3), (4864, 1), (64, 5)])
def test_quantize_act_bitexact(mc, S, torch_cuda, k, m):
    rng = np.random.default_rng(k + m)
    x = (rng.standard_normal((m, k)) * rng.uniform(0.01, 30)).astype(np.float32)
    x[0, 32:64] = 0.0  # an all-zero block: d = 0, q = 0
    got = mc.quantize_act(dev(torch_cuda, x), k).cpu().numpy()
    assert np.array_equal(got, S.quantize_act(x).reshape(-1))


CONFIG1 = [(896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896)]


@pytest.mark.parametrize("n,k", CONFIG1 + [(132, 64), (12, 96), (4096, 2048), (2048, 8192), (3584, 3584)])
def test_gemv_config1_bitexact(mc, S, torch_cuda, n, k):
    torch = torch_cuda
    rng = np.random.default_rng(n + 3 * k)
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    x = rng.standard_normal((1, k), dtype=np.float32)
    act = S.quantize_act(x)
    want = S.mul_mat(w, k, n, act, 1)
    wp = mc.q8_0_pack(dev(torch, w.reshape(-1)), k, n)
    got_fused = mc.mul_mat(wp, k, n, x=dev(torch, x)).cpu().numpy()
    got_act = mc.mul_mat(wp, k, n, act=dev(torch, act.reshape(-1))).cpu().numpy()
    assert np.array_equal(bits(got_fused), bits(want))
    assert np.array_equal(bits(got_act), bits(want))
    # per-block int32 sums through the kernel's dp4a lanes
    isums = mc.block_isums(wp, k, n, dev(torch, act.reshape(-1))).cpu().numpy()
    wq = w.reshape(n, k // 32, 34)[:, :, 2:].view(np.int8).astype(np.int64)
    aq = act.reshape(k // 32, 36)[:, 4:].view(np.int8).astype(np.int64)
    assert np.array_equal(isums, (wq * aq[None]).sum(-1))


@pytest.mark.parametrize("n,k,var,val", [(896, 4864, "MI_CUDA_GEMV_WIDE", "8,8,8"),
                                         (896, 4864, "MI_CUDA_GEMV_WIDE", "8,8,4"),
                                         (200, 2080, "MI_CUDA_GEMV_TPR", "8"),
                                         (896, 4864, "MI_CUDA_GEMV_WIDE", "2,8,64")])
def test_gemv_stage_layouts_bitexact(mc, S, torch_cuda, monkeypatch, n, k, var, val):
    """The 8-thread mapping's quad loads under every stage shape: K-chunks of
    30 and 14 blocks (chunks starting off a multiple of 4 blocks), an odd
    number of blocks per row (K = 2080: no quad loads), and the 2-thread
    mapping on wide rows."""
    monkeypatch.setenv(var, val)
    torch = torch_cuda
    rng = np.random.default_rng(n + 7 * k)
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    x = rng.standard_normal((1, k), dtype=np.float32)
    act = S.quantize_act(x)
    want = S.mul_mat(w, k, n, act, 1)
    wp = mc.q8_0_pack(dev(torch, w.reshape(-1)), k, n)
    assert np.array_equal(bits(mc.mul_mat(wp, k, n, x=dev(torch, x)).cpu().numpy()), bits(want))
    assert np.array_equal(bits(mc.mul_mat(wp, k, n, act=dev(torch, act.reshape(-1))).cpu().numpy()), bits(want))


@pytest.mark.parametrize("n,k,m", [(896, 896, 1), (128, 896, 2), (896, 4864, 1), (12, 1056, 3)])
def test_gemv_scalar_order_bitexact(mc, S, R, torch_cuda, n, k, m):
    """The reference's scalar dot (MI_QUANT_FORCE_SCALAR path): bit-exact
    against the oracle's restatement and the reference's own scalar dot."""
    torch = torch_cuda
    rng = np.random.default_rng(n * 5 + k + m)
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    act = S.quantize_act(rng.standard_normal((m, k), dtype=np.float32))
    wr = w.reshape(n, k // 32 * 34)
    want = np.empty((m, n), dtype=np.float32)
    for j in range(m):
        for i in range(n):
            want[j, i] = S.lib.mio_vec_dot_q8_0_wact_scalar(wr[i].ctypes.data, act[j].ctypes.data, k)
    i = n // 2
    assert np.float32(R.lib.mi_ref_vec_dot_q8_0_wact_scalar(wr[i].ctypes.data, act[0].ctypes.data, k)) == want[0, i]
    wp = mc.q8_0_pack(dev(torch, w.reshape(-1)), k, n)
    got = mc.mul_mat_scalar(wp, k, n, dev(torch, act.reshape(-1)), m).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


def test_gemv_multi_column_and_relative_tolerance(mc, R, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(77)
    n, k, m = 300, 896, 3
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    x = rng.standard_normal((m, k), dtype=np.float32)
    act, want = R.mul_mat(w, k, n, x)
    got = mc.mul_mat(mc.q8_0_pack(dev(torch, w.reshape(-1)), k, n), k, n, x=dev(torch, x), m=m).cpu().numpy()
    # config 1's stated bar is 1e-5 relative; the kernel meets it with zero error
    assert np.all(np.abs(got - want) <= 1e-5 * np.abs(want))
    assert np.array_equal(bits(got), bits(want))


def test_get_rows_q8_0(mc, R, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    n, k = 1000, 896
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    ids = np.array([0, 999, 17, 17, 512], dtype=np.int32)
    want = R.get_rows_q8_0(w, k, n, ids)
    wp = mc.q8_0_pack(dev(torch, w.reshape(-1)), k, n)
    got = mc.get_rows(wp, k, n, dev(torch, ids)).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


def test_elementwise_ops(mc, R, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((3, 896)) * 3).astype(np.float32)
    w = rng.standard_normal(896).astype(np.float32)
    y = rng.standard_normal((3, 896)).astype(np.float32)
    X, W, Y = dev(torch, x), dev(torch, w), dev(torch, y)
    assert np.array_equal(bits(mc.rms_norm(X, 1e-6).cpu()), bits(R.op("rms_norm", x, params=(1e-6,))))
    assert np.array_equal(bits(mc.mul(X, W).cpu()), bits(R.op("mul", x, w)))
    assert np.array_equal(bits(mc.add(X, Y).cpu()), bits(R.op("add", x, y)))
    assert np.array_equal(bits(mc.scale(X, 0.125).cpu()), bits(R.op("scale", x, params=(0.125,))))
    big = (rng.standard_normal(4864 * 4) * 6).astype(np.float32)
    assert np.array_equal(bits(mc.silu(dev(torch, big)).cpu()), bits(R.op("silu", big)))


def _norm_rows(rng, ne0):
    """Rows for the rms_norm chain: plain, heavy-tailed, and one built so the
    float chain drifts hundreds of ulps from the exact prefix sum (every square
    of 0.3 added to 2^20 rounds up by 0.28 ulp), which forces the speculative
    sum's serial fallback on its later segments."""
    plain = (rng.standard_normal(ne0) * 3).astype(np.float32)
    heavy = (rng.standard_normal(ne0) * np.exp(rng.standard_normal(ne0) * 2)).astype(np.float32)
    drift = np.full(ne0, 0.3, dtype=np.float32)
    drift[0] = 1024.0
    zeros = np.zeros(ne0, dtype=np.float32)
    return np.stack([plain, heavy, drift, zeros])


@pytest.mark.parametrize("ne0", [1, 5, 31, 100, 896, 3584, 10240, 12288])
def test_rms_norm_ordered_chain(mc, R, torch_cuda, ne0):
    """rms_norm bit-exact at lengths below, at and above the speculative
    chain's thresholds (CTA-wide speculation up to 10240 elements, one
    thread's serial chain beyond)."""
    torch = torch_cuda
    x = _norm_rows(np.random.default_rng(ne0), ne0)
    want = R.op("rms_norm", x, params=(1e-6,))
    got = mc.rms_norm(dev(torch, x), 1e-6).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("n_past,n_tokens,heads", [(0, 1, 14), (31, 1, 2), (158, 1, 14), (2047, 1, 14), (5, 7, 4)])
def test_rope(mc, R, torch_cuda, n_past, n_tokens, heads):
    torch = torch_cuda
    rng = np.random.default_rng(n_past + heads)
    x = rng.standard_normal((n_tokens, heads, 64), dtype=np.float32)
    want = R.op("rope", x, params=(n_past, 64, 1e6))
    got = mc.rope(dev(torch, x), n_past, 64, 1e6).cpu().numpy()
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("n_kv,n_tokens", [(128, 1), (40, 6)])
def test_attention_ops_separately(mc, S, torch_cuda, n_kv, n_tokens):
    torch = torch_cuda
    rng = np.random.default_rng(n_kv * 13)
    H, HKV, D = 14, 2, 64
    n_ctx = n_kv + 4
    q = rng.standard_normal((n_tokens, H, D), dtype=np.float32)
    k = rng.standard_normal((n_ctx, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_ctx, HKV, D), dtype=np.float32)
    n_past = n_kv - n_tokens
    s_w, p_w, o_w = S.attention(q, k, v, HKV, n_past, n_tokens, 0.125)
    K, V = dev(torch, k), dev(torch, v)
    s = mc.attn_qk(dev(torch, q), K, HKV, n_kv)
    p = mc.softmax(s, n_past, 0.125)
    o = mc.attn_kqv(p, V, HKV, D)
    assert np.array_equal(bits(s.cpu()), bits(s_w))
    assert np.array_equal(bits(p.cpu()), bits(p_w))
    assert np.array_equal(bits(o.cpu()), bits(o_w))


@pytest.mark.parametrize("n_kv", [1, 128, 300, 511, 512, 1024, 4096, 8192, 8193, 20001, 32768, 60001])
def test_attention_decode_config2(mc, S, torch_cuda, n_kv):
    torch = torch_cuda
    rng = np.random.default_rng(n_kv)
    H, HKV, D = 14, 2, 64
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    k = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    _, _, want = S.attention(q, k, v, HKV, n_kv - 1, 1, 0.125)
    got = mc.attention_decode(dev(torch, q[0]), dev(torch, k), dev(torch, v), HKV, n_kv, 0.125).cpu().numpy()
    assert np.array_equal(bits(got), bits(want[0]))


@pytest.mark.parametrize("n_kv,H,HKV,D", [(9001, 28, 4, 128), (12000, 16, 16, 32)])
def test_attention_decode_long_context_shapes(mc, S, torch_cuda, n_kv, H, HKV, D):
    """Past 8192 positions one query's exact attention runs as three kernels
    (scores over many CTAs, the ordered denominator by the speculative sum,
    the ordered value chains): bit-identical to the reference order for other
    head shapes too (7B widths; one query head per KV head, head_dim 32)."""
    torch = torch_cuda
    rng = np.random.default_rng(n_kv + D)
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    k = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    scale = float(np.float32(1.0 / np.sqrt(D)))
    _, _, want = S.attention(q, k, v, HKV, n_kv - 1, 1, scale)
    got = mc.attention_decode(dev(torch, q[0]), dev(torch, k), dev(torch, v), HKV, n_kv, scale).cpu().numpy()
    assert np.array_equal(bits(got), bits(want[0]))


@pytest.mark.parametrize("n_kv,H,HKV,D", [(1, 14, 2, 64), (33, 14, 2, 64), (1024, 14, 2, 64), (32768, 14, 2, 64),
                                          (4100, 28, 4, 128), (300, 4, 4, 16)])
def test_attention_decode_split_mode_tolerance(mc, S, torch_cuda, n_kv, H, HKV, D):
    """The split-over-positions fast mode against the reference-order oracle:
    regrouped sums, so within max-abs 1e-5 and cosine >= 0.999999 of the exact
    output rather than bit-identical."""
    torch = torch_cuda
    rng = np.random.default_rng(n_kv + H)
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    k = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    scale = float(np.float32(1.0 / np.sqrt(D)))
    _, _, want = S.attention(q, k, v, HKV, n_kv - 1, 1, scale)
    got = mc.attention_decode_split(dev(torch, q[0]), dev(torch, k), dev(torch, v), HKV, n_kv, scale).cpu().numpy()
    a, b = got.astype(np.float64).ravel(), want[0].astype(np.float64).ravel()
    assert np.max(np.abs(a - b)) <= 1e-5
    assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b)) >= 0.999999


def test_argmax_first_max(mc, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(1)
    x = rng.standard_normal(151936).astype(np.float32)
    x[[5000, 70000, 151935]] = 9.0  # ties: the lowest index wins
    assert int(mc.argmax(dev(torch, x)).cpu()[0]) == 5000
    y = np.full(1000, -1.0, dtype=np.float32)
    assert int(mc.argmax(dev(torch, y)).cpu()[0]) == 0
    assert int(mc.argmax(dev(torch, x[:1])).cpu()[0]) == 0


def test_bad_arguments_return_status(mc, torch_cuda):
    import ctypes as C
    L = mc.lib()
    assert L.mi_cuda_mul_mat_q8_0(None, 896, 896, None, 1, None, None) == mc.ERR_ARG
    assert L.mi_cuda_attention_decode(None, None, None, 64, 14, 3, 10, 0.1, None, None, None) == mc.ERR_ARG
    code = C.c_int32(-1)
    assert L.mi_cuda_device_error(0, C.byref(code)) == mc.OK and code.value == 0
