"""TEST INFRASTRUCTURE ONLY -- ctypes face of the CPU oracle.

Two libraries, both built by oracle/Makefile into oracle/_ref/:
  libmi_oracle.so  the plain-C restatement (oracle/mi_oracle.c)
  libmi_ref.so     the reference's own sources + oracle/ref_shim.cpp
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
P = C.c_void_p
I64, I32, F32 = C.c_int64, C.c_int32, C.c_float


def build(ref: str | None = None) -> None:
    args = ["make", "-s", "-C", HERE]
    if ref:
        args.append(f"REF={ref}")
    subprocess.run(args, check=True)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(P)


def _load(name: str) -> C.CDLL:
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing; run `make -C oracle`")
    return C.CDLL(path)


# ---------------------------------------------------------------------------
# The restatement
# ---------------------------------------------------------------------------

class _MioHparams(C.Structure):
    _fields_ = [("n_vocab", I32), ("n_embd", I32), ("n_layer", I32), ("n_head", I32),
                ("n_head_kv", I32), ("n_ff", I32), ("head_dim", I32), ("rms_eps", F32),
                ("rope_freq_base", F32)]


class _MioLayer(C.Structure):
    _fields_ = [(n, P) for n in ("attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo",
                                 "ffn_norm", "wgate", "wup", "wdown")]


class _MioWeights(C.Structure):
    _fields_ = [("token_embd", P), ("output_norm", P), ("output", P), ("layers", C.POINTER(_MioLayer))]


class Restatement:
    """numpy-level calls into oracle/mi_oracle.c."""

    def __init__(self):
        self.lib = L = _load("libmi_oracle.so")
        L.mio_fp16_to_fp32.restype = F32
        L.mio_fp16_to_fp32.argtypes = [C.c_uint16]
        L.mio_expf.restype = F32
        L.mio_expf.argtypes = [F32]
        L.mio_vec_dot_q8_0_wact.restype = F32
        L.mio_vec_dot_q8_0_wact.argtypes = [P, P, I64]
        L.mio_vec_dot_q8_0_wact_scalar.restype = F32
        L.mio_vec_dot_q8_0_wact_scalar.argtypes = [P, P, I64]
        L.mio_block_isum.restype = I32
        L.mio_block_isum.argtypes = [P, P]
        L.mio_block_lanes.argtypes = [P, P, P]
        L.mio_quantize_row_q8_0_act.argtypes = [P, P, I64]
        L.mio_quantize_row_q8_0.argtypes = [P, P, I64]
        L.mio_mul_mat_q8_0.argtypes = [P, I64, I64, P, I64, P]
        L.mio_get_rows_q8_0.argtypes = [P, I64, P, I64, P]
        L.mio_rms_norm.argtypes = [P, I64, I64, F32, P]
        L.mio_silu.argtypes = [P, I64, P]
        L.mio_rope_neox.argtypes = [P, I64, I64, I64, I32, I32, F32, P]
        L.mio_attn_qk.argtypes = [P, P, I64, I64, I64, I64, I64, P]
        L.mio_softmax.argtypes = [P, I64, I64, I64, I32, F32, P]
        L.mio_attn_kqv.argtypes = [P, P, I64, I64, I64, I64, I64, P]
        L.mio_sample_greedy.restype = I32
        L.mio_sample_greedy.argtypes = [P, I32]
        L.mio_qwen2_forward.argtypes = [C.POINTER(_MioHparams), C.POINTER(_MioWeights), P, P, I32,
                                        P, I32, I32, I32, P, P]

    def quantize_act(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        k = x.shape[-1]
        rows = x.reshape(-1, k)
        out = np.empty((rows.shape[0], k // 32 * 36), dtype=np.uint8)
        for r in range(rows.shape[0]):
            self.lib.mio_quantize_row_q8_0_act(_ptr(rows[r]), _ptr(out[r]), k)
        return out

    def mul_mat(self, w: np.ndarray, k: int, n: int, act: np.ndarray, m: int) -> np.ndarray:
        out = np.empty((m, n), dtype=np.float32)
        self.lib.mio_mul_mat_q8_0(_ptr(np.ascontiguousarray(w)), k, n, _ptr(np.ascontiguousarray(act)), m, _ptr(out))
        return out

    def block_lanes(self, x: np.ndarray, y: np.ndarray) -> np.ndarray:
        out = np.empty(8, dtype=np.int32)
        self.lib.mio_block_lanes(_ptr(x), _ptr(y), _ptr(out))
        return out

    def rms_norm(self, x: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.mio_rms_norm(_ptr(x), x.shape[-1], x.size // x.shape[-1], eps, _ptr(out))
        return out

    def silu(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.mio_silu(_ptr(x), x.size, _ptr(out))
        return out

    def rope(self, x: np.ndarray, n_past: int, n_dims: int, base: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)  # [n_tokens, n_head, head_dim]
        out = np.empty_like(x)
        t, h, d = x.shape
        self.lib.mio_rope_neox(_ptr(x), d, h, t, n_past, n_dims, base, _ptr(out))
        return out

    def attention(self, q, cache_k, cache_v, n_head_kv, n_past, n_tokens, scale):
        """q [T, H, D]; caches [n_ctx, HKV, D]. Returns (scores, probs, out)."""
        T, H, D = q.shape
        n_kv = n_past + n_tokens
        scores = np.empty((H, T, n_kv), dtype=np.float32)
        probs = np.empty_like(scores)
        out = np.empty((T, H, D), dtype=np.float32)
        q = np.ascontiguousarray(q, dtype=np.float32)
        self.lib.mio_attn_qk(_ptr(q), _ptr(cache_k), D, H, n_head_kv, n_kv, T, _ptr(scores))
        self.lib.mio_softmax(_ptr(scores), n_kv, T, H, n_past, scale, _ptr(probs))
        self.lib.mio_attn_kqv(_ptr(probs), _ptr(cache_v), D, H, n_head_kv, n_kv, T, _ptr(out))
        return scores, probs, out

    def expf(self, x: float) -> float:
        return self.lib.mio_expf(x)


class RestatedModel:
    """Whole-model restatement over a GGUF file (weights read zero-copy)."""

    def __init__(self, gguf, n_ctx: int):
        self.rs = Restatement()
        self.g = gguf
        s = gguf.shape()
        self.shape = s
        self.n_ctx = n_ctx
        self.hp = _MioHparams(s.n_vocab, s.n_embd, s.n_layer, s.n_head, s.n_head_kv, s.n_ff,
                              s.head_dim, s.rms_eps, s.rope_freq_base)
        L = (_MioLayer * s.n_layer)()
        self._keep = []

        def p(name):
            a = gguf.tensors[name].data
            self._keep.append(a)
            return a.ctypes.data

        for l in range(s.n_layer):
            b = f"blk.{l}."
            L[l] = _MioLayer(*[p(b + n) for n in (
                "attn_norm.weight", "attn_q.weight", "attn_q.bias", "attn_k.weight", "attn_k.bias",
                "attn_v.weight", "attn_v.bias", "attn_output.weight", "ffn_norm.weight",
                "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight")])
        out = "output.weight" if "output.weight" in gguf.tensors else "token_embd.weight"
        self.layers = L
        self.w = _MioWeights(p("token_embd.weight"), p("output_norm.weight"), p(out), L)
        kvsz = n_ctx * s.n_head_kv * s.head_dim
        self.cache_k = [np.zeros(kvsz, dtype=np.float32) for _ in range(s.n_layer)]
        self.cache_v = [np.zeros(kvsz, dtype=np.float32) for _ in range(s.n_layer)]
        self._kp = (P * s.n_layer)(*[c.ctypes.data for c in self.cache_k])
        self._vp = (P * s.n_layer)(*[c.ctypes.data for c in self.cache_v])

    def forward(self, tokens, n_past: int, last_logits_only: bool = False, layers: bool = False):
        s = self.shape
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        T = tok.size
        logits = np.empty((1 if last_logits_only else T, s.n_vocab), dtype=np.float32)
        lo = np.empty((s.n_layer, T, s.n_embd), dtype=np.float32) if layers else None
        self.rs.lib.mio_qwen2_forward(C.byref(self.hp), C.byref(self.w), self._kp, self._vp, self.n_ctx,
                                      _ptr(tok), T, n_past, int(last_logits_only), _ptr(logits),
                                      _ptr(lo) if lo is not None else None)
        return (logits, lo) if layers else logits


# ---------------------------------------------------------------------------
# The reference itself (compiled from source)
# ---------------------------------------------------------------------------

class Reference:
    """numpy-level calls into the reference's own code (oracle/_ref/libmi_ref.so)."""

    MI_OP = dict(get_rows=1, rms_norm=2, mul=3, add=4, mul_mat=5, rope=6, softmax=7, silu=8,
                 scale=9, cpy=10, quantize_q8_0=11, attn_qk=16, attn_kqv=17)

    def __init__(self):
        self.lib = L = _load("libmi_ref.so")
        L.mi_ref_last_error.restype = C.c_char_p
        L.mi_ref_quantize_row_q8_0_act.argtypes = [P, P, I64]
        L.mi_ref_quantize_row_q8_0.argtypes = [P, P, I64]
        L.mi_ref_vec_dot_q8_0_wact.restype = F32
        L.mi_ref_vec_dot_q8_0_wact.argtypes = [P, P, I64]
        L.mi_ref_vec_dot_q8_0_wact_scalar.restype = F32
        L.mi_ref_vec_dot_q8_0_wact_scalar.argtypes = [P, P, I64]
        L.mi_ref_block_isum_scalar.restype = I32
        L.mi_ref_block_isum_scalar.argtypes = [P, P]
        L.mi_ref_block_isum_avx2.restype = I32
        L.mi_ref_block_isum_avx2.argtypes = [P, P]
        L.mi_ref_fp16_to_fp32.restype = F32
        L.mi_ref_fp16_to_fp32.argtypes = [C.c_uint16]
        L.mi_ref_mul_mat_q8_0.argtypes = [P, I64, I64, P, I64, P, P]
        L.mi_ref_attention.argtypes = [P, P, P, I64, I64, I64, I64, I32, I64, F32, P, P, P]
        L.mi_ref_unary_op.argtypes = [I32, P, I64, I64, I64, P, I64, I64, I64, P, I32, P]
        L.mi_ref_get_rows_q8_0.argtypes = [P, I64, I64, P, I64, P]
        L.mi_ref_model_open.restype = P
        L.mi_ref_model_open.argtypes = [C.c_char_p, I32, I32]
        L.mi_ref_model_close.argtypes = [P]
        L.mi_ref_model_hparams.argtypes = [P, P]
        L.mi_ref_forward.argtypes = [P, P, I32, I32, I32, P]
        L.mi_ref_forward_dump.argtypes = [P, P, I32, I32, P, P, P]
        L.mi_ref_sample_greedy.restype = I32
        L.mi_ref_sample_greedy.argtypes = [P, I32]
        L.mi_ref_generate.restype = I32
        L.mi_ref_generate.argtypes = [P, P, I32, I32, P, C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.mi_ref_set_n_past.argtypes = [P, I32]

    def quantize_act(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        k = x.shape[-1]
        rows = x.reshape(-1, k)
        out = np.empty((rows.shape[0], k // 32 * 36), dtype=np.uint8)
        for r in range(rows.shape[0]):
            self.lib.mi_ref_quantize_row_q8_0_act(_ptr(rows[r]), _ptr(out[r]), k)
        return out

    def mul_mat(self, w: np.ndarray, k: int, n: int, x: np.ndarray):
        """W Q8_0 [n rows of k], x F32 [m, k] -> (act bytes [m, k/32*36], out [m, n])."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
        m = x.shape[0]
        act = np.empty((m, k // 32 * 36), dtype=np.uint8)
        out = np.empty((m, n), dtype=np.float32)
        self.lib.mi_ref_mul_mat_q8_0(_ptr(np.ascontiguousarray(w)), k, n, _ptr(x), m, _ptr(act), _ptr(out))
        return act, out

    def attention(self, q, cache_k, cache_v, n_head_kv, n_past, n_tokens, scale):
        T, H, D = q.shape
        n_ctx = cache_k.shape[0]
        n_kv = n_past + n_tokens
        scores = np.empty((H, T, n_kv), dtype=np.float32)
        probs = np.empty_like(scores)
        out = np.empty((T, H, D), dtype=np.float32)
        self.lib.mi_ref_attention(_ptr(np.ascontiguousarray(q, dtype=np.float32)), _ptr(cache_k),
                                  _ptr(cache_v), D, H, n_head_kv, n_ctx, n_past, T, scale,
                                  _ptr(scores), _ptr(probs), _ptr(out))
        return scores, probs, out

    def op(self, name: str, x: np.ndarray, y: np.ndarray | None = None, params=()) -> np.ndarray:
        """Run one mi_compute_<name> on x ([ne2, ne1, ne0] numpy order)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        xs = (1,) * (3 - x.ndim) + x.shape
        out = np.empty_like(x)
        ys = (0, 0, 0)
        if y is not None:
            y = np.ascontiguousarray(y, dtype=np.float32)
            ys = (1,) * (3 - y.ndim) + y.shape
        pr = np.zeros(8, dtype=np.int32)
        for i, v in enumerate(params):
            pr[i] = np.array([v], dtype=np.float32).view(np.int32)[0] if isinstance(v, float) else v
        self.lib.mi_ref_unary_op(self.MI_OP[name], _ptr(x), xs[2], xs[1], xs[0],
                                 _ptr(y) if y is not None else None, ys[2], ys[1], ys[0],
                                 _ptr(pr), len(params), _ptr(out))
        return out

    def get_rows_q8_0(self, table: np.ndarray, ne0: int, n_rows: int, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, ne0), dtype=np.float32)
        self.lib.mi_ref_get_rows_q8_0(_ptr(np.ascontiguousarray(table)), ne0, n_rows, _ptr(ids), ids.size, _ptr(out))
        return out


class ReferenceModel:
    """mi_qwen2_model_load + mi_kv_cache_init of the reference, one session."""

    def __init__(self, path: str, n_ctx: int, n_threads: int = 1):
        self.ref = Reference()
        self.h = self.ref.lib.mi_ref_model_open(path.encode(), n_ctx, n_threads)
        if not self.h:
            raise RuntimeError(self.ref.lib.mi_ref_last_error().decode())
        hp = np.zeros(10, dtype=np.int32)
        self.ref.lib.mi_ref_model_hparams(self.h, _ptr(hp))
        self.n_vocab, self.n_embd, self.n_layer = int(hp[0]), int(hp[1]), int(hp[2])
        self.n_ctx = n_ctx

    def forward(self, tokens, n_past: int, last_logits_only: bool = False) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        rows = 1 if last_logits_only else tok.size
        out = np.empty((rows, self.n_vocab), dtype=np.float32)
        self.ref.lib.mi_ref_forward(self.h, _ptr(tok), tok.size, n_past, int(last_logits_only), _ptr(out))
        return out

    def forward_dump(self, tokens, n_past: int):
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        T = tok.size
        layers = np.empty((self.n_layer, T, self.n_embd), dtype=np.float32)
        norm = np.empty((T, self.n_embd), dtype=np.float32)
        logits = np.empty((T, self.n_vocab), dtype=np.float32)
        self.ref.lib.mi_ref_forward_dump(self.h, _ptr(tok), T, n_past, _ptr(layers), _ptr(norm), _ptr(logits))
        return layers, norm, logits

    def generate(self, prompt, n_predict: int):
        """The reference CLI's --bench loop: returns (tokens, prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_predict, dtype=np.int32)
        pm, dm = C.c_double(), C.c_double()
        self.ref.lib.mi_ref_set_n_past(self.h, 0)
        n = self.ref.lib.mi_ref_generate(self.h, _ptr(p), p.size, n_predict, _ptr(out), C.byref(pm), C.byref(dm))
        return out[:n], pm.value, dm.value

    def close(self):
        if self.h:
            self.ref.lib.mi_ref_model_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
