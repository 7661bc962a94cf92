"""ctypes binding of the B200 decode backend (lib/libmi_cuda.so, include/mi_cuda.h).

Host-side mirror of the reference's operator and model interfaces:

  per-op calls      mi_compute_<op> (reference src/ops_cpu.h:62-138) on device
                    tensors: quantize_act, mul_mat, get_rows, rms_norm, mul,
                    add, scale, silu, rope, attn_qk, softmax, attn_kqv, ...
  model API         mi_qwen2_model_load / mi_kv_cache_init / mi_qwen2_forward /
                    mi_qwen2_sample_greedy (reference src/model_qwen2.h:83-189)
                    as Qwen2Model / KVCache / forward / sample_greedy.

Device tensors are torch CUDA tensors (torch is only the allocator and stream
provider here); every computation runs in libmi_cuda.so. There is no CPU
fallback: importing this module on a machine without the built library, or
calling a compute function without a GPU, raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmi_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "mi_cuda.h")

P, I32, I64, U64, F32, SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_size_t

# status codes (include/mi_cuda.h)
OK, ERR_ARG, ERR_CUDA, ERR_IO, ERR_FORMAT, ERR_TIMEOUT, ERR_STATE = range(7)


class MiCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"mi_cuda error {code}: {msg}")
        self.code = code


class Hparams(C.Structure):
    _fields_ = [("n_vocab", I32), ("n_embd", I32), ("n_layer", I32), ("n_head", I32),
                ("n_head_kv", I32), ("n_ff", I32), ("head_dim", I32), ("n_ctx_train", I32),
                ("rms_eps", F32), ("rope_freq_base", F32)]


_SIGS = {
    "mi_cuda_last_error": (C.c_char_p, []),
    "mi_cuda_init": (I32, [I32]),
    "mi_cuda_device_error": (I32, [I32, P]),
    "mi_cuda_q8_0_packed_bytes": (SZ, [I64, I64]),
    "mi_cuda_q8_0_pack": (I32, [P, I64, I64, P, P]),
    "mi_cuda_quantize_q8_0_act": (I32, [P, I64, I64, P, P]),
    "mi_cuda_mul_mat_q8_0": (I32, [P, I64, I64, P, I64, P, P]),
    "mi_cuda_mul_mat_q8_0_f32": (I32, [P, I64, I64, P, I64, P, P]),
    "mi_cuda_mul_mat_q8_0_scalar": (I32, [P, I64, I64, P, I64, P, P]),
    "mi_cuda_q8_0_block_isums": (I32, [P, I64, I64, P, P, P]),
    "mi_cuda_get_rows_q8_0": (I32, [P, I64, I64, P, I64, P, P]),
    "mi_cuda_rms_norm": (I32, [P, I64, I64, F32, P, P]),
    "mi_cuda_mul": (I32, [P, P, I64, I64, I64, P, P]),
    "mi_cuda_add": (I32, [P, P, I64, I64, I64, P, P]),
    "mi_cuda_scale": (I32, [P, I64, F32, P, P]),
    "mi_cuda_silu": (I32, [P, I64, P, P]),
    "mi_cuda_rope_neox": (I32, [P, I64, I64, I64, I32, I32, F32, P, P]),
    "mi_cuda_attn_qk": (I32, [P, P, I64, I64, I64, I64, I64, P, P]),
    "mi_cuda_softmax": (I32, [P, I64, I64, I64, I32, F32, P, P]),
    "mi_cuda_attn_kqv": (I32, [P, P, I64, I64, I64, I64, I64, P, P]),
    "mi_cuda_attention_decode_scratch_bytes": (SZ, [I64, I64]),
    "mi_cuda_attention_decode": (I32, [P, P, P, I64, I64, I64, I64, F32, P, P, P]),
    "mi_cuda_attention_decode_noalloc": (I32, [P, P, P, I64, I64, I64, I64, F32, P, P]),
    "mi_cuda_attention_decode_split_scratch_bytes": (SZ, [I64, I64, I64, I64]),
    "mi_cuda_attention_decode_split": (I32, [P, P, P, I64, I64, I64, I64, F32, P, P, P]),
    "mi_cuda_argmax": (I32, [P, I64, P, P]),
    "mi_cuda_expf": (I32, [P, I64, P, P]),
    "mi_cuda_expf_verify": (I32, [U64, U64, P]),
    "mi_cuda_qwen2_model_load": (I32, [C.c_char_p, I32, P]),
    "mi_cuda_qwen2_model_free": (None, [P]),
    "mi_cuda_qwen2_get_hparams": (I32, [P, P]),
    "mi_cuda_qwen2_weight_bytes": (SZ, [P]),
    "mi_cuda_kv_cache_init": (I32, [P, I32, P]),
    "mi_cuda_kv_cache_free": (None, [P]),
    "mi_cuda_qwen2_forward": (I32, [P, P, P, I32, I32, I32, P]),
    "mi_cuda_qwen2_last_token": (I32, [P, P]),
    "mi_cuda_qwen2_sample_greedy": (I32, [P, I32]),
    "mi_cuda_qwen2_generate": (I32, [P, P, P, I32, I32, P, P, P]),
    "mi_cuda_qwen2_set_position": (I32, [P, P, I32, I32]),
    "mi_cuda_qwen2_decode_steps": (I32, [P, I32, I32, I32]),
    "mi_cuda_qwen2_read_tokens": (I32, [P, I32, I32, P]),
    "mi_cuda_qwen2_stream": (P, [P]),
    "mi_cuda_qwen2_kernels_per_step": (I32, [P]),
    "mi_cuda_qwen2_set_fast_mode": (I32, [P, I32]),
    "mi_cuda_qwen2_fast_mode": (I32, [P]),
    "mi_cuda_qwen2_step_trace": (I32, [P, P, I32, P]),
    "mi_cuda_qwen2_model_load_shard": (I32, [C.c_char_p, I32, I32, I32, P]),
    "mi_cuda_tp_shard_range": (I32, [I64, I32, I32, P, P]),
    "mi_cuda_ipc_handle_bytes": (I32, []),
    "mi_cuda_tp_exchange_handle": (I32, [P, P]),
    "mi_cuda_tp_connect": (I32, [P, P]),
}

_lib = None


def header_symbols(path: str = HEADER) -> list[str]:
    """Names of every function include/mi_cuda.h declares."""
    text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
    return sorted(set(re.findall(r"\b(mi_cuda_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    """The loaded library. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise MiCudaError(rc, lib().mi_cuda_last_error().decode())


def init(device: int = 0) -> None:
    check(lib().mi_cuda_init(device))


# ---------------------------------------------------------------------------
# torch plumbing
# ---------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def _p(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int | None:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def to_device(a: np.ndarray, device: int = 0):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{device}")


# ---------------------------------------------------------------------------
# Per-op entry points (mirrors of mi_compute_<op>)
# ---------------------------------------------------------------------------

def q8_0_pack(raw, k: int, n: int):
    """GGUF Q8_0 rows (uint8 CUDA tensor, n*k/32*34 bytes) -> packed matrix."""
    torch = _torch()
    out = torch.empty(lib().mi_cuda_q8_0_packed_bytes(k, n), dtype=torch.uint8, device=raw.device)
    check(lib().mi_cuda_q8_0_pack(_p(raw), k, n, _p(out), _stream()))
    return out


def quantize_act(x, k: int):
    torch = _torch()
    m = x.numel() // k
    out = torch.empty(m * (k // 32) * 36, dtype=torch.uint8, device=x.device)
    check(lib().mi_cuda_quantize_q8_0_act(_p(x), k, m, _p(out), _stream()))
    return out


def mul_mat(w_packed, k: int, n: int, act=None, x=None, m: int = 1):
    """mi_compute_mul_mat for a Q8_0 weight: from Q8_0_ACT `act` or F32 `x`."""
    torch = _torch()
    out = torch.empty((m, n), dtype=torch.float32, device=w_packed.device)
    if act is not None:
        check(lib().mi_cuda_mul_mat_q8_0(_p(w_packed), k, n, _p(act), m, _p(out), _stream()))
    else:
        check(lib().mi_cuda_mul_mat_q8_0_f32(_p(w_packed), k, n, _p(x), m, _p(out), _stream()))
    return out


def mul_mat_scalar(w_packed, k: int, n: int, act, m: int = 1):
    """mi_compute_mul_mat on the reference's scalar dot path (MI_QUANT_FORCE_SCALAR)."""
    torch = _torch()
    out = torch.empty((m, n), dtype=torch.float32, device=w_packed.device)
    check(lib().mi_cuda_mul_mat_q8_0_scalar(_p(w_packed), k, n, _p(act), m, _p(out), _stream()))
    return out


def block_isums(w_packed, k: int, n: int, act):
    torch = _torch()
    out = torch.empty((n, k // 32), dtype=torch.int32, device=w_packed.device)
    check(lib().mi_cuda_q8_0_block_isums(_p(w_packed), k, n, _p(act), _p(out), _stream()))
    return out


def get_rows(table_packed, ne0: int, n_rows: int, ids):
    torch = _torch()
    out = torch.empty((ids.numel(), ne0), dtype=torch.float32, device=ids.device)
    check(lib().mi_cuda_get_rows_q8_0(_p(table_packed), ne0, n_rows, _p(ids), ids.numel(), _p(out), _stream()))
    return out


def rms_norm(x, eps: float):
    out = _torch().empty_like(x)
    ne0 = x.shape[-1]
    check(lib().mi_cuda_rms_norm(_p(x), ne0, x.numel() // ne0, eps, _p(out), _stream()))
    return out


def mul(a, b):
    out = _torch().empty_like(a)
    ne0 = a.shape[-1]
    check(lib().mi_cuda_mul(_p(a), _p(b), ne0, a.numel() // ne0, b.numel() // ne0, _p(out), _stream()))
    return out


def add(a, b):
    out = _torch().empty_like(a)
    ne0 = a.shape[-1]
    check(lib().mi_cuda_add(_p(a), _p(b), ne0, a.numel() // ne0, b.numel() // ne0, _p(out), _stream()))
    return out


def scale(x, v: float):
    out = _torch().empty_like(x)
    check(lib().mi_cuda_scale(_p(x), x.numel(), v, _p(out), _stream()))
    return out


def silu(x):
    out = _torch().empty_like(x)
    check(lib().mi_cuda_silu(_p(x), x.numel(), _p(out), _stream()))
    return out


def expf(x):
    out = _torch().empty_like(x)
    check(lib().mi_cuda_expf(_p(x), x.numel(), _p(out), _stream()))
    return out


def expf_verify(first: int, count: int) -> int:
    n = C.c_uint64()
    check(lib().mi_cuda_expf_verify(first, count, C.byref(n)))
    return n.value


def rope(x, n_past: int, n_dims: int, freq_base: float):
    """x [n_tokens, n_head, head_dim]."""
    out = _torch().empty_like(x)
    t, h, d = x.shape
    check(lib().mi_cuda_rope_neox(_p(x), d, h, t, n_past, n_dims, freq_base, _p(out), _stream()))
    return out


def attn_qk(q, cache_k, n_head_kv: int, n_kv: int):
    """q [T, H, D], cache_k [n_ctx, HKV, D] -> scores [H, T, n_kv]."""
    torch = _torch()
    T, H, D = q.shape
    out = torch.empty((H, T, n_kv), dtype=torch.float32, device=q.device)
    check(lib().mi_cuda_attn_qk(_p(q), _p(cache_k), D, H, n_head_kv, n_kv, T, _p(out), _stream()))
    return out


def softmax(x, n_past: int, scale_: float):
    """x [H, T, n_kv] -> probs."""
    out = _torch().empty_like(x)
    H, T, n_kv = x.shape
    check(lib().mi_cuda_softmax(_p(x), n_kv, T, H, n_past, scale_, _p(out), _stream()))
    return out


def attn_kqv(probs, cache_v, n_head_kv: int, head_dim: int):
    """probs [H, T, n_kv], cache_v [n_ctx, HKV, D] -> out [T, H, D]."""
    torch = _torch()
    H, T, n_kv = probs.shape
    out = torch.empty((T, H, head_dim), dtype=torch.float32, device=probs.device)
    check(lib().mi_cuda_attn_kqv(_p(probs), _p(cache_v), head_dim, H, n_head_kv, n_kv, T, _p(out), _stream()))
    return out


def attention_decode(q, cache_k, cache_v, n_head_kv: int, n_kv: int, scale_: float, scratch=None):
    """Fused decode attention: q [H, D] rotated -> out [H, D]."""
    torch = _torch()
    H, D = q.shape
    if scratch is None:
        nb = lib().mi_cuda_attention_decode_scratch_bytes(H, n_kv)
        scratch = torch.empty(nb, dtype=torch.uint8, device=q.device)
    out = torch.empty((H, D), dtype=torch.float32, device=q.device)
    check(lib().mi_cuda_attention_decode(_p(q), _p(cache_k), _p(cache_v), D, H, n_head_kv, n_kv, scale_,
                                         _p(scratch), _p(out), _stream()))
    return out


def attention_decode_split(q, cache_k, cache_v, n_head_kv: int, n_kv: int, scale_: float, scratch=None):
    """Split-over-positions fast mode of attention_decode (regrouped sums, not bit-exact)."""
    torch = _torch()
    H, D = q.shape
    if scratch is None:
        nb = lib().mi_cuda_attention_decode_split_scratch_bytes(H, n_head_kv, n_kv, D)
        scratch = torch.empty(nb, dtype=torch.uint8, device=q.device)
    out = torch.empty((H, D), dtype=torch.float32, device=q.device)
    check(lib().mi_cuda_attention_decode_split(_p(q), _p(cache_k), _p(cache_v), D, H, n_head_kv, n_kv, scale_,
                                               _p(scratch), _p(out), _stream()))
    return out


def argmax(x):
    torch = _torch()
    out = torch.empty(1, dtype=torch.int32, device=x.device)
    check(lib().mi_cuda_argmax(_p(x), x.numel(), _p(out), _stream()))
    return out


# ---------------------------------------------------------------------------
# Model API (mirrors of mi_qwen2_* / mi_kv_cache_*)
# ---------------------------------------------------------------------------

def sample_greedy(logits: np.ndarray) -> int:
    """mi_qwen2_sample_greedy: first index of the maximum."""
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().mi_cuda_qwen2_sample_greedy(a.ctypes.data, a.size))


def shard_range(n_units: int, rank: int, world: int) -> tuple[int, int]:
    """(first, count) of the units rank `rank` owns (mi_cuda_tp_shard_range)."""
    first, count = C.c_int64(), C.c_int64()
    check(lib().mi_cuda_tp_shard_range(n_units, rank, world, C.byref(first), C.byref(count)))
    return first.value, count.value


class Qwen2Model:
    """mi_qwen2_model_load: GGUF -> weights resident in HBM. With world > 1
    only this rank's rows of every projection are loaded (tensor
    parallelism; see mi_cuda_qwen2_model_load_shard)."""

    def __init__(self, gguf_path: str, device: int = 0, rank: int = 0, world: int = 1):
        h = P()
        if world == 1:
            check(lib().mi_cuda_qwen2_model_load(gguf_path.encode(), device, C.byref(h)))
        else:
            check(lib().mi_cuda_qwen2_model_load_shard(gguf_path.encode(), device, rank, world, C.byref(h)))
        self.h = h
        self.device = device
        self.rank, self.world = rank, world
        hp = Hparams()
        check(lib().mi_cuda_qwen2_get_hparams(self.h, C.byref(hp)))
        self.hparams = hp
        self.n_vocab = hp.n_vocab

    @property
    def weight_bytes(self) -> int:
        return int(lib().mi_cuda_qwen2_weight_bytes(self.h))

    def free(self):
        if self.h:
            lib().mi_cuda_qwen2_model_free(self.h)
            self.h = None


class KVCache:
    """mi_kv_cache_init: KV cache, step workspace and captured step graphs."""

    def __init__(self, model: Qwen2Model, n_ctx: int):
        h = P()
        check(lib().mi_cuda_kv_cache_init(model.h, n_ctx, C.byref(h)))
        self.h = h
        self.model = model
        self.n_ctx = n_ctx
        self.n_past = 0

    def exchange_handle(self) -> bytes:
        """This rank's exchange-buffer handle (sharded models)."""
        buf = (C.c_uint8 * int(lib().mi_cuda_ipc_handle_bytes()))()
        check(lib().mi_cuda_tp_exchange_handle(self.h, buf))
        return bytes(buf)

    def connect(self, handles: list[bytes]):
        """Map every rank's exchange buffer (handles in rank order) and capture
        the step graphs."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().mi_cuda_tp_connect(self.h, buf))

    def forward(self, tokens, n_past: int, last_logits_only: bool = False, want_logits: bool = True):
        """mi_qwen2_forward: returns logits [rows, n_vocab] (rows = 1 with last_logits_only)."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        rows = 1 if last_logits_only else tok.size
        out = np.empty((rows, self.model.n_vocab), dtype=np.float32) if want_logits else None
        check(lib().mi_cuda_qwen2_forward(self.model.h, self.h, tok.ctypes.data, tok.size, n_past,
                                          int(last_logits_only), out.ctypes.data if out is not None else None))
        return out

    def last_token(self) -> int:
        v = C.c_int32()
        check(lib().mi_cuda_qwen2_last_token(self.h, C.byref(v)))
        return v.value

    def generate(self, prompt, n_predict: int):
        """The reference CLI's --bench loop on the device: (tokens, prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_predict, dtype=np.int32)
        a, b = C.c_double(), C.c_double()
        check(lib().mi_cuda_qwen2_generate(self.model.h, self.h, p.ctypes.data, p.size, n_predict,
                                           out.ctypes.data, C.byref(a), C.byref(b)))
        return out, a.value, b.value

    def set_position(self, tokens, pos: int):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(lib().mi_cuda_qwen2_set_position(self.h, t.ctypes.data if t.size else None, t.size, pos))

    def decode_steps(self, n: int, pos0: int = 0, period: int = 0):
        check(lib().mi_cuda_qwen2_decode_steps(self.h, n, pos0, period))

    def read_tokens(self, first: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        check(lib().mi_cuda_qwen2_read_tokens(self.h, first, n, out.ctypes.data))
        return out

    @property
    def stream_handle(self) -> int:
        return int(lib().mi_cuda_qwen2_stream(self.h) or 0)

    @property
    def kernels_per_step(self) -> int:
        return int(lib().mi_cuda_qwen2_kernels_per_step(self.h))

    @property
    def fast_mode(self) -> bool:
        return bool(lib().mi_cuda_qwen2_fast_mode(self.h))

    def set_fast_mode(self, on: bool):
        """Labelled fast mode of the decode step (regrouped sums; NOT
        bit-identical to the reference): on / off. Raises where the
        persistent step is not in use."""
        check(lib().mi_cuda_qwen2_set_fast_mode(self.h, int(bool(on))))

    def step_trace(self) -> np.ndarray:
        """[slots, 8] globaltimer stamps (ns) of the last step. Kernel-per-phase
        step: one slot per kernel (first CTA): entry, predecessor done,
        prologue done, epilogue start, then the kernel's own phase marks
        (attention: scores, exp, sum, KV done). Persistent step (one kernel):
        two slots per layer -- attention CTA 0 (layer start, x ready, prologue
        done, rows done, k/v received, exp done, sum done, O rows signalled)
        and the first projection CTA (layer start, norm weights loaded,
        gate/up wait done, its prologue done, gate/up signalled, down wait
        done, down signalled)
        -- then the LM head (wait done, prologue done, rows done, step closed,
        then the first projection CTA's totals over its LM-head items: ns
        waiting for ring items, ns in the rows, ns issuing copies, items)."""
        n = self.kernels_per_step if self.kernels_per_step > 1 else 2 * self.model.hparams.n_layer + 1
        out = np.zeros((n, 8), dtype=np.uint64)
        got = C.c_int32()
        check(lib().mi_cuda_qwen2_step_trace(self.h, out.ctypes.data, n, C.byref(got)))
        return out[:got.value]

    def free(self):
        if self.h:
            lib().mi_cuda_kv_cache_free(self.h)
            self.h = None


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's exchange handle, in rank order, over torch.distributed
    (any backend; the handles are small host objects)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def tp_connect(kv: "KVCache", group=None):
    """Exchange-buffer handshake of a sharded model's KV cache on every rank."""
    kv.connect(gather_handles(kv.exchange_handle(), group))
