"""GGUF v3 reader and random-init Qwen2 GGUF writer (numpy).

The writer produces the synthetic models the decode benchmarks run on: a
Qwen2-architecture GGUF v3 file with seeded N(0, 0.02) weights quantized to
Q8_0 (blocks of 32 int8 with an fp16 scale amax/127), norm weights 1.0,
N(0, 0.02) biases, tied or untied lm_head, and the tokenizer arrays the
reference loader requires.

File-format facts it must honour (reference: src/gguf.cpp:259-436, the GGUF v3
spec): magic "GGUF", u32 version 3, u64 tensor/kv counts, length-prefixed
strings, tensor infos of (name, n_dims, ne[], ggml type, offset), data section
aligned to general.alignment (default 32). ggml type ids: F32 0, F16 1, Q8_0 8.
Metadata keys the reference reads: src/model_qwen2.cpp:426-464 (hparams) and
src/gguf.cpp:751-785 (tokenizer.ggml.tokens is required).

Q8_0 quantization follows mi_quantize_row_q8_0 (src/quant.cpp:130-160):
float32 amax, d = amax/127, id = 1/d, q = round-half-even(x*id) clamped to
+-127, d stored as fp16 (round to nearest even).
"""
from __future__ import annotations

import dataclasses
import mmap
import os
import struct
import subprocess

import numpy as np

GGUF_MAGIC = b"GGUF"
GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR_FMT = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
               T_F32: "<f", T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}
Q8_0_DTYPE = np.dtype([("d", "<f2"), ("qs", "i1", (32,))])
assert Q8_0_DTYPE.itemsize == 34


@dataclasses.dataclass(frozen=True)
class Qwen2Shape:
    """Architecture of a Qwen2 model as the GGUF metadata describes it."""
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_vocab: int
    tied: bool = True
    rms_eps: float = 1e-6
    rope_freq_base: float = 1e6
    n_ctx_train: int = 32768

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


# The decode, prefill and sweep workloads (Qwen2.5-0.5B architecture) and the
# tensor-parallel workload (Qwen2.5-7B architecture).
QWEN2_05B = Qwen2Shape(n_layer=24, n_embd=896, n_head=14, n_head_kv=2, n_ff=4864, n_vocab=151936)
QWEN2_7B = Qwen2Shape(n_layer=28, n_embd=3584, n_head=28, n_head_kv=4, n_ff=18944, n_vocab=152064,
                      tied=False)
# Small shapes for parity tests that the CPU oracle finishes in seconds.
TINY = Qwen2Shape(n_layer=2, n_embd=64, n_head=4, n_head_kv=2, n_ff=128, n_vocab=256)
SMALL = Qwen2Shape(n_layer=4, n_embd=256, n_head=4, n_head_kv=2, n_ff=512, n_vocab=2048)
# The 7B shape's widths (head_dim 128, FFN 18944, untied LM head) in two layers.
MID7B = Qwen2Shape(n_layer=2, n_embd=3584, n_head=28, n_head_kv=4, n_ff=18944, n_vocab=4096,
                   tied=False)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """F32 rows [n, k] -> Q8_0 blocks [n, k/32] (structured, 34 B each)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    blocks = x.reshape(-1, 32)
    amax = np.abs(blocks).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.rint(blocks * inv[:, None])
    np.clip(q, -127, 127, out=q)
    out = np.empty(blocks.shape[0], dtype=Q8_0_DTYPE)
    out["d"] = d.astype(np.float16)
    out["qs"] = q.astype(np.int8)
    return out.reshape(x.shape[0], -1) if x.ndim == 2 else out


def dequantize_q8_0(blocks: np.ndarray) -> np.ndarray:
    b = blocks.reshape(-1)
    return (b["qs"].astype(np.float32) * b["d"].astype(np.float32)[:, None]).reshape(-1)


# ---------------------------------------------------------------------------
# Writer
# ---------------------------------------------------------------------------

def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, typ: int, value) -> bytes:
    out = _str(key) + struct.pack("<I", typ)
    if typ == T_STR:
        return out + _str(value)
    if typ == T_ARR:
        etyp, items = value
        out += struct.pack("<IQ", etyp, len(items))
        if etyp == T_STR:
            return out + b"".join(_str(s) for s in items)
        return out + np.asarray(items, dtype=np.dtype(_SCALAR_FMT[etyp][1:]).newbyteorder("<")).tobytes()
    return out + struct.pack(_SCALAR_FMT[typ], value)


def _tensor_plan(shape: Qwen2Shape):
    """(name, ggml type, ne) in file order, matching model_qwen2.cpp:496-538."""
    E, D = shape.n_embd, shape.head_dim
    kvd = shape.n_head_kv * D
    plan = [("token_embd.weight", GGML_Q8_0, (E, shape.n_vocab)),
            ("output_norm.weight", GGML_F32, (E,))]
    if not shape.tied:
        plan.append(("output.weight", GGML_Q8_0, (E, shape.n_vocab)))
    for l in range(shape.n_layer):
        p = f"blk.{l}."
        plan += [(p + "attn_norm.weight", GGML_F32, (E,)),
                 (p + "attn_q.weight", GGML_Q8_0, (E, E)), (p + "attn_q.bias", GGML_F32, (E,)),
                 (p + "attn_k.weight", GGML_Q8_0, (E, kvd)), (p + "attn_k.bias", GGML_F32, (kvd,)),
                 (p + "attn_v.weight", GGML_Q8_0, (E, kvd)), (p + "attn_v.bias", GGML_F32, (kvd,)),
                 (p + "attn_output.weight", GGML_Q8_0, (E, E)),
                 (p + "ffn_norm.weight", GGML_F32, (E,)),
                 (p + "ffn_gate.weight", GGML_Q8_0, (E, shape.n_ff)),
                 (p + "ffn_up.weight", GGML_Q8_0, (E, shape.n_ff)),
                 (p + "ffn_down.weight", GGML_Q8_0, (shape.n_ff, E))]
    return plan


def _nbytes(typ: int, ne) -> int:
    n = int(np.prod(ne))
    return n * 4 if typ == GGML_F32 else n * 2 if typ == GGML_F16 else n // 32 * 34


def _header(shape: Qwen2Shape, alignment: int):
    """GGUF v3 header bytes (padded to `alignment`) and [(name, type, ne, data offset)]."""
    plan = _tensor_plan(shape)
    kvs = [
        _kv("general.architecture", T_STR, "qwen2"),
        _kv("general.name", T_STR, "random-init-qwen2"),
        _kv("general.alignment", T_U32, alignment),
        _kv("qwen2.context_length", T_U32, shape.n_ctx_train),
        _kv("qwen2.embedding_length", T_U32, shape.n_embd),
        _kv("qwen2.block_count", T_U32, shape.n_layer),
        _kv("qwen2.feed_forward_length", T_U32, shape.n_ff),
        _kv("qwen2.attention.head_count", T_U32, shape.n_head),
        _kv("qwen2.attention.head_count_kv", T_U32, shape.n_head_kv),
        _kv("qwen2.rope.freq_base", T_F32, shape.rope_freq_base),
        _kv("qwen2.attention.layer_norm_rms_epsilon", T_F32, shape.rms_eps),
        _kv("tokenizer.ggml.model", T_STR, "gpt2"),
        _kv("tokenizer.ggml.tokens", T_ARR, (T_STR, [f"t{i}" for i in range(shape.n_vocab)])),
        _kv("tokenizer.ggml.token_type", T_ARR, (T_I32, [1] * shape.n_vocab)),
    ]
    infos, offsets, offset = [], [], 0
    for name, typ, ne in plan:
        infos.append(_str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
                     + struct.pack("<IQ", typ, offset))
        offsets.append(offset)
        offset += _nbytes(typ, ne)
        offset = (offset + alignment - 1) // alignment * alignment
    header = GGUF_MAGIC + struct.pack("<IQQ", 3, len(plan), len(kvs)) + b"".join(kvs) + b"".join(infos)
    header += b"\0" * ((-len(header)) % alignment)
    return header, [(n, t, ne, o) for (n, t, ne), o in zip(plan, offsets)], offset


def write_qwen2_gguf(path: str, shape: Qwen2Shape, seed: int, std: float = 0.02,
                     alignment: int = 32, chunk_rows: int = 8192) -> None:
    """Write a random-init Q8_0 Qwen2 GGUF v3 file (deterministic in `seed`):
    numpy PCG64 stream, norm weights 1.0, every other value N(0, std)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    header, plan, _ = _header(shape, alignment)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header)
        written = 0
        for name, typ, ne, _off in plan:
            if typ == GGML_F32:
                if name.endswith("norm.weight"):
                    data = np.ones(ne, dtype=np.float32)
                else:
                    data = (rng.standard_normal(ne, dtype=np.float32) * np.float32(std)).astype(np.float32)
                f.write(data.tobytes())
            else:
                k, n = ne
                for r0 in range(0, n, chunk_rows):
                    r1 = min(n, r0 + chunk_rows)
                    w = rng.standard_normal((r1 - r0, k), dtype=np.float32) * np.float32(std)
                    quantize_q8_0(w).tofile(f)
            written += _nbytes(typ, ne)
            p = (-written) % alignment
            f.write(b"\0" * p)
            written += p
    os.replace(tmp, path)


GEN_BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "mi_gguf_gen")


def write_qwen2_gguf_fast(path: str, shape: Qwen2Shape, seed: int, std: float = 0.02,
                          alignment: int = 32, threads: int | None = None) -> None:
    """The same file layout as write_qwen2_gguf, with the tensor data filled by
    the multithreaded lib/mi_gguf_gen (its own seeded per-row streams, so the
    values differ from the numpy writer's; the bytes do not depend on the
    thread count). A 7B-shape file takes seconds instead of tens of minutes."""
    if not os.path.exists(GEN_BIN):
        raise FileNotFoundError(f"{GEN_BIN} is missing: run __graft_entry__.build()")
    header, plan, data_bytes = _header(shape, alignment)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header)
        f.truncate(len(header) + data_bytes)
    plan_path = tmp + ".plan"
    with open(plan_path, "w") as f:
        for i, (name, typ, ne, off) in enumerate(plan):
            ne0, ne1 = (ne[0], ne[1]) if len(ne) == 2 else (ne[0], 1)
            ones = 1 if name.endswith("norm.weight") else 0
            f.write(f"{i} {typ} {ne0} {ne1} {len(header) + off} {ones}\n")
    n = threads or os.cpu_count() or 1
    try:
        subprocess.run([GEN_BIN, tmp, plan_path, str(seed), repr(float(std)), str(n)], check=True)
    finally:
        os.remove(plan_path)
    os.replace(tmp, path)


def ensure_qwen2_gguf(path: str, shape: Qwen2Shape, seed: int, fast: bool = False) -> str:
    """Write the model once; later calls reuse the file if it is complete.
    fast=True uses write_qwen2_gguf_fast (a different, equally seeded file)."""
    if not os.path.exists(path):
        d = os.path.dirname(path)
        if d:
            os.makedirs(d, exist_ok=True)
        (write_qwen2_gguf_fast if fast else write_qwen2_gguf)(path, shape, seed)
    return path


# ---------------------------------------------------------------------------
# Reader
# ---------------------------------------------------------------------------

@dataclasses.dataclass
class GGUFTensor:
    name: str
    ggml_type: int
    ne: tuple
    offset: int
    data: np.ndarray  # uint8 view of the tensor's bytes inside the mmap


class GGUFFile:
    """Minimal zero-copy GGUF v3 reader (mmap)."""

    def __init__(self, path: str):
        self.path = path
        fd = os.open(path, os.O_RDONLY)
        try:
            self._mm = mmap.mmap(fd, 0, access=mmap.ACCESS_READ)
        finally:
            os.close(fd)
        buf = memoryview(self._mm)
        pos = 0

        def rd(fmt):
            nonlocal pos
            v = struct.unpack_from(fmt, buf, pos)
            pos += struct.calcsize(fmt)
            return v[0] if len(v) == 1 else v

        def rstr():
            nonlocal pos
            n = rd("<Q")
            s = bytes(buf[pos:pos + n]).decode("utf-8", "replace")
            pos += n
            return s

        def rval(t):
            nonlocal pos
            if t == T_STR:
                return rstr()
            if t == T_ARR:
                et, n = rd("<I"), rd("<Q")
                if et == T_STR:
                    return [rstr() for _ in range(n)]
                dt = np.dtype(_SCALAR_FMT[et][1:]).newbyteorder("<")
                a = np.frombuffer(buf, dtype=dt, count=n, offset=pos)
                pos += n * dt.itemsize
                return a
            return rd(_SCALAR_FMT[t])

        if bytes(buf[0:4]) != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file (bad magic)")
        pos = 4
        self.version = rd("<I")
        if self.version != 3:
            raise ValueError(f"{path}: unsupported GGUF version {self.version}")
        n_tensors, n_kv = rd("<Q"), rd("<Q")
        self.kv = {}
        for _ in range(n_kv):
            key = rstr()
            self.kv[key] = rval(rd("<I"))
        self.alignment = int(self.kv.get("general.alignment", 32))
        raw = []
        for _ in range(n_tensors):
            name = rstr()
            nd = rd("<I")
            ne = tuple(struct.unpack_from(f"<{nd}Q", buf, pos))
            pos += 8 * nd
            typ, off = rd("<I"), rd("<Q")
            raw.append((name, typ, ne, off))
        data_start = (pos + self.alignment - 1) // self.alignment * self.alignment
        self.data_offset = data_start
        self.tensors = {}
        whole = np.frombuffer(self._mm, dtype=np.uint8)
        for name, typ, ne, off in raw:
            nb = _nbytes(typ, ne)
            start = data_start + off
            self.tensors[name] = GGUFTensor(name, typ, ne, start, whole[start:start + nb])

    def shape(self) -> Qwen2Shape:
        kv = self.kv
        E = int(kv["qwen2.embedding_length"])
        return Qwen2Shape(n_layer=int(kv["qwen2.block_count"]), n_embd=E,
                          n_head=int(kv["qwen2.attention.head_count"]),
                          n_head_kv=int(kv["qwen2.attention.head_count_kv"]),
                          n_ff=int(kv["qwen2.feed_forward_length"]),
                          n_vocab=int(self.tensors["token_embd.weight"].ne[1]),
                          tied="output.weight" not in self.tensors,
                          rms_eps=float(kv["qwen2.attention.layer_norm_rms_epsilon"]),
                          rope_freq_base=float(kv["qwen2.rope.freq_base"]),
                          n_ctx_train=int(kv["qwen2.context_length"]))

    def f32(self, name: str) -> np.ndarray:
        return self.tensors[name].data.view(np.float32)

    def raw(self, name: str) -> np.ndarray:
        return self.tensors[name].data

    def close(self):
        self.tensors = {}
        try:
            self._mm.close()
        except BufferError:
            pass
