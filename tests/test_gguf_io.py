"""The random-init GGUF writer and the reader: the reference's own loader
accepts the files (hyperparameters, tied/untied lm_head), the numpy Q8_0
quantizer round-trips, and the reader sees what the writer wrote."""
import numpy as np

import mi_gguf
import mi_oracle


def test_writer_reader_roundtrip(tmp_path):
    p = str(tmp_path / "t.gguf")
    mi_gguf.write_qwen2_gguf(p, mi_gguf.TINY, seed=3)
    g = mi_gguf.GGUFFile(p)
    assert g.version == 3 and g.alignment == 32
    sh = g.shape()
    assert (sh.n_layer, sh.n_embd, sh.n_head, sh.n_head_kv, sh.n_ff, sh.n_vocab, sh.tied) == (2, 64, 4, 2, 128, 256, True)
    assert np.float32(sh.rms_eps) == np.float32(1e-6) and sh.rope_freq_base == 1e6
    assert g.tensors["token_embd.weight"].ne == (64, 256)
    assert g.tensors["blk.1.ffn_down.weight"].ne == (128, 64)
    assert np.all(g.f32("output_norm.weight") == 1.0)
    assert len(g.kv["tokenizer.ggml.tokens"]) == 256
    for t in g.tensors.values():
        assert t.offset % 32 == 0


def test_writer_is_deterministic(tmp_path):
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    mi_gguf.write_qwen2_gguf(a, mi_gguf.TINY, seed=9)
    mi_gguf.write_qwen2_gguf(b, mi_gguf.TINY, seed=9)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_reference_loader_accepts_files(tmp_path):
    for shape in (mi_gguf.TINY, mi_gguf.Qwen2Shape(n_layer=1, n_embd=64, n_head=2, n_head_kv=1,
                                                    n_ff=96, n_vocab=128, tied=False)):
        p = str(tmp_path / f"m{shape.n_ff}.gguf")
        mi_gguf.write_qwen2_gguf(p, shape, seed=1)
        m = mi_oracle.ReferenceModel(p, n_ctx=32)
        assert (m.n_vocab, m.n_embd, m.n_layer) == (shape.n_vocab, shape.n_embd, shape.n_layer)
        logits = m.forward([1, 2, 3], 0)
        assert logits.shape == (3, shape.n_vocab) and np.all(np.isfinite(logits))
        m.close()


def test_quantizer_roundtrip_error_bound():
    rng = np.random.default_rng(7)
    x = rng.uniform(-3, 3, (5, 32 * 4)).astype(np.float32)
    q = mi_gguf.quantize_q8_0(x)
    back = mi_gguf.dequantize_q8_0(q).reshape(x.shape)
    d = q["d"].astype(np.float32).reshape(5, 4)
    assert np.all(np.abs(back - x).reshape(5, 4, 32) <= d[..., None] * 0.5 + 1e-3)
    assert np.all(np.abs(q["qs"]) <= 127)


def test_fast_writer_matches_layout_and_is_thread_invariant(tmp_path):
    """The multithreaded writer (lib/mi_gguf_gen) produces the numpy writer's
    header byte for byte, the same file size, bytes independent of the thread
    count, N(0, 0.02) weights, 1.0 norms, and a file the reference loads."""
    shape = mi_gguf.SMALL
    a, b, c = (str(tmp_path / n) for n in ("a.gguf", "b.gguf", "c.gguf"))
    mi_gguf.write_qwen2_gguf_fast(a, shape, seed=9, threads=1)
    mi_gguf.write_qwen2_gguf_fast(b, shape, seed=9, threads=5)
    mi_gguf.write_qwen2_gguf(c, shape, seed=9)
    da, db, dc = (open(p, "rb").read() for p in (a, b, c))
    header, _, _ = mi_gguf._header(shape, 32)
    assert da == db
    assert len(da) == len(dc) and da[:len(header)] == dc[:len(header)]
    g = mi_gguf.GGUFFile(a)
    w = mi_gguf.dequantize_q8_0(g.raw("blk.1.ffn_gate.weight").view(mi_gguf.Q8_0_DTYPE))
    assert abs(float(w.std()) - 0.02) < 1e-3 and abs(float(w.mean())) < 1e-3
    assert np.all(g.f32("blk.1.ffn_norm.weight") == 1.0)
    bias = g.f32("blk.0.attn_k.bias")
    assert bias.std() > 0.01 and np.isfinite(bias).all()
    g.close()
    m = mi_oracle.ReferenceModel(a, n_ctx=16)
    logits = m.forward(np.array([1, 2, 3], dtype=np.int32), 0, last_logits_only=True)
    assert np.isfinite(logits).all()
