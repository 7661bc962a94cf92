"""Generates tests/golden/golden.json from the reference itself.

Runs the reference's own code (compiled from its sources into
oracle/_ref/libmi_ref.so by oracle/Makefile) on seeded synthetic inputs and
records SHA-256 digests of the exact output bytes, plus a few readable values.
The fixture is small and travels with the repository; the tests regenerate the
same inputs from the seeds (their digests are recorded too, so a change in the
input generator is reported as such) and check the oracle restatement and the
CUDA path against the reference's bytes.

  python tests/golden/make_golden.py          (needs oracle/_ref/libmi_ref.so)
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mini-infer-llama.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import mi_gguf  # noqa: E402

GEMV_SHAPES = [(896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896)]
ATTN_NKV = [128, 1024, 4096, 32768]
MODELS = [("TINY", 1, 64, 9, 40), ("SMALL", 4, 256, 16, 64)]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gemv_inputs(n, k):
    rng = np.random.default_rng(1000 + n + 7 * k)
    w = mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
    x = rng.standard_normal((1, k), dtype=np.float32)
    return w, x


def attn_inputs(n_kv):
    rng = np.random.default_rng(2000 + n_kv)
    H, HKV, D = 14, 2, 64
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    k = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    v = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
    return q, k, v


def model_prompt(seed, n_vocab, n):
    return np.random.default_rng(3000 + seed).integers(0, n_vocab, n).astype(np.int32)


def main():
    import mi_oracle
    R = mi_oracle.Reference()
    out = {"generator": "tests/golden/make_golden.py", "source": "reference compiled from source (oracle/_ref/libmi_ref.so)",
           "gemv": [], "attention": [], "models": []}
    for n, k in GEMV_SHAPES:
        w, x = gemv_inputs(n, k)
        act, y = R.mul_mat(w, k, n, x)
        wq = w.reshape(n, k // 32, 34)[:, :, 2:].view(np.int8).astype(np.int64)
        aq = act.reshape(k // 32, 36)[:, 4:].view(np.int8).astype(np.int64)
        isums = (wq * aq[None]).sum(-1).astype(np.int32)
        out["gemv"].append({"n": n, "k": k, "inputs": sha(w) + sha(x), "act": sha(act), "out": sha(y),
                            "isums": sha(isums), "out_head": [float(v) for v in y[0, :4]]})
    for n_kv in ATTN_NKV:
        q, k, v = attn_inputs(n_kv)
        s, p, o = R.attention(q, k, v, 2, n_kv - 1, 1, 0.125)
        out["attention"].append({"n_kv": n_kv, "inputs": sha(q) + sha(k) + sha(v), "scores": sha(s),
                                 "probs": sha(p), "out": sha(o), "out_head": [float(x) for x in o[0, 0, :4]]})
    for shape, seed, n_ctx, n_prompt, n_predict in MODELS:
        path = os.path.join("/tmp", f"mi_golden_{shape.lower()}_{seed}.gguf")
        mi_gguf.write_qwen2_gguf(path, getattr(mi_gguf, shape), seed)
        m = mi_oracle.ReferenceModel(path, n_ctx=n_ctx)
        prompt = model_prompt(seed, m.n_vocab, n_prompt)
        logits = m.forward(prompt, 0)
        m.close()
        m = mi_oracle.ReferenceModel(path, n_ctx=n_ctx)
        toks, _, _ = m.generate(prompt, n_predict)
        m.close()
        out["models"].append({"shape": shape, "seed": seed, "n_ctx": n_ctx, "gguf": sha(np.fromfile(path, np.uint8)),
                              "prompt": prompt.tolist(), "prefill_logits": sha(logits),
                              "last_logits_head": [float(x) for x in logits[-1, :4]],
                              "greedy_tokens": [int(t) for t in toks]})
        os.remove(path)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
