"""Golden fixtures recorded from the reference itself (tests/golden/golden.json,
written by tests/golden/make_golden.py from the reference compiled from
source). The inputs are regenerated from their seeds (their digests are
checked first), then the oracle restatement (CPU) and the CUDA path (GPU) must
reproduce the reference's output bytes exactly."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN, MODEL_DIR

sys.path.insert(0, GOLDEN)
import make_golden as mg  # noqa: E402
import mi_gguf  # noqa: E402
import mi_oracle  # noqa: E402

G = json.load(open(os.path.join(GOLDEN, "golden.json")))
sha = mg.sha


def _gguf(entry):
    path = os.path.join(MODEL_DIR, f"golden_{entry['shape'].lower()}_{entry['seed']}.gguf")
    mi_gguf.ensure_qwen2_gguf(path, getattr(mi_gguf, entry["shape"]), entry["seed"])
    assert sha(np.fromfile(path, np.uint8)) == entry["gguf"], "model generator output changed"
    return path


@pytest.mark.parametrize("e", G["gemv"], ids=lambda e: f"{e['n']}x{e['k']}")
def test_gemv_restatement(e):
    w, x = mg.gemv_inputs(e["n"], e["k"])
    assert sha(w) + sha(x) == e["inputs"], "input generator changed"
    S = mi_oracle.Restatement()
    act = S.quantize_act(x)
    assert sha(act) == e["act"]
    assert sha(S.mul_mat(w, e["k"], e["n"], act, 1)) == e["out"]


@pytest.mark.parametrize("e", G["attention"], ids=lambda e: f"nkv{e['n_kv']}")
def test_attention_restatement(e):
    q, k, v = mg.attn_inputs(e["n_kv"])
    assert sha(q) + sha(k) + sha(v) == e["inputs"]
    s, p, o = mi_oracle.Restatement().attention(q, k, v, 2, e["n_kv"] - 1, 1, 0.125)
    assert (sha(s), sha(p), sha(o)) == (e["scores"], e["probs"], e["out"])


@pytest.mark.parametrize("e", G["models"], ids=lambda e: e["shape"])
def test_model_restatement(e):
    path = _gguf(e)
    rs = mi_oracle.RestatedModel(mi_gguf.GGUFFile(path), n_ctx=e["n_ctx"])
    prompt = np.array(e["prompt"], dtype=np.int32)
    logits = rs.forward(prompt, 0)
    assert sha(logits) == e["prefill_logits"]
    toks = [int(np.argmax(logits[-1]))]
    n_past = prompt.size
    while len(toks) < len(e["greedy_tokens"]):
        lg = rs.forward([toks[-1]], n_past)
        n_past += 1
        toks.append(int(np.argmax(lg[0])))
    assert toks == e["greedy_tokens"]


@pytest.mark.gpu
@pytest.mark.parametrize("e", G["gemv"], ids=lambda e: f"{e['n']}x{e['k']}")
def test_gemv_cuda(torch_cuda, e):
    import mi_cuda
    torch = torch_cuda
    w, x = mg.gemv_inputs(e["n"], e["k"])
    wp = mi_cuda.q8_0_pack(torch.from_numpy(w.reshape(-1)).cuda(), e["k"], e["n"])
    X = torch.from_numpy(x).cuda()
    act = mi_cuda.quantize_act(X, e["k"])
    assert sha(act.cpu().numpy()) == e["act"]
    assert sha(mi_cuda.mul_mat(wp, e["k"], e["n"], x=X).cpu().numpy()) == e["out"]
    assert sha(mi_cuda.block_isums(wp, e["k"], e["n"], act).cpu().numpy()) == e["isums"]


@pytest.mark.gpu
@pytest.mark.parametrize("e", G["attention"], ids=lambda e: f"nkv{e['n_kv']}")
def test_attention_cuda(torch_cuda, e):
    import mi_cuda
    torch = torch_cuda
    q, k, v = mg.attn_inputs(e["n_kv"])
    o = mi_cuda.attention_decode(torch.from_numpy(q[0]).cuda(), torch.from_numpy(k).cuda(),
                                 torch.from_numpy(v).cuda(), 2, e["n_kv"], 0.125)
    assert sha(o.cpu().numpy()) == e["out"]


@pytest.mark.gpu
@pytest.mark.parametrize("e", G["models"], ids=lambda e: e["shape"])
def test_model_cuda(torch_cuda, e):
    import mi_cuda
    path = _gguf(e)
    model = mi_cuda.Qwen2Model(path)
    kv = mi_cuda.KVCache(model, e["n_ctx"])
    prompt = np.array(e["prompt"], dtype=np.int32)
    assert sha(kv.forward(prompt, 0)) == e["prefill_logits"]
    toks, _, _ = kv.generate(prompt, len(e["greedy_tokens"]))
    assert toks.tolist() == e["greedy_tokens"]
    kv.free()
    model.free()
