"""The bench's algorithmic byte and MAC counts against the figures derived from
the model shapes: a decode step reads every weight once (Q8_0 at 34/32 B per
weight, F32 norms and biases), one embedding row, and the K/V rows; a prefill
multiplies every projection by every token and the LM head by the last."""
import importlib.util
import os

import mi_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _HP:
    def __init__(self, s):
        self.n_embd, self.head_dim, self.n_ff = s.n_embd, s.head_dim, s.n_ff
        self.n_layer, self.n_vocab, self.n_head_kv = s.n_layer, s.n_vocab, s.n_head_kv


def test_decode_step_bytes():
    b = _bench()
    hp05 = _HP(mi_gguf.QWEN2_05B)
    # weights + norms/biases + embedding row: 525,120,952 B; KV: 24,576 B per position
    assert b.step_bytes(hp05, 0) - 24576 == 525_120_952
    assert b.step_bytes(hp05, 96) - b.step_bytes(hp05, 95) == 24576
    hp7 = _HP(mi_gguf.QWEN2_7B)
    assert b.step_bytes(hp7, 0) - 114688 == 7_513_515_744
    assert b.step_bytes(hp7, 1) - b.step_bytes(hp7, 0) == 114688


def test_prefill_macs():
    b = _bench()
    hp05 = _HP(mi_gguf.QWEN2_05B)
    per_token = 357_826_560  # 24 layers x (QKV + O + gate/up + down) int8 MACs
    head = 151936 * 896
    assert b.prefill_macs(hp05, 1) == per_token + head
    assert b.prefill_macs(hp05, 1024) == 1024 * per_token + head


def test_reference_arms_for_ops_print_json(capsys):
    """Configs 1 and 2 on the reference's own single-thread ops print one line
    per shape with the metric fields the GPU arms print."""
    import json
    import types
    b = _bench()
    args = types.SimpleNamespace(shapes="128x896", nkv="64", config="gemv")
    b.run_reference_arm(args, 0)
    args.config = "attention"
    b.run_reference_arm(args, 0)
    b.run_reference_arm(args, 1)  # other ranks print nothing
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert [d["config"] for d in lines] == ["gemv", "attention"]
    for d in lines:
        assert d["impl"] == "reference" and d["cores"] == 1
        assert d["us_per_call"] > 0 and d["achieved_gbs"] > 0
    assert lines[0]["bytes_per_call"] == 128 * 896 // 32 * 34 + 896 // 32 * 36 + 4 * 128 + 4 * 896
    assert lines[1]["bytes_per_call"] == 2 * 64 * 2 * 64 * 4 + 2 * 14 * 64 * 4


def test_decode_config_is_the_same_on_both_arms():
    """The reference arm and the GPU arm describe the decode workload with one
    dict, so a comparison of their lines sees the same configuration."""
    b = _bench()
    c = b.decode_config()
    assert c == b.decode_config()
    assert c["n_ctx"] == 2048 and c["prompt"] == 32 and c["n_predict"] == 128


def test_fast_mode_argmax_agreement():
    """The fast-mode object's statistics on crafted logits: a flip at a near
    tie (gap inside the typical error) passes the gap check; a flip of a clear
    winner by one outlying error fails it."""
    import numpy as np
    b = _bench()
    rng = np.random.default_rng(0)
    exact = rng.standard_normal((8, 4000)).astype(np.float32)
    exact[:, 0] = 10.0                                    # a clear winner at every position
    noise = (rng.standard_normal(exact.shape) * 1e-3).astype(np.float32)
    fast = exact + noise                                  # typical error ~3e-3 at the 99.9th percentile
    exact[3, 1] = 10.0 - 1e-3                             # position 3: a near tie...
    fast[3, 1] = 10.0 + 1e-3                              # ...that the fast mode resolves the other way
    fast[3, 0] = 10.0 - 1e-3
    r = b.argmax_agreement(fast, exact)
    assert r["n_positions"] == 8 and r["disagreements"] == 1 and r["teacher_forced"] == 7 / 8
    assert r["gap_check"] and r["disagree_max_exact_gap"] < 2e-3
    assert r["exact_top2_gap_median"] > 5.0
    bad = fast.copy()
    bad[5, 7] = 12.0                                      # one outlier overturns position 5's winner (gap ~10)
    r2 = b.argmax_agreement(bad, exact)
    assert r2["disagreements"] == 2 and not r2["gap_check"]
    assert r2["max_abs_logit_diff"] > 10.0 and r2["p999_abs_logit_diff"] < 0.01
