"""Decode benchmark: Qwen2.5-0.5B-shape Q8_0 greedy decode at ctx 2048.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token: one replay of the captured decode-step graph
(embedding, 24 layers, LM head, greedy argmax fed back on the device). The
workload: random-init 0.5B-shape Q8_0 GGUF (seed 1234), a 32-token
uniform-random prompt (seed 7), greedy decode at positions 32..158 (the
reference CLI's 127 decode forwards of a 128-token run); a run of K steps
cycles through that position range on the device.

Printed JSON (rank 0, one line):
  value     device-timed decode tok/s (CUDA events on the executor stream,
            weights resident in HBM; 527 MB of weights per step > 126 MB L2)
  e2e       the same metric through the public per-token API: every step the
            token H2D from pinned memory, mi_cuda_qwen2_forward, and the greedy
            token D2H (mi_cuda_qwen2_last_token); e2e_logits reads the logits
            row instead and samples on the host, as the reference's loop does
  roofline  algorithmic bytes per decode step / step time vs the measured
            HBM copy bandwidth (MEASURED_PEAKS.json)
  parity    the 128 greedy tokens of one full untimed generation (127 decode
            steps from the prompt) against the reference's, whatever K is
  cpu_baseline  the reference's own CPU decode (compiled from its sources,
            oracle/_ref) on this host's cores, same model and prompt
  tp7b      the 7B-shape decode row-sharded over all N ranks (one request):
            tok/s, ms per token, GB/s, greedy-token parity
  sweeps    (N = 1) the isolated GEMV shapes (GB/s, cold), decode attention
            at n_kv 128..32768 (µs), the 1024-token prefill (tok/s)
With --gpus N > 1 (torchrun) every rank runs an independent 0.5B replica (the
0.5B decode does not shard; value is the sum of tokens over the max time), and
then all ranks run the 7B shape together, row-sharded (the tp7b object).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mini-infer-llama.cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import mi_gguf  # noqa: E402

def _model_dir() -> str:
    """Where the seeded GGUF files are written: MI_B200_MODEL_DIR, else a RAM
    file system with room for the 7.5 GB 7B-shape file (writing it to a slow
    disk took minutes), else /tmp."""
    if os.environ.get("MI_B200_MODEL_DIR"):
        return os.environ["MI_B200_MODEL_DIR"]
    try:
        st = os.statvfs("/dev/shm")
        if st.f_bavail * st.f_frsize > 24 * 2 ** 30:
            return "/dev/shm/mi_b200_models"
    except OSError:
        pass
    return "/tmp/mi_b200_models"


MODEL_DIR = _model_dir()
SEED_MODEL, SEED_PROMPT = 1234, 7
N_CTX, N_PROMPT, N_PREDICT = 2048, 32, 128
PERIOD = N_PREDICT - 1  # decode forwards per generated sequence
METRIC = "decode tok/s (0.5B-shape Q8_0, ctx 2048)"
PUBLISHED_BEST = 64.035  # reference Q8_0 decode tok/s, 4 threads (reference README.md:106)
# DRAM bytes (read + write) of one decode step: dram__bytes_read.sum +
# dram__bytes_write.sum of one launch of the persistent step kernel (the whole
# step) at n_kv = 34, from an ncu capture of this build;
# profiles/decode_step_qwen2_05b.md gives the command and the figures.
TRAFFIC_PER_STEP = 531_855_872
TRAFFIC_SOURCE = "ncu dram__bytes_read+write of one persistent-step launch at n_kv 34 (527.1 MB read, 4.7 MB written)"


def step_bytes(hp, n_kv: int) -> int:
    """Algorithmic HBM bytes of one decode step: every weight once (Q8_0 at
    34/32 B per weight, F32 norms and biases), one embedding row, the KV rows
    read (n_kv positions) and written (one)."""
    E, D, FF, L, V = hp.n_embd, hp.head_dim, hp.n_ff, hp.n_layer, hp.n_vocab
    kvd = hp.n_head_kv * D
    q8 = lambda n: n * 34 // 32
    per_layer = q8(E * E * 2 + E * kvd * 2 + E * FF * 3) + (2 * E + E + 2 * kvd) * 4
    return L * per_layer + q8(V * E) + E * 4 + q8(E) + L * 2 * kvd * 4 * (n_kv + 1)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 100 ms while the
    context is open. The bench opens it before the warm-up and closes it after
    the untimed passes that follow the timed region (parity, e2e), so a timed
    region of a few milliseconds still lies inside a sampled busy span."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout_s: float = 3.0):
        """Blocks until the first sample arrived (nvidia-smi takes a moment to
        start), so the span that follows is sampled from its beginning."""
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout_s:
            time.sleep(0.02)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def ensure_model(rank: int, dist) -> str:
    path = os.path.join(MODEL_DIR, f"qwen2_05b_seed{SEED_MODEL}.gguf")
    if rank == 0:
        mi_gguf.ensure_qwen2_gguf(path, mi_gguf.QWEN2_05B, SEED_MODEL)
    if dist is not None:
        dist.barrier()
    return path


def prompt_ids(n_vocab: int) -> np.ndarray:
    return np.random.default_rng(SEED_PROMPT).integers(0, n_vocab, N_PROMPT).astype(np.int32)


def reference_decode(path: str, steps: int, warmup: int, threads: int):
    """The reference's own decode loop (mi_qwen2_forward + greedy, its --bench
    loop) on `threads` host threads; returns (tok/s, tokens of one sequence, sample)."""
    import mi_oracle
    m = mi_oracle.ReferenceModel(path, n_ctx=N_CTX, n_threads=threads)
    prompt = prompt_ids(m.n_vocab)
    if warmup > 0:
        m.generate(prompt, min(N_PREDICT, warmup + 1))
    total_ms, total_steps, first = 0.0, 0, None
    while total_steps < steps:
        n = min(PERIOD, steps - total_steps)
        toks, _, dms = m.generate(prompt, n + 1)
        if first is None:
            first = toks
        total_ms += dms
        total_steps += n
    m.close()
    return total_steps / (total_ms / 1e3), first, f"{total_steps} decode forwards at positions 32..158, {threads} threads"


def persist_trace_summary(kv) -> dict:
    """Phase timeline of the last timed persistent step (one kernel): per
    layer, from attention CTA 0 (the attention cluster also runs the O
    projection) and the first projection CTA, means over the layers in
    microseconds."""
    t = kv.step_trace().astype(np.int64)
    L = kv.model.hparams.n_layer
    a, g, h = t[0:2 * L:2], t[1:2 * L:2], t[2 * L]
    us = lambda v: float(np.mean(v)) / 1e3
    return {
        "schedule": "persistent (one kernel per step; attention + O on one cluster)",
        "step_us": float(h[2] - a[0, 0]) / 1e3,
        "per_layer_us": us(np.diff(a[:, 1])) if L > 1 else None,
        "attention_cta_us": {"x_wait": us(a[1:, 1] - g[:-1, 6]) if L > 1 else None,
                             "norm_quant": us(a[:, 2] - a[:, 1]), "qkv_rows": us(a[:, 3] - a[:, 2]),
                             "kv_handover": us(a[:, 4] - a[:, 3]), "scores_exp": us(a[:, 5] - a[:, 4]),
                             "softmax_sum": us(a[:, 6] - a[:, 5]),
                             "values_exchange_o": us(a[:, 7] - a[:, 6])},
        "projection_cta_us": {"gate_up_wait_after_o": us(g[:, 2] - a[:, 7]),
                              "gate_up_norm_quant": us(g[:, 3] - g[:, 2]),
                              "gate_up_rows": us(g[:, 4] - g[:, 3]), "down_wait": us(g[:, 5] - g[:, 4]),
                              "down": us(g[:, 6] - g[:, 5])},
        "lm_head_us": {"wait": float(h[0] - g[-1, 6]) / 1e3, "norm_quant": float(h[1] - h[0]) / 1e3,
                       "rows_argmax": float(h[2] - h[1]) / 1e3, "of_which_ring_wait": float(h[4]) / 1e3,
                       "of_which_rows": float(h[5]) / 1e3, "of_which_free_issue": float(h[6]) / 1e3,
                       "ring_items": int(h[7])}}


def step_trace_summary(kv) -> dict:
    """Per-kernel timeline of the last timed step (first CTA of each kernel):
    dependency wait -> prologue done, prologue -> epilogue, hand-off from the
    predecessor, and the attention phases."""
    if kv.kernels_per_step == 1:
        return persist_trace_summary(kv)
    t = kv.step_trace().astype(np.int64)
    per = (t.shape[0] - 1) // kv.model.hparams.n_layer
    # 4 kernels a layer when QKV and attention run as one cluster kernel
    names = ["qkv_attn", "o", "gate_up", "down"] if per == 4 else ["qkv", "attn", "o", "gate_up", "down"]
    kinds = [names[i % per] for i in range(t.shape[0] - 1)] + ["lm_head"]
    trace = {"step_us": float(t[-1, 3] - t[0, 0]) / 1e3, "per_kernel_us": {}}
    for k in dict.fromkeys(kinds):
        idx = [i for i, kk in enumerate(kinds) if kk == k]
        dep = [t[i, 1] - t[i - 1, 3] for i in idx if i > 0]  # wait after the predecessor's epilogue started
        trace["per_kernel_us"][k] = {
            "dep_to_prologue": float(np.mean([t[i, 2] - t[i, 1] for i in idx])) / 1e3,
            "prologue_to_epilogue": float(np.mean([t[i, 3] - t[i, 2] for i in idx])) / 1e3,
            "handoff": float(np.mean(dep)) / 1e3 if dep else None}
    if per == 4:
        # fused kernel marks: 2 prologue, 4 k/v handed over, 5 scores, 6 exp, 7 sum, 3 KV done
        ai = [i for i, kk in enumerate(kinds) if kk == "qkv_attn"]
        phases = (("qkv_rows_and_handover", 2, 4), ("scores", 4, 5), ("max_exp", 5, 6), ("sum", 6, 7),
                  ("kv", 7, 3))
    else:
        ai = [i for i, kk in enumerate(kinds) if kk == "attn"]
        phases = (("scores", 2, 4), ("max_exp", 4, 5), ("sum", 5, 6), ("kv", 6, 7))
    trace["attention_phases_us"] = {
        name: float(np.mean([t[i, b] - t[i, a] for i in ai])) / 1e3 for name, a, b in phases}
    return trace




def argmax_agreement(fast: np.ndarray, exact: np.ndarray) -> dict:
    """Teacher-forced agreement of two [positions, vocab] logit arrays: the
    share of positions whose greedy argmax matches, the logit error, and the
    gap-aware check. A flip always needs the two logits involved to move by
    half the exact gap between them, so the check compares each
    disagreement's exact gap (exact top logit minus the exact logit of the
    fast mode's pick) with the TYPICAL error, twice the 99.9th percentile of
    |fast - exact| over all logits: a disagreement passes only at a near tie,
    not where a few outlying errors overturned a clear winner. The median
    exact top-two gap gives the scale of a clear winner."""
    fa, ea = np.argmax(fast, axis=1), np.argmax(exact, axis=1)
    rows = np.arange(fast.shape[0])
    diff = np.abs(fast.astype(np.float64) - exact)
    mad = float(np.max(diff))
    typ = float(np.quantile(diff, 0.999))
    a, b = fast.astype(np.float64).ravel(), exact.astype(np.float64).ravel()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    gaps = (exact[rows, ea] - exact[rows, fa])[fa != ea]
    top2 = np.sort(exact, axis=1)[:, -2:]
    return {"teacher_forced": float(np.mean(fa == ea)), "n_positions": int(fast.shape[0]),
            "disagreements": int(gaps.size), "max_abs_logit_diff": mad, "p999_abs_logit_diff": typ, "cos": cos,
            "disagree_max_exact_gap": float(gaps.max()) if gaps.size else None,
            "exact_top2_gap_median": float(np.median(top2[:, 1] - top2[:, 0])),
            "gap_check": bool(np.all(gaps <= 2 * typ))}


def fast_mode_measure(args, kv, seed_tokens, exact_gen, stream, dist, local: int, world: int, hp,
                      peak: float, peak_kind: str) -> dict:
    """The labelled fast mode of the decode step (mi_cuda_qwen2_set_fast_mode:
    regrouped sums, CUDA expf; never the parity result): the same timed decode
    steps, then its accuracy -- teacher-forced on the exact run's 128 tokens,
    the argmax at every position against the exact step's, with the exact
    top-two gap wherever they differ (a disagreement is expected only where
    that gap is within the fast mode's logit error), and the length of the
    identical prefix of a free-running fast greedy generation."""
    import torch
    kv.set_fast_mode(True)
    kv.set_position(seed_tokens, N_PROMPT)
    kv.decode_steps(args.warmup, N_PROMPT, PERIOD)
    torch.cuda.synchronize()
    kv.set_position(seed_tokens, N_PROMPT)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    kv.decode_steps(args.steps, N_PROMPT, PERIOD)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    trace = step_trace_summary(kv) if args.trace else None
    kv.set_position(seed_tokens, N_PROMPT)
    kv.decode_steps(PERIOD)
    free_run = kv.read_tokens(N_PROMPT, N_PREDICT)
    same = free_run == exact_gen
    prefix = int(np.argmin(same)) if not np.all(same) else int(same.size)

    seq = np.concatenate([seed_tokens[:N_PROMPT], exact_gen]).astype(np.int32)

    def teacher_forced():
        return np.stack([kv.forward(seq[N_PROMPT + t:N_PROMPT + t + 1], N_PROMPT + t, last_logits_only=True)[0]
                         for t in range(PERIOD)])

    fast = teacher_forced()
    kv.set_fast_mode(False)
    exact = teacher_forced()
    n_kvs = [N_PROMPT + (i % PERIOD) + 1 for i in range(args.steps)]
    achieved = sum(step_bytes(hp, n) for n in n_kvs) / (ms / 1e3) / 1e9
    out = {
        "label": "fast mode: tree-reduced rms_norm and softmax sums, split value sums and down-projection "
                 "dots, CUDA expf; NOT bit-identical, not the parity result",
        "value": args.steps * world / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / args.steps,
        "steps": args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind},
        "argmax_agreement": {
            **argmax_agreement(fast, exact),
            "run": "exact run's tokens fed back (positions 32..158), fast vs exact step argmax"},
        "free_run": {"tokens_identical_prefix": prefix, "n_tokens": int(exact_gen.size)},
    }
    if trace is not None:
        out["trace"] = trace
    return out


def decode_config() -> dict:
    """The decode workload, the same dict on both arms."""
    return {"workload": "qwen2.5-0.5b-shape Q8_0 greedy decode, ctx 2048, prompt 32, positions 32..158",
            "n_ctx": N_CTX, "prompt": N_PROMPT, "n_predict": N_PREDICT,
            "l2": "inputs larger than L2: 527 MB of weights streamed from HBM every step"}


# ---------------------------------------------------------------------------
# Reference arm: the reference's own CPU code (compiled from its sources into
# oracle/_ref) on this host's cores.
# ---------------------------------------------------------------------------

def _time_host(fn, n_copies: int, budget_s: float, min_calls: int = 3):
    """Seconds per call of fn(copy_index), rotating copies, for about budget_s."""
    fn(0)
    n, t0 = 0, time.perf_counter()
    while n < min_calls or time.perf_counter() - t0 < budget_s:
        fn(n % n_copies)
        n += 1
    return (time.perf_counter() - t0) / n


def reference_gemv_rows(shapes, budget_s: float) -> list:
    """Config 1 on the reference: its quantize + mul_mat nodes (mi_compute_forward,
    one thread, as tools/bench_matvec times them), weights rotated through copies
    larger than the host's last-level cache."""
    import mi_oracle
    R = mi_oracle.Reference()
    rows = []
    for n, k in shapes:
        rng = np.random.default_rng(n + 3 * k)
        wbytes = n * k // 32 * 34
        n_copies = max(1, min(512, -(-256 * 2 ** 20 // wbytes)))  # >= 256 MB of weights in rotation
        ws = [mi_gguf.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).view(np.uint8)
              for _ in range(min(n_copies, 2))]
        ws = [ws[i % len(ws)].copy() for i in range(n_copies)]
        x = rng.standard_normal((1, k), dtype=np.float32)
        sec = _time_host(lambda i: R.mul_mat(ws[i], k, n, x), n_copies, budget_s)
        algo = wbytes + k // 32 * 36 + 4 * n + 4 * k
        rows.append({"shape": f"{n}x{k}", "us_per_call": sec * 1e6, "bytes_per_call": algo,
                     "achieved_gbs": algo / sec / 1e9, "cores": 1,
                     "sample": f"mi_compute_forward quantize + mul_mat, 1 thread, {n_copies} weight copies"})
        del ws
    return rows


def reference_attention_rows(nkvs, budget_s: float) -> list:
    """Config 2 on the reference: its ATTN_QK, SOFTMAX, ATTN_KQV nodes on one
    thread (mi_compute_forward), 14 query / 2 KV heads, head_dim 64."""
    import mi_oracle
    R = mi_oracle.Reference()
    H, HKV, D = 14, 2, 64
    rows = []
    for n_kv in nkvs:
        rng = np.random.default_rng(n_kv)
        q = rng.standard_normal((1, H, D), dtype=np.float32)
        k = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
        v = rng.standard_normal((n_kv, HKV, D), dtype=np.float32)
        sec = _time_host(lambda i: R.attention(q, k, v, HKV, n_kv - 1, 1, 0.125), 1, budget_s, min_calls=2)
        algo = 2 * n_kv * HKV * D * 4 + 2 * H * D * 4
        rows.append({"n_kv": n_kv, "us_per_call": sec * 1e6, "bytes_per_call": algo,
                     "achieved_gbs": algo / sec / 1e9, "cores": 1,
                     "sample": "mi_compute_forward attn_qk + softmax + attn_kqv, 1 thread"})
    return rows


def reference_prefill(path: str, steps: int, threads: int) -> dict:
    """Config 3 on the reference: its mi_qwen2_forward of the 1024-token prompt
    (last logits) on `threads` host threads, after one untimed forward."""
    import mi_oracle
    m = mi_oracle.ReferenceModel(path, n_ctx=N_CTX, n_threads=threads)
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, m.n_vocab, N_PREFILL).astype(np.int32)
    m.forward(prompt, 0, last_logits_only=True)
    t0 = time.perf_counter()
    for _ in range(steps):
        m.forward(prompt, 0, last_logits_only=True)
    s = (time.perf_counter() - t0) / steps
    m.close()
    return {"value": N_PREFILL / s, "unit": "tok/s", "ms_per_prompt": s * 1e3, "cores": threads,
            "sample": f"{steps} forwards of the {N_PREFILL}-token prompt (last logits), {threads} threads"}


def reference_7b(n_dec: int, threads: int) -> dict:
    """Config 4 on the reference: its decode loop over the 7B-shape model on
    `threads` host cores (one process, no GPUs), n_dec decode forwards."""
    import mi_oracle
    path = ensure_7b_model(0, None)
    m = mi_oracle.ReferenceModel(path, n_ctx=N_CTX_7B, n_threads=threads)
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, m.n_vocab, N_PROMPT_7B).astype(np.int32)
    toks, pre_ms, dec_ms = m.generate(prompt, n_dec + 1)
    m.close()
    return {"value": n_dec / (dec_ms / 1e3), "unit": "tok/s", "ms_per_token": dec_ms / n_dec, "cores": threads,
            "tokens": [int(t) for t in toks],
            "sample": f"{n_dec} decode forwards at positions 64..{64 + n_dec - 1} after the 64-token prefill "
                      f"({pre_ms / 1e3:.1f} s), {threads} threads"}


def run_reference_arm(args, rank: int):
    """--impl reference: rank 0 times the reference's CPU path of the chosen
    config on the host cores and prints the line; other ranks exit."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if args.config == "gemv":
        for r in reference_gemv_rows(parse_shapes(args.shapes), 1.0):
            print(json.dumps({"config": "gemv", "impl": "reference", **r}), flush=True)
        return
    if args.config == "attention":
        for r in reference_attention_rows([int(v) for v in args.nkv.split(",")], 1.0):
            print(json.dumps({"config": "attention", "impl": "reference", **r}), flush=True)
        return
    if args.config == "prefill":
        r = reference_prefill(ensure_model(0, None), max(1, min(args.steps, 3)), threads)
        tps = r["value"]
        print(json.dumps({
            "metric": METRIC_PREFILL, "value": tps, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": max(1, min(args.steps, 3)), "warmup": 1, "ms_per_step": r["ms_per_prompt"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": tps / PUBLISHED_PREFILL,
            "dtype": "i8*i8->f32", "data": "synthetic", "config": prefill_config(),
            "parallelism": f"cpu threads x{threads}",
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": r["sample"]},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return
    if args.config == "tp7b":
        r = reference_7b(max(1, min(args.steps, 16)), threads)
        tps = r["value"]
        print(json.dumps({
            "metric": METRIC_7B, "value": tps, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": max(1, min(args.steps, 16)), "warmup": 0, "ms_per_step": r["ms_per_token"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "i8*i8->f32",
            "data": "synthetic", "config": tp7b_config(), "parallelism": f"cpu threads x{threads}",
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": r["sample"]},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return
    path = ensure_model(0, None)
    tps, _, sample = reference_decode(path, args.steps, args.warmup, threads)
    line = {
        "metric": METRIC, "value": tps, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / tps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": tps / PUBLISHED_BEST, "dtype": "i8*i8->f32",
        "data": "synthetic: random-init N(0,0.02) Q8_0 GGUF (seed 1234), 32 uniform prompt ids (seed 7)",
        "config": decode_config(), "parallelism": f"cpu threads x{threads}",
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_sweeps:
        line["sweeps"] = {
            "gemv": reference_gemv_rows(parse_shapes(args.shapes), 0.5),
            "attention": reference_attention_rows([int(v) for v in args.nkv.split(",")], 0.3),
            "prefill": reference_prefill(path, 1, threads)}
    if not args.no_tp7b:
        line["tp7b"] = reference_7b(8, threads)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
L2_BYTES = 126 * 2 ** 20


def parse_shapes(spec: str):
    return [tuple(int(v) for v in s.split("x")) for s in spec.split(",")]


def _time_rotating(torch, fn, n_copies, launches, warmup):
    """Device time per launch of fn(copy_index), cycling over copies."""
    for i in range(warmup):
        fn(i % n_copies)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(launches):
        fn(i % n_copies)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / launches


def gemv_rows(shapes, launches: int, warmup: int, cold: bool) -> list:
    """Config 1: isolated Q8_0 GEMV (activation quantize fused) at the 0.5B shapes;
    distinct weight copies rotate so every launch reads its weights from HBM."""
    import torch
    import mi_cuda
    peak, peak_kind = load_peaks()
    L = mi_cuda.lib()
    rows = []
    for n, k in shapes:
        nb = L.mi_cuda_q8_0_packed_bytes(k, n)
        npad = (n + 7) // 8 * 8
        n_copies = max(1, -(-4 * L2_BYTES // nb)) if cold else 1
        g = torch.Generator(device="cuda").manual_seed(n + k)
        copies = []
        for _ in range(n_copies):
            buf = torch.empty(nb, dtype=torch.uint8, device="cuda")
            buf[:npad * k].view(torch.int8).copy_(torch.randint(-127, 128, (npad * k,), generator=g, device="cuda",
                                                                dtype=torch.int8))
            sc = (torch.rand(npad * k // 32, generator=g, device="cuda") * 0.004 + 1e-4).to(torch.float16)
            buf[npad * k:].view(torch.float16).copy_(sc)
            copies.append(buf)
        x = torch.randn(k, generator=g, device="cuda")
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream

        def fn(i):
            mi_cuda.check(L.mi_cuda_mul_mat_q8_0_f32(copies[i].data_ptr(), k, n, x.data_ptr(), 1, out.data_ptr(), st))

        ms = _time_rotating(torch, fn, n_copies, launches, warmup)
        algo = n * k * 34 // 32 + 4 * k + 4 * n
        gbs = algo / (ms / 1e3) / 1e9
        rows.append({"shape": f"{n}x{k}", "us_per_launch": ms * 1e3, "bytes_per_launch": algo,
                     "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak, "peak_kind": peak_kind,
                     "weight_copies": n_copies, "launches": launches})
        del copies
    return rows


def attention_rows(nkvs, launches: int, warmup: int, cold: bool) -> list:
    """Config 2: fused decode attention, 14 query / 2 KV heads, head_dim 64, F32 KV,
    one query token; K/V copies rotate so each launch reads its cache from HBM.
    exact: the reference's summation order (bit-identical); split: positions
    split over CTAs, sums regrouped (labelled fast mode, not bit-identical)."""
    import torch
    import mi_cuda
    peak, peak_kind = load_peaks()
    H, HKV, D = 14, 2, 64
    L = mi_cuda.lib()
    rows = []
    for n_kv in nkvs:
        kvb = 2 * n_kv * HKV * D * 4
        n_copies = max(1, -(-4 * L2_BYTES // kvb)) if cold else 1
        g = torch.Generator(device="cuda").manual_seed(n_kv)
        ks = [torch.randn((n_kv, HKV, D), generator=g, device="cuda") for _ in range(n_copies)]
        vs = [torch.randn((n_kv, HKV, D), generator=g, device="cuda") for _ in range(n_copies)]
        q = torch.randn((H, D), generator=g, device="cuda")
        out = torch.empty((H, D), dtype=torch.float32, device="cuda")
        scratch = torch.empty(L.mi_cuda_attention_decode_scratch_bytes(H, n_kv), dtype=torch.uint8, device="cuda")
        split_scratch = torch.empty(L.mi_cuda_attention_decode_split_scratch_bytes(H, HKV, n_kv, D),
                                    dtype=torch.uint8, device="cuda")
        st = torch.cuda.current_stream().cuda_stream

        def fn(i):
            mi_cuda.check(L.mi_cuda_attention_decode(q.data_ptr(), ks[i].data_ptr(), vs[i].data_ptr(), D, H, HKV,
                                                     n_kv, 0.125, scratch.data_ptr(), out.data_ptr(), st))

        def fn_split(i):
            mi_cuda.check(L.mi_cuda_attention_decode_split(q.data_ptr(), ks[i].data_ptr(), vs[i].data_ptr(), D, H,
                                                           HKV, n_kv, 0.125, split_scratch.data_ptr(),
                                                           out.data_ptr(), st))

        algo = kvb + 2 * H * D * 4
        for mode, f in (("exact", fn), ("split", fn_split)):
            ms = _time_rotating(torch, f, n_copies, launches, warmup)
            gbs = algo / (ms / 1e3) / 1e9
            rows.append({"mode": mode, "n_kv": n_kv, "us_per_launch": ms * 1e3, "bytes_per_launch": algo,
                         "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak, "peak_kind": peak_kind,
                         "kv_copies": n_copies, "launches": launches})
        del ks, vs
    return rows


def run_gemv_sweep(args):
    import mi_cuda
    mi_cuda.init(0)
    for r in gemv_rows(parse_shapes(args.shapes), args.steps, args.warmup, bool(args.cold)):
        print(json.dumps({"config": "gemv", **r}), flush=True)


def run_attention(args):
    import mi_cuda
    mi_cuda.init(0)
    for r in attention_rows([int(v) for v in args.nkv.split(",")], args.steps, args.warmup, bool(args.cold)):
        print(json.dumps({"config": "attention", **r}), flush=True)


# Config 3: batched prefill of a 1024-token prompt (0.5B shape, ctx 2048).
N_PREFILL = 1024
METRIC_PREFILL = "prefill tok/s (0.5B-shape Q8_0, 1024-token prompt, ctx 2048)"
PUBLISHED_PREFILL = 46.855  # reference Q8_0 prefill tok/s, 1024 tokens, 4 threads (docs/stage6.md:734)


def prefill_config() -> dict:
    return {"workload": "qwen2.5-0.5b-shape Q8_0 prefill, 1024-token prompt, ctx 2048, last logits",
            "n_ctx": N_CTX, "prompt": N_PREFILL,
            "l2": "weights 527 MB > L2; activations of a layer re-read per weight tile"}


def prefill_macs(hp, n: int) -> int:
    """int8 multiply-adds of a prefill of n tokens: every layer's projections
    for every token, the LM head for the last token only."""
    E, FF, L, V = hp.n_embd, hp.n_ff, hp.n_layer, hp.n_vocab
    kvd = hp.n_head_kv * hp.head_dim
    per_token = L * (E * (E + 2 * kvd) + E * E + E * 2 * FF + FF * E)
    return n * per_token + V * E


def prefill_measure(path: str, model, kv, steps: int, warmup: int, with_cpu: bool) -> dict:
    """mi_cuda_qwen2_forward of a 1024-token prompt (last-position logits),
    timed on the device; each step re-runs the whole prompt."""
    import torch
    hp = model.hparams
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, hp.n_vocab, N_PREFILL).astype(np.int32)
    stream = torch.cuda.ExternalStream(kv.stream_handle, device=f"cuda:{model.device}")
    for _ in range(warmup):
        kv.forward(prompt, 0, last_logits_only=True, want_logits=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        kv.forward(prompt, 0, last_logits_only=True, want_logits=False)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    logits = kv.forward(prompt, 0, last_logits_only=True)
    # e2e: logits D2H included (the call a user makes)
    t0 = time.perf_counter()
    for _ in range(3):
        kv.forward(prompt, 0, last_logits_only=True)
    e2e_s = (time.perf_counter() - t0) / 3
    cpu = parity = None
    if with_cpu:
        import mi_oracle
        threads = os.cpu_count() or 1
        m = mi_oracle.ReferenceModel(path, n_ctx=N_CTX, n_threads=threads)
        t0 = time.perf_counter()
        want = m.forward(prompt, 0, last_logits_only=True)
        cpu_s = time.perf_counter() - t0
        m.close()
        a, b = logits[0].astype(np.float64), want[0].astype(np.float64)
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        cpu = {"value": N_PREFILL / cpu_s, "unit": "tok/s", "cores": threads, "kind": "reference",
               "sample": f"one mi_qwen2_forward of the {N_PREFILL}-token prompt (last logits), {threads} threads"}
        parity = {"last_logits_max_abs": float(np.max(np.abs(a - b))), "last_logits_cos": cos,
                  "bit_identical": bool(np.array_equal(logits[0].view(np.uint32), want[0].view(np.uint32))),
                  "vs": "reference AVX2 CPU path (oracle/_ref)"}
    value = N_PREFILL * steps / (ms / 1e3)
    peak_tops = 2 * load_peaks_bf16()
    ops = 2 * prefill_macs(hp, N_PREFILL) * steps / (ms / 1e3) / 1e12
    return {
        "value": value, "unit": "tok/s", "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
        "roofline": {"bound": "tensor", "achieved": ops, "peak": peak_tops, "unit": "TOPS",
                     "frac": ops / peak_tops, "traffic": None,
                     "peak_kind": "2 x measured bf16 TF/s (the int8 tensor rate)",
                     "achieved_counts": "useful int8 multiply-adds of the projections (x2); the GEMMs run them "
                                        "as lane-expanded fp16 tcgen05 MMAs (4x the useful MACs on the tensor "
                                        "pipe) feeding the exact FMA chains on the CUDA cores",
                     "kernel": "prefill (24 layers x (norm, QKV GEMM, RoPE/KV, attention, O GEMM, norm, "
                               "gate/up GEMM, down GEMM) + LM head)",
                     "ops_per_step": 2 * prefill_macs(hp, N_PREFILL)},
        "e2e": {"value": N_PREFILL / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": N_PREFILL * 4 + 36,
                "d2h_bytes_per_step": hp.n_vocab * 4 + 4, "api": "mi_cuda_qwen2_forward (1024 tokens, last logits)"},
        "gpu_launches": steps * (hp.n_layer * 8 + 1),
        "cpu_baseline": cpu, "parity": parity}


def run_prefill(args):
    """Config 3 as its own bench line."""
    import mi_cuda
    mi_cuda.init(0)
    path = ensure_model(0, None)
    model = mi_cuda.Qwen2Model(path)
    kv = mi_cuda.KVCache(model, N_CTX)
    t0 = time.perf_counter()
    with ClockSampler(0) as clk:
        clk.wait_first()
        r = prefill_measure(path, model, kv, args.steps, args.warmup, not args.no_cpu_baseline)
    line = {"metric": METRIC_PREFILL, "n_gpus": 1, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": r["value"] / PUBLISHED_PREFILL, "dtype": "i8*i8->f32",
            "data": "synthetic: random-init N(0,0.02) Q8_0 GGUF (seed 1234), 1024 uniform prompt ids (seed 7)",
            "config": prefill_config(), "parallelism": "1 GPU", **r, "clocks": clk.summary(),
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    kv.free()
    model.free()


def load_peaks_bf16() -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0


# Config 4: Qwen2.5-7B shape, tensor-parallel over the ranks (strong scaling:
# one request, its weights split by rows across the GPUs).
N_CTX_7B, N_PROMPT_7B = 4096, 64
METRIC_7B = "decode tok/s (7B-shape Q8_0, ctx 4096, one request, row-sharded over the GPUs)"
N_PARITY_7B = 8  # decode forwards compared with the reference (its CPU path runs ~14 tok/s)


def tp7b_config() -> dict:
    return {"workload": "qwen2.5-7b-shape Q8_0 greedy decode, ctx 4096, prompt 64, positions 64..190",
            "n_ctx": N_CTX_7B, "prompt": N_PROMPT_7B,
            "l2": "inputs larger than L2: 7.5 GB of weights streamed every step"}


def ensure_7b_model(rank: int, dist) -> str:
    path = os.path.join(MODEL_DIR, f"qwen2_7b_seed{SEED_MODEL}_fast.gguf")
    if rank == 0:
        mi_gguf.ensure_qwen2_gguf(path, mi_gguf.QWEN2_7B, SEED_MODEL, fast=True)
    if dist is not None:
        dist.barrier()
    return path


def tp7b_measure(dist, rank: int, world: int, local: int, steps: int, warmup: int, e2e_steps: int,
                 with_cpu: bool, trace: bool = False, clk=None):
    """Config 4 on `world` GPUs, one rank each (every rank calls this): the 7B
    shape row-sharded over the ranks, decode timed on the device (max over
    ranks). Greedy-token parity from a dedicated untimed pass of N_PARITY_7B
    decode steps, against the reference's CPU path. Returns the result dict on
    rank 0, None elsewhere."""
    import torch
    import mi_cuda
    t0 = time.time()
    path = ensure_7b_model(rank, dist)
    gen_s = time.time() - t0
    t0 = time.time()
    model = mi_cuda.Qwen2Model(path, device=local, rank=rank, world=world)
    hp = model.hparams
    kv = mi_cuda.KVCache(model, N_CTX_7B)
    if dist:
        mi_cuda.tp_connect(kv)
    load_s = time.time() - t0
    prompt = np.random.default_rng(SEED_PROMPT).integers(0, hp.n_vocab, N_PROMPT_7B).astype(np.int32)
    kv.forward(prompt, 0, last_logits_only=True, want_logits=False)
    first = kv.last_token()
    seed_tokens = np.concatenate([prompt, [first]]).astype(np.int32)
    stream = torch.cuda.ExternalStream(kv.stream_handle, device=f"cuda:{local}")
    kv.set_position(seed_tokens, N_PROMPT_7B)
    kv.decode_steps(warmup, N_PROMPT_7B, PERIOD)
    torch.cuda.synchronize()
    kv.set_position(seed_tokens, N_PROMPT_7B)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    kv.decode_steps(steps, N_PROMPT_7B, PERIOD)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tr = step_trace_summary(kv) if trace else None
    # parity pass, independent of `steps`: the first N_PARITY_7B decode steps again
    kv.set_position(seed_tokens, N_PROMPT_7B)
    kv.decode_steps(N_PARITY_7B)
    gen = kv.read_tokens(N_PROMPT_7B, N_PARITY_7B + 1)

    # e2e through the public per-token API: token H2D, the device's greedy
    # token D2H (4 bytes; the logits stay sharded on the GPUs)
    n_e2e = max(1, min(e2e_steps, PERIOD))
    tok = first
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        kv.forward([tok], N_PROMPT_7B + i, last_logits_only=True, want_logits=False)
        tok = kv.last_token()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    kernels = kv.kernels_per_step
    kv.free()
    model.free()

    out = None
    if rank == 0:
        cpu = parity = None
        if with_cpu:
            r = reference_7b(N_PARITY_7B, os.cpu_count() or 1)
            ref_tok = np.array(r.pop("tokens"), dtype=np.int32)
            cpu = {**r, "kind": "reference"}
            parity = {"greedy_tokens_identical": bool(np.array_equal(ref_tok, gen)),
                      "n_tokens": int(gen.size), "vs": "reference AVX2 CPU path (oracle/_ref)"}
        value = steps / (ms / 1e3)
        n_kvs = [N_PROMPT_7B + (i % PERIOD) + 1 for i in range(steps)]
        total_bytes = sum(step_bytes(hp, n) for n in n_kvs)
        peak, peak_kind = load_peaks()
        achieved = total_bytes / (ms / 1e3) / 1e9
        out = {
            "metric": METRIC_7B, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "scaling": "strong",
            "parallelism": f"tp{world} (row-sharded GEMVs, peer-store exchange)", "config": tp7b_config(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
                         "frac": achieved / (peak * world), "per_rank_gbs": achieved / world,
                         "peak_kind": f"{peak_kind} x {world}",
                         "kernel": f"decode step graph ({kernels} kernels per rank)",
                         "bytes_per_step": total_bytes / steps},
            "e2e": {"value": n_e2e / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 + 36,
                    "d2h_bytes_per_step": 4, "api": "mi_cuda_qwen2_forward (no logits) + mi_cuda_qwen2_last_token"},
            "gpu_launches": steps * kernels * world,
            "cpu_baseline": cpu, "parity": parity,
            "setup_s": {"gguf_write": gen_s, "load_and_connect": load_s}}
        if tr is not None:
            out["trace"] = tr
    return out


def init_dist(world: int, local: int):
    import datetime
    import torch
    torch.cuda.set_device(local)
    if world <= 1:
        return None
    import torch.distributed as td
    td.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    return td


def run_tp7b(args):
    """Config 4 as its own bench line (`--config tp7b`, torchrun for N > 1)."""
    import mi_cuda
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = init_dist(world, local)
    mi_cuda.init(local)
    with ClockSampler(local) as clk:
        clk.wait_first()
        r = tp7b_measure(dist, rank, world, local, args.steps, args.warmup, args.e2e_steps,
                         not args.no_cpu_baseline, args.trace)
    if rank == 0:
        print(json.dumps({**r, "higher_is_better": True, "vs_baseline": None, "dtype": "i8*i8->f32",
                          "data": f"synthetic: random-init N(0,0.02) Q8_0 GGUF (mi_gguf_gen, seed {SEED_MODEL}), "
                                  f"64 uniform prompt ids (seed {SEED_PROMPT})",
                          "clocks": clk.summary()}), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def decode_measure(args, dist, rank: int, world: int, local: int) -> dict:
    """Config 0 on this rank's GPU (an independent replica when world > 1)."""
    import torch
    import mi_cuda
    path = ensure_model(rank, dist)
    model = mi_cuda.Qwen2Model(path, device=local)
    hp = model.hparams
    kv = mi_cuda.KVCache(model, N_CTX)
    prompt = prompt_ids(hp.n_vocab)
    kv.forward(prompt, 0, last_logits_only=True, want_logits=False)
    first = kv.last_token()
    seed_tokens = np.concatenate([prompt, [first]]).astype(np.int32)
    stream = torch.cuda.ExternalStream(kv.stream_handle, device=f"cuda:{local}")

    clk = ClockSampler(local).__enter__()
    clk.wait_first()
    # warm-up, then the timed decode steps
    kv.set_position(seed_tokens, N_PROMPT)
    kv.decode_steps(args.warmup, N_PROMPT, PERIOD)
    torch.cuda.synchronize()
    kv.set_position(seed_tokens, N_PROMPT)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    kv.decode_steps(args.steps, N_PROMPT, PERIOD)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    trace = step_trace_summary(kv) if args.trace else None
    # parity pass, untimed and independent of --steps: one full generation
    # (127 decode steps from the prompt and its greedy token), all 128 tokens
    kv.set_position(seed_tokens, N_PROMPT)
    kv.decode_steps(PERIOD)
    gen = kv.read_tokens(N_PROMPT, N_PREDICT)

    # roofline: algorithmic bytes of the timed steps over their device time
    n_kvs = [N_PROMPT + (i % PERIOD) + 1 for i in range(args.steps)]
    total_bytes = sum(step_bytes(hp, n) for n in n_kvs)
    peak, peak_kind = load_peaks()
    achieved = total_bytes / (ms / 1e3) / 1e9

    # e2e through the public per-token API, every step: the token H2D (with the
    # step state) from pinned memory, mi_cuda_qwen2_forward, and the step's
    # result D2H -- the greedy token from the device argmax (e2e), or the
    # logits row sampled on the host as the reference's loop does (e2e_logits).
    lib = mi_cuda.lib()
    n_e2e = max(1, min(args.e2e_steps, PERIOD))

    def e2e_run(with_logits: bool) -> float:
        pinned = torch.empty((1, hp.n_vocab), dtype=torch.float32, pin_memory=True)
        out = pinned.numpy()
        tok = first
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(n_e2e):
            tb = np.array([tok], dtype=np.int32)
            mi_cuda.check(lib.mi_cuda_qwen2_forward(model.h, kv.h, tb.ctypes.data, 1, N_PROMPT + i, 1,
                                                    out.ctypes.data if with_logits else None))
            tok = mi_cuda.sample_greedy(out[0]) if with_logits else kv.last_token()
        e2e_s = time.perf_counter() - t0
        if dist:
            t = torch.tensor([e2e_s], device=f"cuda:{local}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        return n_e2e * world / e2e_s

    e2e_tps = e2e_run(False)
    e2e_logits_tps = e2e_run(True)
    fast = None
    if not args.no_fast_mode and kv.kernels_per_step == 1:
        fast = fast_mode_measure(args, kv, seed_tokens, gen, stream, dist, local, world, hp, peak, peak_kind)
    clk.__exit__(None, None, None)
    kernels = kv.kernels_per_step

    sweeps = None
    if world == 1 and not args.no_sweeps:
        # configs 1-3 on the same GPU, outside the timed region
        sweeps = {"gemv": gemv_rows(parse_shapes(args.shapes), 50, 10, True),
                  "attention": attention_rows([int(v) for v in args.nkv.split(",")], 20, 5, True)}
        p = prefill_measure(path, model, kv, 3, 1, not args.no_cpu_baseline)
        sweeps["prefill"] = {k: p[k] for k in ("value", "unit", "ms_per_step", "roofline", "cpu_baseline", "parity")}
    kv.free()
    model.free()

    cpu = parity = None
    if rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tps, ref_tokens, sample = reference_decode(path, PERIOD, 0, threads)
        cpu = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample}
        parity = {"greedy_tokens_identical": bool(np.array_equal(ref_tokens, gen)),
                  "n_tokens": int(gen.size), "vs": "reference AVX2 CPU path (oracle/_ref)",
                  "run": "one untimed generation: prompt, then 127 device decode steps"}

    value = args.steps * world / (ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_BEST, "dtype": "i8*i8->f32",
        "data": "synthetic: random-init N(0,0.02) Q8_0 GGUF (seed 1234), 32 uniform prompt ids (seed 7)",
        "config": decode_config(), "parallelism": f"replicas x{world}",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": TRAFFIC_PER_STEP, "traffic_source": TRAFFIC_SOURCE,
                     "peak_kind": peak_kind,
                     "kernel": ("persistent decode step (one launch per token)" if kernels == 1
                                else f"decode step graph ({kernels} kernels)"),
                     "bytes_per_step": total_bytes / args.steps},
        "e2e": {"value": e2e_tps, "unit": "tok/s", "h2d_bytes_per_step": 4 + 32, "d2h_bytes_per_step": 4 + 4,
                "api": "mi_cuda_qwen2_forward (token in) + mi_cuda_qwen2_last_token (greedy token out)"},
        "e2e_logits": {"value": e2e_logits_tps, "unit": "tok/s", "h2d_bytes_per_step": 4 + 32,
                       "d2h_bytes_per_step": hp.n_vocab * 4 + 4,
                       "api": "mi_cuda_qwen2_forward (logits row out) + host greedy, as the reference loop"},
        "gpu_launches": args.steps * kernels + (args.steps - 1) // PERIOD,
        "clocks": {**clk.summary(), "span": "warm-up, timed steps, parity pass, e2e runs and the fast-mode run"},
        "cpu_baseline": cpu,
        "parity": parity,
    }
    if trace is not None:
        line["trace"] = trace
    if fast is not None:
        line["fast_mode"] = fast
    if sweeps is not None:
        line["sweeps"] = sweeps
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=PERIOD * 16)
    ap.add_argument("--warmup", type=int, default=PERIOD)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=PERIOD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp7b", action="store_true", help="decode: skip the 7B tensor-parallel object")
    ap.add_argument("--no-sweeps", action="store_true", help="decode: skip the configs 1-3 sweeps")
    ap.add_argument("--no-fast-mode", action="store_true", help="decode: skip the labelled fast-mode object")
    ap.add_argument("--config", choices=["decode", "gemv", "attention", "prefill", "tp7b"], default="decode",
                    help="decode: config 0 (default); gemv: config-1 GEMV sweep; attention: config 2; "
                         "prefill: config 3, 1024-token prompt; tp7b: config 4, 7B shape tensor-parallel over the "
                         "torchrun ranks")
    ap.add_argument("--shapes", default="896x896,128x896,4864x896,896x4864,151936x896",
                    help="gemv: NxK list")
    ap.add_argument("--nkv", default="128,1024,4096,32768", help="attention: n_kv list")
    ap.add_argument("--cold", type=int, default=1, help="gemv/attention: rotate copies past L2")
    ap.add_argument("--trace", action="store_true", help="decode: add the last step's kernel timeline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank)
    if args.config == "gemv":
        return run_gemv_sweep(args)
    if args.config == "attention":
        return run_attention(args)
    if args.config == "tp7b":
        return run_tp7b(args)
    if args.config == "prefill":
        return run_prefill(args)

    import mi_cuda
    dist = init_dist(world, local)
    mi_cuda.init(local)
    line = decode_measure(args, dist, rank, world, local)
    if not args.no_tp7b:
        # the path that shards: the 7B shape row-sharded over all ranks
        tp = tp7b_measure(dist, rank, world, local, PERIOD, 10, 10, not args.no_cpu_baseline)
        if rank == 0:
            line["tp7b"] = tp
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
