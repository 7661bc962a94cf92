"""Tensor parallelism on 2+ GPUs: one process per GPU (torch.distributed.run),
each rank holding its rows of every projection and exchanging the GEMV outputs
through peer stores. Logits and greedy tokens must equal the reference's bit
for bit, exactly as on one GPU. Skipped when fewer than two GPUs are visible."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def n_gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("shape,seed", [("SMALL", 31), ("MID7B", 21)])
def test_tensor_parallel_bitexact(tmp_path, shape, seed, torch_cuda):
    n = n_gpus()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 2 if shape == "SMALL" else min(n, 4)
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, "tp_worker.py"), shape, str(seed), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["logits_bitexact"], res
    assert res["tokens_identical"], res
    assert res["device_argmax"], res


def test_stopped_rank_times_out_without_fault(tmp_path, torch_cuda):
    """Failure made on the host: rank 1 stops launching steps. Rank 0's
    exchange waits run out (a bounded spin, then an error word; no trap, no
    fault) and the call returns MI_CUDA_ERR_TIMEOUT within seconds."""
    if n_gpus() < 2:
        pytest.skip("needs at least 2 GPUs")
    out = tmp_path / "stall.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534",
           os.path.join(HERE, "tp_worker.py"), "SMALL", "31", str(out), "stall"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["ok"], res
    assert res["seconds"] < 60, res
