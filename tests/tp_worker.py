"""One rank of the tensor-parallel parity check (launched by test_gpu_tp.py
through torch.distributed.run, one process per GPU).

Each rank loads its shard of the model, connects the exchange buffers, and
  1. runs a prefill + decode through mi_cuda_qwen2_forward; rank 0 gathers the
     vocabulary shards of every logits row and compares them bit for bit with
     the reference's mi_qwen2_forward on the CPU;
  2. generates greedily on the device (token feedback through the ranks'
     argmax exchange) and compares the tokens with the reference's.
Rank 0 writes {"ok": bool, ...} to the path given as argv[3]."""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "mini-infer-llama.cpp_b200"), os.path.join(ROOT, "oracle")):
    sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import mi_cuda  # noqa: E402
import mi_gguf  # noqa: E402


def gather_logits(kv, model, rows):
    """Full logits rows from every rank's vocabulary shard."""
    n_vocab = model.n_vocab
    first, count = mi_cuda.shard_range((n_vocab + 7) // 8, model.rank, model.world)
    v0 = first * 8
    nv = min(count * 8, n_vocab - v0)
    parts = [None] * model.world
    dist.all_gather_object(parts, (v0, rows[:, v0:v0 + nv].copy()))
    full = np.empty_like(rows)
    for v, block in parts:
        full[:, v:v + block.shape[1]] = block
    return full


def stall_check(kv, rank, out_path):
    """Rank 1 stops stepping (it launches nothing); rank 0 runs one decode step,
    whose exchange waits must expire with MI_CUDA_ERR_TIMEOUT in bounded time
    and leave the process able to report and clean up."""
    import time
    dist.barrier()
    res = None
    if rank == 0:
        kv.set_position(np.array([1, 2, 3], dtype=np.int32), 2)
        t0 = time.time()
        code = 0
        try:
            kv.decode_steps(1)
            kv.read_tokens(0, 3)
        except mi_cuda.MiCudaError as e:
            code = e.code
        res = {"ok": code == mi_cuda.ERR_TIMEOUT, "code": code, "seconds": time.time() - t0}
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.barrier()


def main():
    shape_name, seed, out_path = sys.argv[1], int(sys.argv[2]), sys.argv[3]
    mode = sys.argv[4] if len(sys.argv) > 4 else "parity"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=120))
    model_dir = os.environ.get("MI_B200_MODEL_DIR", "/tmp/mi_b200_models")
    shape = getattr(mi_gguf, shape_name)
    path = os.path.join(model_dir, f"{shape_name.lower()}_seed{seed}_fast.gguf")
    if rank == 0:
        mi_gguf.ensure_qwen2_gguf(path, shape, seed, fast=True)
    dist.barrier()
    n_ctx = 128
    mi_cuda.init(local)
    model = mi_cuda.Qwen2Model(path, device=local, rank=rank, world=world)
    kv = mi_cuda.KVCache(model, n_ctx)
    mi_cuda.tp_connect(kv)
    if mode == "stall":
        stall_check(kv, rank, out_path)
        kv.free()
        model.free()
        dist.destroy_process_group()
        return
    prompt = np.random.default_rng(seed).integers(0, model.n_vocab, 10).astype(np.int32)

    # 1. forward with logits (prefill rows, then decode steps)
    got = [gather_logits(kv, model, kv.forward(prompt, 0))]
    toks = []
    tok = mi_cuda.sample_greedy(got[0][-1])
    for step in range(6):
        toks.append(tok)
        got.append(gather_logits(kv, model, kv.forward([tok], prompt.size + step)))
        tok = mi_cuda.sample_greedy(got[-1][0])
    device_tok = kv.last_token()

    # 2. on-device greedy generation
    gen, _, _ = kv.generate(prompt, 24)
    dist.barrier()
    kv.free()
    model.free()

    if rank == 0:
        import mi_oracle
        ref = mi_oracle.ReferenceModel(path, n_ctx=n_ctx, n_threads=os.cpu_count() or 1)
        want = [ref.forward(prompt, 0)]
        for step, t in enumerate(toks):
            want.append(ref.forward([t], prompt.size + step))
        ref.close()
        ref = mi_oracle.ReferenceModel(path, n_ctx=n_ctx, n_threads=os.cpu_count() or 1)
        want_gen, _, _ = ref.generate(prompt, 24)
        ref.close()
        logits_ok = all(np.array_equal(np.ascontiguousarray(g).view(np.uint32),
                                       np.ascontiguousarray(w).view(np.uint32)) for g, w in zip(got, want))
        res = {"ok": bool(logits_ok and np.array_equal(gen, want_gen) and device_tok == mi_cuda.sample_greedy(want[-1][0])),
               "logits_bitexact": bool(logits_ok), "tokens_identical": bool(np.array_equal(gen, want_gen)),
               "device_argmax": bool(device_tok == mi_cuda.sample_greedy(want[-1][0])),
               "world": world, "shape": shape_name, "gen": gen.tolist(), "want": want_gen.tolist()}
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
