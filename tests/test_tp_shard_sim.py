"""Tensor-parallel row sharding simulated on the CPU with the oracle.

Two gloo ranks each compute only their own rows of every projection of a
decode step -- the same split the GPU executor uses (mi_cuda_tp_shard_range:
8-row units of the stacked QKV, O, down and LM-head matrices; whole 32-element
activation blocks of the FFN, so a rank quantizes exactly the blocks it
produced) -- through the oracle's ops, and gather the pieces in rank order. The
concatenated results must equal the unsharded oracle step bit for bit: row
sharding keeps each output row's reduction (ref src/ops_cpu.cpp:226-237), and
this checks the split itself (unit bounds, the stacked-QKV offsets, the FFN
block ownership, the argmax over sharded logits) without a GPU.
"""
import os
import socket

import numpy as np
import pytest

from conftest import bits

N_STEPS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class ShardedStep:
    """One rank's view of a decode step of a Qwen2 GGUF (T = 1)."""

    def __init__(self, path, rank, world, n_ctx, gather):
        import mi_cuda
        import mi_gguf
        import mi_oracle
        self.rs = mi_oracle.Restatement()
        self.g = mi_gguf.GGUFFile(path)
        self.s = self.g.shape()
        self.rank, self.world, self.gather = rank, world, gather
        self.shard = lambda units: mi_cuda.shard_range(units, rank, world)
        s = self.s
        kvd = s.n_head_kv * s.head_dim
        self.cache_k = [np.zeros((n_ctx, s.n_head_kv, s.head_dim), np.float32) for _ in range(s.n_layer)]
        self.cache_v = [np.zeros((n_ctx, s.n_head_kv, s.head_dim), np.float32) for _ in range(s.n_layer)]
        # stacked q | k | v rows (GGUF Q8_0 rows are contiguous, 34 B per 32 weights)
        t = self.g.tensors
        self.wqkv = [np.concatenate([t[f"blk.{l}.attn_{n}.weight"].data for n in "qkv"]) for l in range(s.n_layer)]
        self.nqkv = s.n_embd + 2 * kvd

    def w(self, name):
        return self.g.tensors[name].data

    def f32(self, name):
        return self.g.tensors[name].data.view(np.float32)

    def rows(self, w_raw, k, n, act, r0, r1):
        """Rows [r0, r1) of W . act through the oracle's mul_mat."""
        if r1 <= r0:
            return np.empty(0, np.float32)
        rb = k // 32 * 34
        return self.rs.mul_mat(w_raw[r0 * rb:r1 * rb], k, r1 - r0, act, 1)[0]

    def gemv8(self, w_raw, k, n, act):
        """This rank's 8-row units of an n-row GEMV, gathered in rank order."""
        f, c = self.shard((n + 7) // 8)
        part = self.rows(w_raw, k, n, act, min(8 * f, n), min(8 * (f + c), n))
        return np.concatenate(self.gather(part))

    def norm(self, x, w):
        return self.rs.rms_norm(x, self.s.rms_eps) * w

    def step(self, tok, n_past):
        s, rs = self.s, self.rs
        E, H, HKV, D, FF, V = s.n_embd, s.n_head, s.n_head_kv, s.head_dim, s.n_ff, s.n_vocab
        kvd = HKV * D
        x = np.empty((1, E), np.float32)
        rs.lib.mio_get_rows_q8_0(self.w("token_embd.weight").ctypes.data, E,
                                 np.array([tok], np.int32).ctypes.data, 1, x.ctypes.data)
        x = x[0]
        scale = np.float32(1.0) / np.sqrt(np.float32(D))
        for l in range(s.n_layer):
            b = f"blk.{l}."
            qa = rs.quantize_act(self.norm(x, self.f32(b + "attn_norm.weight")))[0]
            qkv = self.gemv8(self.wqkv[l], E, self.nqkv, qa)
            q = qkv[:E] + self.f32(b + "attn_q.bias")
            k = qkv[E:E + kvd] + self.f32(b + "attn_k.bias")
            v = qkv[E + kvd:] + self.f32(b + "attn_v.bias")
            qr = rs.rope(q.reshape(1, H, D), n_past, D, s.rope_freq_base)
            kr = rs.rope(k.reshape(1, HKV, D), n_past, D, s.rope_freq_base)
            self.cache_k[l][n_past] = kr[0]
            self.cache_v[l][n_past] = v.reshape(HKV, D)
            _, _, att = rs.attention(qr, self.cache_k[l], self.cache_v[l], HKV, n_past, 1, scale)
            o = self.gemv8(self.w(b + "attn_output.weight"), E, E, rs.quantize_act(att.reshape(E))[0])
            x = x + o
            qa = rs.quantize_act(self.norm(x, self.f32(b + "ffn_norm.weight")))[0]
            # the FFN in whole 32-element blocks: gate and up rows of this
            # rank's blocks, SiLU * up, and the quantized blocks themselves
            f, c = self.shard(FF // 32)
            r0, r1 = 32 * f, 32 * (f + c)
            gate = self.rows(self.w(b + "ffn_gate.weight"), E, FF, qa, r0, r1)
            up = self.rows(self.w(b + "ffn_up.weight"), E, FF, qa, r0, r1)
            act_part = rs.quantize_act(rs.silu(gate) * up)[0] if c else np.empty(0, np.uint8)
            act = np.concatenate(self.gather(act_part))
            x = x + self.gemv8(self.w(b + "ffn_down.weight"), FF, E, act)
        head = "output.weight" if "output.weight" in self.g.tensors else "token_embd.weight"
        qa = rs.quantize_act(self.norm(x, self.f32("output_norm.weight")))[0]
        return self.gemv8(self.w(head), E, V, qa)


def _rank_main(rank, world, port, path, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def gather(part):
        out = [None] * world
        dist.all_gather_object(out, part)
        return out

    st = ShardedStep(path, rank, world, 64, gather)
    tok, logits = 3, []
    for step in range(N_STEPS):
        lg = st.step(tok, step)
        logits.append(lg)
        tok = int(np.argmax(lg))  # numpy's argmax is the first maximum, as the reference's
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.stack(logits))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_decode_equals_unsharded(tmp_path, model_path, world):
    import mi_gguf
    import mi_oracle
    import torch.multiprocessing as mp
    path = model_path("SMALL", 4)
    mp.spawn(_rank_main, args=(world, _free_port(), path, str(tmp_path)), nprocs=world, join=True)
    oracle = mi_oracle.RestatedModel(mi_gguf.GGUFFile(path), n_ctx=64)
    tok = 3
    got = [np.load(tmp_path / f"r{r}.npy") for r in range(world)]
    for step in range(N_STEPS):
        want = oracle.forward([tok], step)[0]
        for r in range(world):
            assert np.array_equal(bits(got[r][step]), bits(want)), f"rank {r} step {step}"
        tok = int(np.argmax(want))


def test_sharded_step_single_rank_matches_oracle(model_path):
    """The simulation itself at world 1 is the oracle's decode step."""
    import mi_gguf
    import mi_oracle
    path = model_path("TINY", 1)
    st = ShardedStep(path, 0, 1, 64, lambda part: [part])
    oracle = mi_oracle.RestatedModel(mi_gguf.GGUFFile(path), n_ctx=64)
    tok = 7
    for step in range(N_STEPS):
        got = st.step(tok, step)
        want = oracle.forward([tok], step)[0]
        assert np.array_equal(bits(got), bits(want)), f"step {step}"
        tok = int(np.argmax(want))
