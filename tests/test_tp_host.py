"""Host logic of tensor parallelism, on the CPU: the row split every rank
applies to every matrix, and the exchange-handle handshake over
torch.distributed (gloo, two processes)."""
import os
import socket

import pytest


def test_shard_range_partitions_every_matrix():
    import mi_cuda
    for units in (1, 7, 8, 9, 100, 144, 148, 448, 576, 592, 18992, 19008):
        for world in range(1, 9):
            if units < world:
                continue
            spans = [mi_cuda.shard_range(units, r, world) for r in range(world)]
            assert spans[0][0] == 0
            for (f0, c0), (f1, _) in zip(spans, spans[1:]):
                assert f0 + c0 == f1                      # contiguous, in rank order
            assert sum(c for _, c in spans) == units      # covers every unit once
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_shard_range_rejects_bad_arguments():
    import mi_cuda
    for args in ((10, 2, 2), (10, -1, 2), (10, 0, 0), (-1, 0, 1)):
        with pytest.raises(mi_cuda.MiCudaError) as e:
            mi_cuda.shard_range(*args)
        assert e.value.code == mi_cuda.ERR_ARG


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    import mi_cuda
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    handles = mi_cuda.gather_handles(bytes([rank + 1]) * 64)
    with open(os.path.join(out_dir, f"r{rank}"), "wb") as f:
        f.write(b"".join(handles))
    dist.destroy_process_group()


def test_handle_exchange_is_rank_ordered(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    want = b"".join(bytes([r + 1]) * 64 for r in range(world))
    for r in range(world):
        assert (tmp_path / f"r{r}").read_bytes() == want
