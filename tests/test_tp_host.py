"""Host side of tensor parallelism on the CPU: the handle exchange as gloo
ranks (the GPU mapping itself needs GPUs, tests/test_gpu_tp.py)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from distcomp_b200 import tensor_parallel as TP


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_path, bad):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * (63 if (bad and rank == 1) else 64)
        try:
            got = TP.exchange_handles(mine, world)
            res = [h[0] for h in got]
        except RuntimeError as e:
            res = str(e)
        if rank == 0:
            with open(out_path, "w") as f:
                f.write(repr(res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,bad", [(2, False), (3, False), (3, True)])
def test_exchange_handles(tmp_path, world, bad):
    out = str(tmp_path / "res.txt")
    mp.start_processes(_rank, args=(world, _free_port(), out, bad), nprocs=world, join=True, start_method="spawn")
    res = open(out).read()
    if bad:
        assert "rank 1 sent a malformed handle" in res
    else:
        assert res == repr(list(range(world)))
