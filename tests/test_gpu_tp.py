"""Tensor parallelism on real GPUs: ranks as torchrun processes, one per GPU
(never two ranks on one GPU: their persistent steps wait on each other).
Each rank's tokens and logits slice must equal the one-GPU step's bit for
bit (tests/tp_ranks.py)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def run_ranks(tmp_path, world, key, port):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(ROOT / "tests" / "tp_ranks.py"),
           str(tmp_path), key]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-4000:]
    for k in range(world):
        assert (tmp_path / f"ok.{k}").exists(), r.stdout[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("key", ["mini-q4", "mini-q8", "mini-q4k"])
def test_tp2_matches_one_gpu(tmp_path, key):
    run_ranks(tmp_path, 2, key, {"mini-q4": 29541, "mini-q8": 29542, "mini-q4k": 29544}[key])


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_tp4_matches_one_gpu(tmp_path):
    # mini-q8: 4 KV heads, one per rank
    run_ranks(tmp_path, 4, "mini-q8", 29543)
