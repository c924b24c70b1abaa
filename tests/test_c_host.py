"""The drop-in from C: tests/c_host/shard_local.c, compiled with gcc against
include/engine_cuda.h and libdcb200.so, drives the engine the way distcomp's
local run drives its CPU engine (GGUF image in memory, EMBED / LAYERS / HEAD
stages, prompt token by token, greedy decode through the host), or with
--full one FULL context and ecu_prefill.  Its greedy tokens must be the
oracle's.  Without a GPU the program must fail loudly."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from distcomp_b200 import synth

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c_host" / "shard_local.c"
LIBDIR = ROOT / "distcomp_b200"


@pytest.fixture(scope="module")
def shard_local(tmp_path_factory):
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    if not (LIBDIR / "libdcb200.so").exists():
        pytest.skip("libdcb200.so not built")
    out = tmp_path_factory.mktemp("c_host") / "shard_local"
    subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(SRC),
                    "-L", str(LIBDIR), "-ldcb200", f"-Wl,-rpath,{LIBDIR}", "-o", str(out)],
                   check=True, capture_output=True, text=True)
    return out


def write_model(tmp_path, buf, name):
    p = tmp_path / f"{name}.gguf"
    np.asarray(buf, dtype=np.uint8).tofile(p)
    return p


def run(prog, args):
    return subprocess.run([str(prog), *map(str, args)], capture_output=True, text=True, timeout=600)


def test_c_host_fails_loudly_without_gpu(shard_local, model_buf, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = write_model(tmp_path, model_buf("tiny"), "tiny")
    r = run(shard_local, [p, 4, 5, 6, 7])
    assert r.returncode == 1
    assert "ecu_ctx_open" in r.stderr and "CUDA" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["mini-q4", "mini-q4k", "tiny"])
@pytest.mark.parametrize("full", [False, True])
def test_c_host_greedy_matches_oracle(shard_local, oracle_port, model_buf, tmp_path, key, full):
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    prompt = synth.prompt_tokens(7, s.n_vocab, seed=40)
    n_gen = 20
    want = oracle.greedy(oracle_port, buf, prompt, n_gen)
    p = write_model(tmp_path, buf, key)
    r = run(shard_local, (["--full"] if full else []) + [p, n_gen, *prompt])
    assert r.returncode == 0, r.stderr
    assert [int(t) for t in r.stdout.split()] == want
