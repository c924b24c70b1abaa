"""The reference's own shard pipeline with its stages on the GPU.

_build/dcd_gpu/dcd-gpu is the reference's dcd compiled from its sources with
distcomp_b200/host/engine_cuda.c in place of src/engine.c (the engine API
over libdcb200.so); _build/dcd_gpu/dcctl is the reference's dcctl, unmodified
(both built by distcomp_b200/host/Makefile).  This is the reference's
localhost multi-daemon scenario (its scripts/test.sh, sections 18-19): five
shard daemons with different free memory, `dcctl llm deploy` lays the
llama_ref model's layers out over them, `dcctl llm prompt ... distcomp 4`
runs the greedy pipeline stage by stage over UDP -- every stage's
llm_ctx_open / llm_forward / llm_pick now on the GPU -- and dcctl checks the
tokens against its own CPU engine run locally (src/shard.c:1207-1250),
printing that all generated tokens matched."""
import os
import shutil
import signal
import subprocess
import time
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BUILD = ROOT / "_build" / "dcd_gpu"
MODEL = ROOT / "tests" / "golden" / "llama_ref_tiny.gguf"


@pytest.fixture()
def shards(tmp_path):
    dcd, dcctl = BUILD / "dcd-gpu", BUILD / "dcctl"
    if not (dcd.exists() and dcctl.exists()):
        pytest.skip("dcd-gpu not built (make -C distcomp_b200/host with the reference sources)")
    base = 39000 + os.getpid() % 2000
    mems = [("in", 450000), ("big", 450000), ("sm1", 250000), ("sm2", 250000), ("out", 450000)]
    procs = []
    state = tmp_path / "state"
    state.mkdir()
    for i, (tag, mem) in enumerate(mems):
        log = open(tmp_path / f"sh{i}.log", "w")
        procs.append(subprocess.Popen([str(dcd), "--port", str(base + i), "--tag", tag, "--free-mem", str(mem),
                                       "--state", str(state)], stdout=log, stderr=subprocess.STDOUT,
                                      start_new_session=True))
    time.sleep(1.5)
    conf = tmp_path / "shard.conf"
    conf.write_text("[llm]\n\n[role shard]\n" + "".join(f"daemon = 127.0.0.1:{base + i}\n" for i in range(5)) +
                    "[scheduler]\ntimeout_ms = 20000\nretries = 0\n")
    model = tmp_path / "model.gguf"
    shutil.copy(MODEL, model)
    try:
        yield dcctl, conf, model, tmp_path
    finally:
        for p in procs:
            if p.poll() is None:
                os.killpg(p.pid, signal.SIGTERM)
        for p in procs:
            try:
                p.wait(timeout=10)
            except subprocess.TimeoutExpired:
                os.killpg(p.pid, signal.SIGKILL)


def test_dcd_pipeline_on_gpu_matches_local_engine(shards):
    dcctl, conf, model, tmp = shards
    env = dict(os.environ, DC_THREADS="4")
    dep = subprocess.run([str(dcctl), "-c", str(conf), "llm", "deploy", str(model)], capture_output=True,
                         text=True, timeout=120, env=env)
    out = dep.stdout + dep.stderr
    logs = "".join((tmp / f"sh{i}.log").read_text(errors="replace") for i in range(5))
    assert "Веса разложены" in out, out[-2000:] + logs[-2000:]
    assert "ОШИБКА" not in out, out[-2000:]
    run = subprocess.run([str(dcctl), "-c", str(conf), "llm", "prompt", str(model), "distcomp", "4"],
                         capture_output=True, text=True, timeout=300, env=env)
    out = run.stdout + run.stderr
    logs = "".join((tmp / f"sh{i}.log").read_text(errors="replace") for i in range(5))
    assert run.returncode == 0, out[-3000:] + logs[-2000:]
    assert "Генерация (жадная)" in out, out[-3000:]
    assert "все 4 сгенерированных токенов совпали" in out, out[-3000:]
