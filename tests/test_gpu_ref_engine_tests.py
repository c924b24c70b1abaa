"""The reference's own engine tests, unmodified, on the GPU engine.

tests/engine_test.c (three stages EMBED | LAYERS | HEAD, the prompt token,
its logits and argmax, then greedy generation) and tests/engine_stages.c
(the state after the embedding, before every layer through llm_layer_once
with the caller rewinding `lay.pos`, before the head, the logits and the
argmax) are compiled from the reference's sources twice by
distcomp_b200/host/Makefile: with distcomp_b200/host/engine_cuda.c (the
engine API over libdcb200.so) and with the reference's src/engine.c.  Both
builds run on the same GGUF files; the GPU build must print the same
geometry, argmax and generated tokens, and values within 1e-3 of the
printed vector's scale (the bar the oracle comparisons use)."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BUILD = ROOT / "_build" / "dcd_gpu"
TOL = 1e-3


def run(binary, *args):
    r = subprocess.run([str(binary), *map(str, args)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-1500:] + r.stderr[-1500:]
    return r.stdout


def parse(out):
    """{label: [fields...]} for the printed lines, in print order (a label
    seen again gets a numeric suffix)."""
    lines = {}
    for ln in out.splitlines():
        parts = ln.split()
        if not parts:
            continue
        key, k, i = parts[0], parts[0], 1
        while k in lines:
            k = f"{key}#{i}"
            i += 1
        lines[k] = parts[1:]
    return lines


def compare(cpu_out, gpu_out):
    a, b = parse(cpu_out), parse(gpu_out)
    assert a.keys() == b.keys(), (sorted(a), sorted(b))
    for k in a:
        if k.startswith(("geom", "argmax", "gen", "prompt")):
            assert a[k] == b[k], (k, a[k], b[k])
            continue
        va = np.array([float(x) for x in a[k]])
        vb = np.array([float(x) for x in b[k]])
        scale = max(float(np.max(np.abs(va))), 1e-6)
        err = float(np.max(np.abs(va - vb))) / scale
        assert err <= TOL, (k, err, a[k], b[k])


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    need = [BUILD / f"{t}-{k}" for t in ("engine_test", "engine_stages") for k in ("gpu", "cpu")]
    if not all(p.exists() for p in need):
        pytest.skip("reference engine tests not built (make -C distcomp_b200/host with the reference sources)")
    d = tmp_path_factory.mktemp("ref_engine_tests")
    files = [ROOT / "tests" / "golden" / "llama_ref_tiny.gguf"]
    for key in ("mini-q4", "mini-q8"):
        p = d / f"{key}.gguf"
        synth.build_model(synth.spec(key, n_layer=2), seed=0).tofile(p)
        files.append(p)
    return files


def test_engine_test_matches_reference_build(models):
    for f in models:
        cpu = run(BUILD / "engine_test-cpu", f, 6)
        gpu = run(BUILD / "engine_test-gpu", f, 6)
        compare(cpu, gpu)
        assert re.search(r"^gen( \d+){6}$", gpu, re.M), gpu


def test_engine_stages_matches_reference_build(models):
    for f in models:
        prompt = [1, 7, 3]
        cpu = run(BUILD / "engine_stages-cpu", f, *prompt)
        gpu = run(BUILD / "engine_stages-gpu", f, *prompt)
        compare(cpu, gpu)
