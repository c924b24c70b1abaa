"""The 8B-shaped Q4_0 model (the decode benchmark's shape) against the
reference engine's own outputs.

tests/golden/llama3_8b_q4_0.npz holds what the reference engine (compiled
from src/engine.c, src/gguf.c and src/thread.c, run as src/shard.c's local
three-stage loop) produced on the seeded model synth.spec("llama3-8b"),
seed 0 -- dim 4096, 32 layers, 32/8 heads, FFN 14336, vocab 128256, Q4_0
layers, Q8_0 embedding and head -- written by tests/golden/make_golden_8b.py.
The model is rebuilt here from the same seed and its sha256 checked first.
What is compared (the bars of the north star: per-layer activations and
logits within 1e-3 of the vector's scale, identical greedy tokens):

  * every layer's output state for the first prompt token (llm_layer_once),
    and the state after all 32 layers from the persistent LAYERS step;
  * the first step's logits (the reference's 256 largest) and token;
  * 64 greedy tokens after 16 prompt tokens, one token at a time through
    the persistent FULL step (src/shard.c:1207-1250 checks exactly this
    against llm_forward / llm_pick);
  * the whole 512-token prompt through ecu_prefill (tensor-core GEMMs),
    then 16 greedy tokens: the first one and the continuation identical,
    the last prompt step's logits within 1e-3.
"""
import hashlib
import os

import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu

GOLDEN = "llama3_8b_q4_0.npz"


def vec_close(a, b, rel=1e-3):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(float(np.max(np.abs(b))), 1e-30)
    err = float(np.max(np.abs(a - b)) / scale)
    return err <= rel, err


@pytest.fixture(scope="module")
def m8b(golden, eng):
    d = golden(GOLDEN)
    s = synth.spec("llama3-8b")
    # built exactly as the golden file's model was: host normals and the
    # host quantiser (gguf-py's rule), in parallel over tensors
    buf = synth.build_model(s, seed=0, threads=min(32, os.cpu_count() or 1))
    assert hashlib.sha256(buf).hexdigest() == bytes(d["model_sha256"]).decode(), "not the golden model"
    m = eng.GgufModel(buf)
    yield s, m, d
    m.close()


def test_layer_states_and_first_logits(eng, m8b):
    s, m, d = m8b
    prompt = [int(t) for t in d["prompt"]]
    want = d["layer_states"]
    emb = eng.LlmCtx(m, eng.STAGE_EMBED, n_ctx=8)
    lay = eng.LlmCtx(m, eng.STAGE_LAYERS, 0, s.n_layer - 1, n_ctx=8)
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    assert emb.forward(prompt[0], st) == 0
    assert np.array_equal(st[:s.n_embd], want[0])            # the embedding row, exactly
    x0 = st.copy()
    for li in range(s.n_layer):
        assert lay.layer_once(li, st) == 0
        ok, err = vec_close(st[:s.n_embd], want[li + 1])
        assert ok, f"layer {li}: rel err {err:.2e}"
    # all 32 layers in one persistent step
    lay.reset()
    assert lay.path() == "persistent"
    y = x0.copy()
    assert lay.forward(prompt[0], y) == 0
    ok, err = vec_close(y[:s.n_embd], want[s.n_layer])
    assert ok, f"persistent LAYERS step: rel err {err:.2e}"
    emb.close()
    lay.close()
    # first step through a FULL context: logits and token
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=8)
    assert c.path() == "persistent"
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    assert c.forward(prompt[0], out) == 0
    lg = c.logits().astype(np.float64)
    idx = d["top_idx0"].astype(np.int64)
    err = float(np.max(np.abs(lg[idx] - d["top_val0"])) / float(d["logits0_absmax"][0]))
    assert err <= 1e-3, f"first-step logits rel err {err:.2e}"
    assert abs(float(np.max(np.abs(lg))) / float(d["logits0_absmax"][0]) - 1.0) <= 1e-3
    assert int(out[s.n_embd]) == int(idx[0]) == c.pick()
    c.close()


def test_greedy_64_tokens(eng, m8b):
    s, m, d = m8b
    prompt = [int(t) for t in d["prompt"][:16]]
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=128)
    assert c.path() == "persistent"
    got = c.generate(prompt, 64)
    want = [int(t) for t in d["greedy16"]]
    first_diff = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    assert got == want, f"first difference at token {first_diff}"
    c.close()


def test_prefill_512_then_greedy(eng, m8b):
    s, m, d = m8b
    prompt = [int(t) for t in d["prompt"]]
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=1024)
    first = c.prefill(prompt)
    lg = c.logits().astype(np.float64)
    idx = d["top_idx512"].astype(np.int64)
    scale = float(np.max(np.abs(d["top_val512"])))
    err = float(np.max(np.abs(lg[idx] - d["top_val512"])) / scale)
    assert err <= 1e-3, f"last prompt step's logits rel err {err:.2e}"
    want = [int(t) for t in d["greedy512"]]
    assert first == want[0]
    # the continuation, one decode step at a time from the prefilled cache
    got = [first]
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    while len(got) < len(want):
        assert c.forward(got[-1], out) == 0
        got.append(int(out[s.n_embd]))
    assert got == want
    c.close()
