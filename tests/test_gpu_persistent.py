"""The persistent whole-step kernel (k_decode_mega) against the oracle and
the reference fixtures, and against the one-kernel-per-operation step.

The mini Q4_0 / Q8_0 shapes qualify for it (fused projections in the fast
layouts, head_dim 128 / 64 with 4 query heads per KV head); the tiny shape
(head_dim 32) does not and keeps the per-kernel step, which the other engine
tests cover.  ECU_MEGA=0 at open time selects the per-kernel step.
"""
import os

import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu


def vec_close(a, b, rel):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.max(np.abs(b)), 1e-30)
    err = float(np.max(np.abs(a - b)) / scale)
    return err <= rel, err


def open_ctx(eng, m, stage, *args, mega=True, **kw):
    old = os.environ.get("ECU_MEGA")
    os.environ["ECU_MEGA"] = "1" if mega else "0"
    try:
        return eng.LlmCtx(m, stage, *args, **kw)
    finally:
        if old is None:
            del os.environ["ECU_MEGA"]
        else:
            os.environ["ECU_MEGA"] = old


def test_path_selection(eng, model_buf):
    for key in ("mini-q4", "mini-q8"):
        m = eng.GgufModel(model_buf(key))
        s = synth.spec(key)
        assert open_ctx(eng, m, eng.STAGE_FULL).path() == "persistent", key
        assert open_ctx(eng, m, eng.STAGE_LAYERS, 0, s.n_layer - 1).path() == "persistent", key
        assert open_ctx(eng, m, eng.STAGE_FULL, mega=False).path() == "kernels: ECU_MEGA=0"
        assert open_ctx(eng, m, eng.STAGE_HEAD).path().startswith("kernels")
    m = eng.GgufModel(model_buf("tiny"))
    assert open_ctx(eng, m, eng.STAGE_FULL).path().startswith("kernels: head_dim")


@pytest.mark.parametrize("name,key,n_gen", [("mini_q4", "mini-q4", 32), ("mini_q8", "mini-q8", 24)])
def test_matches_reference_fixture(eng, golden, model_buf, name, key, n_gen):
    d = golden(f"{name}.npz")
    s = synth.spec(key)
    m = eng.GgufModel(model_buf(key))
    c = open_ctx(eng, m, eng.STAGE_FULL)
    assert c.path() == "persistent"
    prompt = [int(t) for t in d["prompt"]]
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    assert c.forward(prompt[0], out) == 0
    ok, err = vec_close(c.logits(), d["logits_tok0"], 1e-3)
    assert ok, f"logits rel err {err:.2e}"
    # normed state out (norm weights are 1.0: unit RMS) and the argmax
    assert abs(np.sqrt(np.mean(out[: s.n_embd].astype(np.float64) ** 2)) - 1.0) < 1e-3
    assert int(out[s.n_embd]) == c.pick() == int(np.argmax(c.logits()))
    c.reset()
    assert c.generate(prompt, n_gen) == [int(t) for t in d["greedy"]]
    assert c.pos == len(prompt) + n_gen - 1


def test_long_generation_vs_oracle(eng, oracle_port, model_buf):
    """Positions past several 32-row K/V sub-chunks per split, and the
    per-layer state of a LAYERS stage against the oracle."""
    import oracle
    key = "mini-q4"
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    prompt = synth.prompt_tokens(9, s.n_vocab, seed=5)
    n_gen = s.n_ctx - len(prompt) + 1
    want = oracle.greedy(oracle_port, buf, prompt, n_gen)
    c = open_ctx(eng, m, eng.STAGE_FULL)
    assert c.generate(prompt, n_gen) == want
    # LAYERS stage: state after both layers at every prompt position
    lay = open_ctx(eng, m, eng.STAGE_LAYERS, 0, s.n_layer - 1)
    assert lay.path() == "persistent"
    o = oracle_port.model(buf).ctx(1, 0, s.n_layer - 1)
    rng = np.random.default_rng(1)
    for _ in range(40):
        x = rng.standard_normal(s.n_embd).astype(np.float32)
        a, b = x.copy(), x.copy()
        assert lay.forward(0, a) == 0 and o.forward(0, b) == 0
        ok, err = vec_close(a, b, 1e-3)
        assert ok, err


def test_same_tokens_as_per_kernel_step(eng, model_buf):
    key = "mini-q8"
    s = synth.spec(key)
    m = eng.GgufModel(model_buf(key))
    prompt = synth.prompt_tokens(7, s.n_vocab, seed=9)
    a = open_ctx(eng, m, eng.STAGE_FULL)
    b = open_ctx(eng, m, eng.STAGE_FULL, mega=False)
    assert a.generate(prompt, 40) == b.generate(prompt, 40)
    ok, err = vec_close(a.logits(), b.logits(), 1e-4)
    assert ok, err


def test_profile_phases(eng, model_buf):
    key = "mini-q4"
    s = synth.spec(key)
    m = eng.GgufModel(model_buf(key))
    c = open_ctx(eng, m, eng.STAGE_FULL)
    c.generate(synth.prompt_tokens(4, s.n_vocab, seed=1), 2)
    prof = c.profile_steps(3)
    assert prof["decode_step"][0] == 3
    for kind in ("gemv_qkv", "attention", "gemv_o", "gemv_gate_up", "gemv_down"):
        assert prof[kind][0] == 3 * s.n_layer, kind
    assert prof["gemv_head_argmax"][0] == 3 and prof["embed"][0] == 3
    total = sum(v[1] for k, v in prof.items() if k != "decode_step" and ":" not in k)
    # GEMV phases also report where CTA 0 spent them
    assert prof["gemv_gate_up:main"][0] == 3 * s.n_layer
    assert 0 < total <= prof["decode_step"][1] * 1.05


@pytest.mark.parametrize("key", ["mini-q4", "mini-q8"])
@pytest.mark.parametrize("att,split", [("1", "1"), ("2", "1"), ("2", "3")])
def test_attention_slots_and_splits_vs_oracle(eng, oracle_port, model_buf, key, att, split, monkeypatch):
    """The persistent step's K/V buffers in one slot or in two (the copies
    of round r+1 in flight while round r is computed), with one or three
    position splits per KV head so that a split walks several rounds: the
    oracle's greedy tokens over the whole context."""
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    prompt = synth.prompt_tokens(5, s.n_vocab, seed=31)
    n_gen = s.n_ctx - len(prompt) + 1
    want = oracle.greedy(oracle_port, buf, prompt, n_gen)
    monkeypatch.setenv("ECU_MEGA_ATT", att)
    monkeypatch.setenv("ECU_MEGA_SPLIT", split)
    c = open_ctx(eng, eng.GgufModel(buf), eng.STAGE_FULL)
    assert c.path() == "persistent"
    assert c.generate(prompt, n_gen) == want


@pytest.mark.parametrize("key", ["mini-q4", "mini-q8"])
def test_early_kv_copies_vs_oracle(eng, oracle_port, model_buf, key, monkeypatch):
    """ECU_MEGA_KV_EARLY=1: the Q/K/V phase issues the attention's first K/V
    copies into buffers above its digit planes; the oracle's greedy tokens
    over the whole context (several rounds per split with ECU_MEGA_SPLIT=2)."""
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    prompt = synth.prompt_tokens(5, s.n_vocab, seed=33)
    n_gen = s.n_ctx - len(prompt) + 1
    want = oracle.greedy(oracle_port, buf, prompt, n_gen)
    monkeypatch.setenv("ECU_MEGA_KV_EARLY", "1")
    monkeypatch.setenv("ECU_MEGA_SPLIT", "2")
    c = open_ctx(eng, eng.GgufModel(buf), eng.STAGE_FULL)
    assert c.path() == "persistent"
    assert c.generate(prompt, n_gen) == want
