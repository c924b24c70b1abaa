"""Q4_K layers on the fast paths, and matrices wider than one column segment,
against the oracle.

Q4_K rows are kept in the SPLITK4 layout (16 code bytes per 32-weight
sub-block, then the 16-byte super-block headers) and run through the
digit-plane GEMV of both the persistent step and the per-kernel step; the
sub-block scale and minimum are the reference's two fp32 products
(src/gguf.c:558-590).  "wide-q4k" has n_ff = 20480, above the 16384 inputs
one column segment holds, so ffn_down is stored as two segments and runs as
two residual-adding GEMVs.  Bars: bit-exact readback of every tensor through
its device layout, logits and stage outputs within 1e-3 of the oracle's
(relative to the vector's scale), the oracle's greedy tokens.
"""
import os

import numpy as np
import pytest
from conftest import bits_equal

from distcomp_b200 import gguf as G
from distcomp_b200 import synth

pytestmark = pytest.mark.gpu
KEYS = ["mini-q4k", "wide-q4k"]
REL = 1e-3


def vec_close(a, b, rel=REL):
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


def test_q4k_paths(eng, model_buf):
    for key in KEYS:
        s = synth.spec(key)
        m = eng.GgufModel(model_buf(key))
        assert open_ctx(eng, m, eng.STAGE_FULL).path() == "persistent", key
        assert open_ctx(eng, m, eng.STAGE_LAYERS, 0, s.n_layer - 1).path() == "persistent", key
        assert open_ctx(eng, m, eng.STAGE_FULL, mega=False).path() == "kernels: ECU_MEGA=0"


@pytest.mark.parametrize("key", KEYS)
def test_q4k_weights_read_back_bit_exact(eng, oracle_port, model_buf, key):
    s = synth.spec(key)
    buf = model_buf(key)
    c = eng.LlmCtx(eng.GgufModel(buf), eng.STAGE_FULL)
    tab = G.read_tensor_table(buf)
    for name, dims, gt in synth.tensor_list(s):
        if name.endswith("norm.weight"):
            continue
        total = int(np.prod(dims))
        got = c.dequant_tensor(name, 0, total)
        rc, want = oracle_port.dequant(gt, np.frombuffer(tab[name][2], np.uint8), total, 0, total)
        assert rc == 0
        assert bits_equal(got, want), name


@pytest.mark.parametrize("key", KEYS)
@pytest.mark.parametrize("mega", [True, False])
def test_q4k_greedy_and_logits_vs_oracle(eng, oracle_port, model_buf, key, mega):
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    prompt = synth.prompt_tokens(6, s.n_vocab, seed=13)
    n_gen = 24
    want = oracle.greedy(oracle_port, buf, prompt, n_gen)
    c = open_ctx(eng, m, eng.STAGE_FULL, mega=mega)
    # logits after every prompt token (the oracle's embed -> layers -> head)
    om = oracle_port.model(buf)
    oe, ol, oh = om.ctx(0), om.ctx(1, 0, s.n_layer - 1), om.ctx(2)
    out, ob = np.zeros(s.n_embd + 1, np.float32), np.zeros(s.n_embd + 8, np.float32)
    for t in prompt:
        assert c.forward(t, out) == 0
        for o in (oe, ol, oh):
            assert o.forward(t, ob) == 0
        ok, err = vec_close(c.logits(), oh.logits(s.n_vocab))
        assert ok, f"logits rel err {err:.2e}"
        assert int(out[s.n_embd]) == int(ob[s.n_embd])
    c.reset()
    assert c.generate(prompt, n_gen) == want


@pytest.mark.parametrize("key", KEYS)
def test_q4k_layers_stage_vs_oracle(eng, oracle_port, model_buf, key):
    s = synth.spec(key)
    buf = model_buf(key)
    lay = open_ctx(eng, eng.GgufModel(buf), eng.STAGE_LAYERS, 0, s.n_layer - 1)
    assert lay.path() == "persistent"
    o = oracle_port.model(buf).ctx(1, 0, s.n_layer - 1)
    rng = np.random.default_rng(4)
    for _ in range(12):
        x = rng.standard_normal(s.n_embd).astype(np.float32)
        a, b = x.copy(), x.copy()
        assert lay.forward(0, a) == 0 and o.forward(0, b) == 0
        ok, err = vec_close(a, b)
        assert ok, err


@pytest.mark.parametrize("key", KEYS)
def test_q4k_prefill_vs_per_token(eng, oracle_port, model_buf, key):
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    prompt = synth.prompt_tokens(37, s.n_vocab, seed=22)
    a = eng.LlmCtx(m, eng.STAGE_FULL)
    b = eng.LlmCtx(m, eng.STAGE_FULL)
    out_a = np.zeros(s.n_embd + 1, dtype=np.float32)
    out_b = np.zeros(s.n_embd + 1, dtype=np.float32)
    first = a.prefill(prompt, out_a)
    for t in prompt:
        assert b.forward(t, out_b) == 0
    assert first == int(out_b[s.n_embd])
    ok, err = vec_close(a.logits(), b.logits())
    assert ok, f"logits rel err {err:.2e}"
    n_gen = min(16, s.n_ctx - len(prompt))
    toks, tok = [first], first
    while len(toks) < n_gen:
        assert a.forward(tok, out_a) == 0
        tok = int(out_a[s.n_embd])
        toks.append(tok)
    assert toks == oracle.greedy(oracle_port, buf, prompt, n_gen)


def test_q4k_70b_layer_shape_vs_oracle(eng, oracle_port, model_buf):
    """One layer of the 70B shape: n_embd 8192 (the persistent step's ring
    stages shrink to leave room for its norm staging), ffn_down as two
    14336-input segments, 8 query heads per KV head."""
    import oracle
    key = "l70-1"
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    c = open_ctx(eng, m, eng.STAGE_FULL)
    assert c.path() == "persistent"
    prompt = synth.prompt_tokens(3, s.n_vocab, seed=70)
    om = oracle_port.model(buf)
    oe, ol, oh = om.ctx(0), om.ctx(1, 0, s.n_layer - 1), om.ctx(2)
    out, ob = np.zeros(s.n_embd + 1, np.float32), np.zeros(s.n_embd + 8, np.float32)
    for t in prompt:
        assert c.forward(t, out) == 0
        for o in (oe, ol, oh):
            assert o.forward(t, ob) == 0
        ok, err = vec_close(c.logits(), oh.logits(s.n_vocab))
        assert ok, f"logits rel err {err:.2e}"
    c.reset()
    assert c.generate(prompt, 4) == oracle.greedy(oracle_port, buf, prompt, 4)
