"""ecu_prefill: the prompt as one batch per layer (tensor-core GEMMs), against
the per-token path and the oracle.

After the prompt the logits and the normed state must agree with feeding the
prompt token by token within the 1e-3 bar (relative to the vector's scale),
the picked token must be the same, and greedy decoding that continues from
the prefilled cache must give the oracle's tokens (the reference engine
restated, fed token by token).  A prompt prefilled in two pieces (the second
at a nonzero position) must match one piece.  The tiny shape (head_dim 32)
takes the per-token fallback and is checked the same way.
"""
import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu
REL = 1e-3


def vec_close(a, b, rel=REL):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.max(np.abs(b)), 1e-30)
    err = float(np.max(np.abs(a - b)) / scale)
    return err <= rel, err


def continue_greedy(ctx, first, n, n_embd):
    out = np.zeros(n_embd + 1, dtype=np.float32)
    toks, tok = [first], first
    while len(toks) < n:
        assert ctx.forward(tok, out) == 0
        tok = int(out[n_embd])
        toks.append(tok)
    return toks


@pytest.mark.parametrize("key,n_prompt", [("mini-q4", 40), ("mini-q8", 33), ("mini-q4", 1), ("tiny", 12)])
def test_prefill_matches_per_token_and_oracle(eng, oracle_port, model_buf, key, n_prompt):
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    prompt = synth.prompt_tokens(n_prompt, s.n_vocab, seed=21)
    a = eng.LlmCtx(m, eng.STAGE_FULL)
    b = eng.LlmCtx(m, eng.STAGE_FULL)
    out_a = np.zeros(s.n_embd + 1, dtype=np.float32)
    out_b = np.zeros(s.n_embd + 1, dtype=np.float32)
    first = a.prefill(prompt, out_a)
    for t in prompt:
        assert b.forward(t, out_b) == 0
    assert a.pos == b.pos == n_prompt
    assert first == int(out_b[s.n_embd]) == a.pick()
    ok, err = vec_close(a.logits(), b.logits())
    assert ok, f"logits rel err {err:.2e}"
    ok, err = vec_close(out_a[: s.n_embd], out_b[: s.n_embd])
    assert ok, f"state rel err {err:.2e}"
    n_gen = min(24, s.n_ctx - n_prompt)
    got = continue_greedy(a, first, n_gen, s.n_embd)
    assert got == oracle.greedy(oracle_port, buf, prompt, n_gen)


def test_prefill_in_two_pieces(eng, model_buf):
    key = "mini-q4"
    s = synth.spec(key)
    m = eng.GgufModel(model_buf(key))
    prompt = synth.prompt_tokens(30, s.n_vocab, seed=5)
    one = eng.LlmCtx(m, eng.STAGE_FULL)
    two = eng.LlmCtx(m, eng.STAGE_FULL)
    t1 = one.prefill(prompt)
    two.prefill(prompt[:11])
    t2 = two.prefill(prompt[11:])
    assert t1 == t2 and one.pos == two.pos == 30
    ok, err = vec_close(two.logits(), one.logits())
    assert ok, err
    assert continue_greedy(one, t1, 16, s.n_embd) == continue_greedy(two, t2, 16, s.n_embd)


@pytest.mark.parametrize("key", ["mini-q4", "mini-q8"])
def test_prefill_long_prompt(eng, oracle_port, model_buf, key):
    """300 prompt tokens (3 row tiles of the tensor-core GEMM, ~10 key
    chunks of the prefill attention, a partial last query block) against the
    per-token path and the oracle; and the same prompt in two pieces, the
    second starting at position 150 (inside a key chunk and a row tile)."""
    import oracle
    s = synth.spec(key)
    buf = model_buf(key)
    m = eng.GgufModel(buf)
    n_ctx, n_prompt = 512, 300
    prompt = synth.prompt_tokens(n_prompt, s.n_vocab, seed=17)
    a = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    b = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    out_b = np.zeros(s.n_embd + 1, dtype=np.float32)
    first = a.prefill(prompt)
    for t in prompt:
        assert b.forward(t, out_b) == 0
    assert first == int(out_b[s.n_embd])
    ok, err = vec_close(a.logits(), b.logits())
    assert ok, f"logits rel err {err:.2e}"
    c.prefill(prompt[:150])
    t2 = c.prefill(prompt[150:])
    assert t2 == first and c.pos == a.pos == n_prompt
    ok, err = vec_close(c.logits(), a.logits())
    assert ok, f"two pieces: logits rel err {err:.2e}"
    want = oracle.greedy(oracle_port, buf, prompt, 8, n_ctx=n_ctx)
    assert continue_greedy(a, first, 8, s.n_embd) == want
    assert continue_greedy(c, t2, 8, s.n_embd) == want
    for x in (a, b, c):
        x.close()


def test_prefill_errors(eng, model_buf):
    key = "mini-q4"
    s = synth.spec(key)
    m = eng.GgufModel(model_buf(key))
    c = eng.LlmCtx(m, eng.STAGE_FULL)
    with pytest.raises(eng.EngineError, match="vocabulary"):
        c.prefill([1, s.n_vocab])
    with pytest.raises(eng.EngineError, match="exceeds the context"):
        c.prefill([1] * (s.n_ctx + 1))
    assert c.pos == 0
    lay = eng.LlmCtx(m, eng.STAGE_LAYERS, 0, s.n_layer - 1)
    with pytest.raises(eng.EngineError, match="FULL"):
        lay.prefill([1, 2])
