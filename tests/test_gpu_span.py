"""Span contexts (ecu_ctx_open_span): a layer range with the embedding and/or
the head folded in, the unit a pipeline rank runs per token; a range may
start at a layer's FFN half or end at its attention half.

A chain of spans fed token by token through the host API must produce the
FULL context's states, greedy tokens and logits bit for bit -- a span
boundary moves the state between buffers and changes no arithmetic -- on the
persistent step and on the per-kernel step (ECU_MEGA=0), including a span
that holds the head alone and spans that hold half of a layer."""
import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu


def full_run(eng, m, s, prompt, n_gen, n_ctx):
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    toks, states = [], []
    tok = prompt[0]
    for i in range(len(prompt) + n_gen - 1):
        assert c.forward(tok, out) == 0
        states.append(out.copy())
        nxt = int(out[s.n_embd])
        toks.append(nxt)
        tok = prompt[i + 1] if i + 1 < len(prompt) else nxt
    logits = c.logits()
    c.close()
    return toks, states, logits


def span_run(eng, m, s, plan, prompt, n_gen, n_ctx):
    """plan: [(first, last, flags)] in pipeline order."""
    spans = [eng.LlmCtx(m, eng.STAGE_SPAN, a, b, n_ctx, span=f) for a, b, f in plan]
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    toks, states = [], []
    tok = prompt[0]
    for i in range(len(prompt) + n_gen - 1):
        for c in spans:
            assert c.forward(tok, out) == 0
        states.append(out.copy())
        nxt = int(out[s.n_embd])
        assert nxt == spans[-1].pick()
        toks.append(nxt)
        tok = prompt[i + 1] if i + 1 < len(prompt) else nxt
    logits = spans[-1].logits()
    paths = [c.path() for c in spans]
    for c in spans:
        c.close()
    return toks, states, logits, paths


@pytest.mark.parametrize("mega", ["1", "0"])
@pytest.mark.parametrize("key", ["mini-q4", "mini-q8"])
def test_span_chain_matches_full(eng, model_buf, monkeypatch, mega, key):
    monkeypatch.setenv("ECU_MEGA", mega)
    over = {"n_layer": 4}
    s = synth.spec(key, **over)
    m = eng.GgufModel(model_buf(key, **over))
    prompt = synth.prompt_tokens(5, s.n_vocab, seed=31)
    n_gen, n_ctx = 6, 32
    want_t, want_s, want_l = full_run(eng, m, s, prompt, n_gen, n_ctx)
    E, H = eng.SPAN_EMBED, eng.SPAN_HEAD
    FF, AL = eng.SPAN_FFN_FIRST, eng.SPAN_ATTN_LAST
    for plan in ([(0, 1, E), (2, 3, H)],              # entry node embeds, exit node picks
                 [(0, 0, E), (1, 2, 0), (3, 3, H)],   # a middle span of layers only
                 [(0, 3, E), (4, 3, H)],              # the head alone
                 [(0, 3, E | H)],                     # everything: FULL's work as a span
                 [(0, 1, E | AL), (1, 3, FF | H)],    # layer 1 cut between its halves
                 [(0, 0, E | AL), (0, 2, FF | AL), (2, 3, FF | H)],   # two cuts, a span cut at both ends
                 [(0, 3, E | AL), (3, 3, FF | H)]):   # the last FFN half with the head
        got_t, got_s, got_l, paths = span_run(eng, m, s, plan, prompt, n_gen, n_ctx)
        assert got_t == want_t, plan
        for a, b in zip(got_s, want_s):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), plan
        assert np.array_equal(got_l.view(np.uint32), want_l.view(np.uint32)), plan
        if mega == "1":
            assert all(p == "persistent" for p in paths), (plan, paths)


def test_span_forks_and_step_dev(eng, model_buf):
    """Forked spans (one per sequence) stepped from device-resident input:
    the first span's token word in, the last span's token word out."""
    import torch
    from distcomp_b200 import pipeline as P
    key, over = "mini-q4", {"n_layer": 4}
    s = synth.spec(key, **over)
    m = eng.GgufModel(model_buf(key, **over))
    prompt = synth.prompt_tokens(4, s.n_vocab, seed=8)
    want_t, _, _ = full_run(eng, m, s, prompt, 5, 32)
    a = eng.LlmCtx(m, eng.STAGE_SPAN, 0, 1, 32, span=eng.SPAN_EMBED)
    b = eng.LlmCtx(m, eng.STAGE_SPAN, 2, 3, 32, span=eng.SPAN_HEAD)
    a2, b2 = a.fork(), b.fork()
    assert a2.path() == "persistent" and b2.path() == "persistent"
    ne = s.n_embd
    st = torch.cuda.Stream()
    sa = P.device_view(a2.state_ptr(), ne + 1, "<f4", 0)
    sb = P.device_view(b2.state_ptr(), ne + 1, "<f4", 0)
    ta = P.device_view(a2.token_ptr(), 1, "<i4", 0)
    tb = P.device_view(b2.token_ptr(), 1, "<i4", 0)
    got = []
    with torch.cuda.stream(st):
        for i in range(len(prompt) + 4):
            if i < len(prompt):
                ta.fill_(prompt[i])
            else:
                ta.copy_(tb)
            a2.step_dev(st.cuda_stream)
            sb[:ne].copy_(sa[:ne])
            b2.step_dev(st.cuda_stream)
            got.append(tb.clone())
    st.synchronize()
    assert [int(t.item()) for t in got] == want_t
    for c in (a2, b2, a, b):
        c.close()
