"""Failure detection on the device without a GPU fault.

Every wait inside the persistent step (a tagged word another CTA writes, a
bulk copy's barrier) is bounded: when it runs out, the kernel sets the
context's status word, gives up its remaining waits at once and runs to its
end, and the step returns -1.  Here a wait is made to run out on purpose --
ecu_inject_wait_timeout makes the next step wait for an input word that no
phase writes (a flag that nothing sets) -- with the limit shortened to
0.2 s.  The test checks the -1, the message, the time it took, and that the
same context then produces the oracle's greedy tokens again.  (The
reference's failure paths are host retries and aborts, src/shard.c:533-545.)
"""
import time

import numpy as np
import pytest

from distcomp_b200 import synth

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_context_recovers(eng, oracle_port, model_buf):
    import oracle
    key = "mini-q4"
    s = synth.spec(key)
    buf = model_buf(key)
    prompt = synth.prompt_tokens(6, s.n_vocab, seed=3)
    want = oracle.greedy(oracle_port, buf, prompt, 8)
    c = eng.LlmCtx(eng.GgufModel(buf), eng.STAGE_FULL, n_ctx=64)
    assert c.path() == "persistent"
    assert c.generate(prompt, 8) == want
    eng.set_wait_ns(200_000_000)
    try:
        out = np.zeros(s.n_embd + 1, dtype=np.float32)
        for _ in range(2):                          # twice: the recovery is complete
            c.reset()
            c.inject_wait_timeout()
            t0 = time.perf_counter()
            assert c.forward(prompt[0], out) == -1
            dt = time.perf_counter() - t0
            assert "bounded wait" in eng.last_error()
            assert 0.15 <= dt < 10.0, dt
            c.reset()
            assert c.generate(prompt, 8) == want
    finally:
        eng.set_wait_ns(2_000_000_000)
    c.close()


def test_injection_needs_the_persistent_step(eng, model_buf, monkeypatch):
    monkeypatch.setenv("ECU_MEGA", "0")
    c = eng.LlmCtx(eng.GgufModel(model_buf("mini-q4")), eng.STAGE_FULL, n_ctx=16)
    with pytest.raises(eng.EngineError, match="persistent"):
        c.inject_wait_timeout()
    with pytest.raises(eng.EngineError, match="positive"):
        eng.set_wait_ns(0)
    c.close()
