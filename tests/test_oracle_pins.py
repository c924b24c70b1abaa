"""Pins of the CPU oracle (oracle/dc_oracle.c) before anything is checked
against it: the reference's own known-answer vectors, fixtures produced by
the reference code, and -- where it is built -- the reference engine run live
on the same inputs.  CPU only."""
import numpy as np
import pytest

from distcomp_b200 import gguf as G
from distcomp_b200 import synth


def test_quant_test_vectors(oracle_port, golden):
    """tests/quant_test.c: 2 fixed blocks each of Q2_K/Q3_K/Q4_K/Q6_K, first 64
    weights per block against gguf-py, tolerance 1e-6*(|w|+1e-6) as there
    (quant_test.c:90)."""
    kq = golden("kquant_blocks.json")
    assert set(kq) == {"Q2_K", "Q3_K", "Q4_K", "Q6_K"}
    for name, d in kq.items():
        raw = np.array(d["blocks"], dtype=np.uint8).reshape(-1)
        rc, got = oracle_port.dequant(d["type"], raw, 512, 0, 512)
        assert rc == 0
        want = np.array(d["expect"], dtype=np.float32)
        for b in range(2):
            g = got[b * 256: b * 256 + 64]
            assert np.all(np.abs(g - want[b]) <= 1e-6 * (np.abs(want[b]) + 1e-6)), name


def test_dequant_fixtures_bit_exact(oracle_port, golden):
    """Every format on random blocks (fp16 specials included) equals the
    reference decoder bit for bit."""
    d = golden("dequant_blocks.npz")
    types = sorted({int(k.split("_")[1]) for k in d if k.startswith("raw_")})
    assert G.Q4_0 in types and G.Q8_0 in types and G.Q4_K in types and len(types) == 12
    for t in types:
        total, n = (int(v) for v in d[f"n_{t}"])
        rc, got = oracle_port.dequant(t, d[f"raw_{t}"], total, 0, n)
        assert rc == 0
        want = d[f"out_{t}"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"type {t}"


def test_dequant_rejections(oracle_port):
    """gguf_dequant's rules (src/gguf.c:733-786): range, block alignment,
    unsupported types, n = 0."""
    raw = np.zeros(34 * 8, dtype=np.uint8)
    assert oracle_port.dequant(G.Q8_0, raw, 256, 0, 0)[0] == 0
    assert oracle_port.dequant(G.Q8_0, raw, 256, 16, 32)[0] == -1      # off not on a block
    assert oracle_port.dequant(G.Q8_0, raw, 256, 240, 32)[0] == -1     # past the end
    assert oracle_port.dequant(G.Q8_0, raw, 256, 257, 1)[0] == -1
    assert oracle_port.dequant(G.Q8_1, raw, 256, 0, 32)[0] == -1       # unsupported
    assert oracle_port.dequant(16, raw, 256, 0, 32)[0] == -1           # IQ4_NL
    assert oracle_port.dequant(G.Q8_0, raw, 256, 0, 256)[0] == 0


def test_llama_ref_tiny_model(oracle_port, golden):
    """scripts/llama_ref.py's F32 model: token 1 -> the C engine's logits and
    greedy [234, 15, 155, 46] (what tests/engine_test.c prints), and the
    numpy forward of the script's own prompt within 1e-4."""
    import oracle
    buf = np.frombuffer(golden("llama_ref_tiny.gguf"), dtype=np.uint8).copy()
    j = golden("llama_ref_tiny.json")
    m = oracle_port.model(buf)
    emb, lay, head = m.ctx(0), m.ctx(1, 0, 3, 64), m.ctx(2)
    st = np.zeros(72, dtype=np.float32)
    assert emb.forward(1, st) == 0 and lay.forward(1, st) == 0 and head.forward(1, st) == 0
    lg = head.logits(256)
    assert np.array_equal(lg[:8], np.array(j["c_engine_token1_logits8"], dtype=np.float32))
    assert oracle.greedy(oracle_port, buf, [1], 4, n_ctx=64) == [234, 15, 155, 46]
    # numpy reference forward of the prompt ids the script used
    ids = j["prompt_ids"]
    for k, lay2 in ((0, m.ctx(1, 0, 3, 64)),):
        e2, h2 = m.ctx(0), m.ctx(2)
        for t in ids:
            assert e2.forward(t, st) == 0 and lay2.forward(t, st) == 0 and h2.forward(t, st) == 0
        got = h2.logits(256)[:16]
        want = np.array(j["logits"], dtype=np.float32)
        assert np.max(np.abs(got - want)) <= 1e-4 * max(1.0, np.max(np.abs(want)))
        assert int(np.argmax(h2.logits(256))) == j["greedy"]


@pytest.mark.parametrize("name,key,n_gen", [("tiny_q8", "tiny", 128), ("mini_q4", "mini-q4", 32),
                                            ("mini_q8", "mini-q8", 24)])
def test_engine_fixtures(oracle_port, golden, model_buf, name, key, n_gen):
    """Seeded models: the oracle reproduces the reference engine's greedy
    stream, first-step logits and per-layer states bit for bit."""
    import hashlib
    import oracle
    d = golden(f"{name}.npz")
    buf = model_buf(key)
    assert hashlib.sha256(buf).hexdigest() == bytes(d["model_sha256"]).decode(), "synthetic model drifted"
    prompt = [int(t) for t in d["prompt"]]
    assert oracle.greedy(oracle_port, buf, prompt, n_gen) == [int(t) for t in d["greedy"]]
    s = synth.spec(key)
    m = oracle_port.model(buf)
    emb, lay, head = m.ctx(0), m.ctx(1, 0, s.n_layer - 1), m.ctx(2)
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    assert emb.forward(prompt[0], st) == 0
    states = [st[: s.n_embd].copy()]
    for li in range(s.n_layer):
        assert lay.layer_once(li, st) == 0
        states.append(st[: s.n_embd].copy())
    assert np.array_equal(np.stack(states), d["layer_states"])
    lay.reset()
    emb2 = m.ctx(0)
    assert emb2.forward(prompt[0], st) == 0 and lay.forward(prompt[0], st) == 0 and head.forward(prompt[0], st) == 0
    assert np.array_equal(head.logits(s.n_vocab), d["logits_tok0"])


def test_oracle_matches_reference_live(oracle_port, oracle_ref, model_buf):
    """Where the reference engine is built (this container), the port and the
    reference agree bit for bit on a fresh seed and on every decoder."""
    import oracle
    buf = model_buf("mini-q4", seed=7)
    s = synth.spec("mini-q4")
    p = synth.prompt_tokens(6, s.n_vocab, seed=7)
    assert oracle.greedy(oracle_port, buf, p, 12) == oracle.greedy(oracle_ref, buf, p, 12)
    rng = np.random.default_rng(99)
    for t in (G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q8_0, G.Q2_K, G.Q3_K, G.Q4_K, G.Q5_K, G.Q6_K):
        be, bb = G.BLOCK[t]
        raw = rng.integers(0, 256, size=40 * bb, dtype=np.uint8)
        for off, n in ((0, 40 * be), (be * 3, be * 5 + 7)):
            r1, a = oracle_port.dequant(t, raw, 40 * be, off, n)
            r2, b = oracle_ref.dequant(t, raw, 40 * be, off, n)
            assert r1 == r2 == 0
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), t


def test_oracle_errors_match_reference(oracle_port, oracle_ref, model_buf):
    """Open-time errors: the same models are refused by both."""
    import oracle
    buf = model_buf("tiny")
    for kind in (oracle_port, oracle_ref):
        m = kind.model(buf)
        with pytest.raises(ValueError):
            m.ctx(1, 2, 9)            # layers outside the model
        with pytest.raises(ValueError):
            m.ctx(1, 3, 2)            # empty range
        c = m.ctx(0)
        st = np.zeros(300, dtype=np.float32)
        assert c.forward(-1, st) == -1 and c.forward(4096, st) == -1
        lay = m.ctx(1, 0, 3, 2)       # context of 2 positions
        assert lay.forward(5, st) == 0 and lay.forward(5, st) == 0 and lay.forward(5, st) == -1
    bad = buf.copy()
    bad[:4] = 0
    for kind in (oracle_port, oracle_ref):
        with pytest.raises(ValueError):
            kind.model(bad)
