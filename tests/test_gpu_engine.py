"""GPU parity of the whole token loop against the reference engine's
fixtures and the live oracle: per-layer states and logits within 1e-3
(relative to the vector's scale), identical greedy streams, the stage /
position / error contract of llm_forward, and the repacked device copy of
every weight bit-exact with the file."""
import numpy as np
import pytest
from conftest import bits_equal

from distcomp_b200 import gguf as G
from distcomp_b200 import synth

pytestmark = pytest.mark.gpu

REL = 1e-3


def vec_close(a, b, rel=REL):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.max(np.abs(b)), 1e-30)
    return float(np.max(np.abs(a - b)) / scale) <= rel, float(np.max(np.abs(a - b)) / scale)


def three_stage(eng, buf, n_layer, n_ctx=0):
    m = eng.GgufModel(buf)
    return m, (eng.LlmCtx(m, eng.STAGE_EMBED), eng.LlmCtx(m, eng.STAGE_LAYERS, 0, n_layer - 1, n_ctx),
               eng.LlmCtx(m, eng.STAGE_HEAD))


def greedy_stages(ctxs, prompt, n_gen, n_embd):
    emb, lay, head = ctxs
    st = np.zeros(n_embd + 8, dtype=np.float32)
    out, tok = [], None
    for t in prompt:
        assert emb.forward(t, st) == 0 and lay.forward(t, st) == 0 and head.forward(t, st) == 0
        tok = int(st[n_embd])
    while len(out) < n_gen:
        out.append(tok)
        if len(out) == n_gen:
            break
        assert emb.forward(tok, st) == 0 and lay.forward(tok, st) == 0 and head.forward(tok, st) == 0
        tok = int(st[n_embd])
    return out


@pytest.mark.parametrize("name,key,n_gen", [("tiny_q8", "tiny", 128), ("mini_q4", "mini-q4", 32),
                                            ("mini_q8", "mini-q8", 24)])
def test_stages_match_reference_fixture(eng, golden, model_buf, name, key, n_gen):
    d = golden(f"{name}.npz")
    s = synth.spec(key)
    buf = model_buf(key)
    prompt = [int(t) for t in d["prompt"]]
    m, (emb, lay, head) = three_stage(eng, buf, s.n_layer)
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    # per-layer states of the first token (tests/engine_stages.c pattern)
    assert emb.forward(prompt[0], st) == 0
    assert np.array_equal(st[: s.n_embd], d["layer_states"][0])      # embedding row: exact
    for li in range(s.n_layer):
        assert lay.layer_once(li, st) == 0
        ok, err = vec_close(st[: s.n_embd], d["layer_states"][li + 1])
        assert ok, f"layer {li}: rel err {err:.2e}"
    lay.reset()
    assert emb.forward(prompt[0], st) == 0 and lay.forward(prompt[0], st) == 0 and head.forward(prompt[0], st) == 0
    ok, err = vec_close(head.logits(), d["logits_tok0"])
    assert ok, f"logits rel err {err:.2e}"
    for c in (emb, lay, head):
        c.reset()
    assert greedy_stages((emb, lay, head), prompt, n_gen, s.n_embd) == [int(t) for t in d["greedy"]]


@pytest.mark.parametrize("name,key,n_gen", [("tiny_q8", "tiny", 128), ("mini_q4", "mini-q4", 32)])
def test_full_context_generate(eng, golden, model_buf, name, key, n_gen):
    """One FULL context, device-side token feedback (CUDA graph replays)."""
    d = golden(f"{name}.npz")
    m = eng.GgufModel(model_buf(key))
    c = eng.LlmCtx(m, eng.STAGE_FULL)
    prompt = [int(t) for t in d["prompt"]]
    assert c.generate(prompt, n_gen) == [int(t) for t in d["greedy"]]
    assert c.pos == len(prompt) + n_gen - 1
    c.reset()
    assert c.generate(prompt, n_gen) == [int(t) for t in d["greedy"]]


def test_full_forward_contract(eng, golden, model_buf):
    """FULL ecu_forward: out[0..n_embd) = normed state, out[n_embd] = argmax."""
    d = golden("tiny_q8.npz")
    s = synth.spec("tiny")
    m = eng.GgufModel(model_buf("tiny"))
    c = eng.LlmCtx(m, eng.STAGE_FULL)
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    toks = []
    for t in [int(x) for x in d["prompt"]]:
        assert c.forward(t, out) == 0
        toks.append(int(out[s.n_embd]))
    assert toks[-1] == int(d["greedy"][0])
    assert c.pick() == toks[-1]
    ok, _ = vec_close(c.logits(), d["logits_last_prompt"])
    assert ok
    # normed state has unit RMS (norm weights are 1.0)
    assert abs(np.sqrt(np.mean(out[: s.n_embd].astype(np.float64) ** 2)) - 1.0) < 1e-3


def test_llama_ref_tiny_greedy(eng, golden):
    """scripts/llama_ref.py's F32 model: token 1 -> [234, 15, 155, 46]
    (tests/engine_test.c with the reference engine)."""
    buf = np.frombuffer(golden("llama_ref_tiny.gguf"), dtype=np.uint8).copy()
    j = golden("llama_ref_tiny.json")
    m, ctxs = three_stage(eng, buf, 4, 64)
    st = np.zeros(72, dtype=np.float32)
    emb, lay, head = ctxs
    assert emb.forward(1, st) == 0 and lay.forward(1, st) == 0 and head.forward(1, st) == 0
    ok, _ = vec_close(head.logits()[:8], np.array(j["c_engine_token1_logits8"]))
    assert ok
    for c in ctxs:
        c.reset()
    assert greedy_stages(ctxs, [1], 4, 64) == [234, 15, 155, 46]


@pytest.mark.parametrize("over", [dict(qkv_bias=True, arch="qwen2"), dict(head_dim=64),
                                  dict(tied=True), dict(n_head_kv=2)])
def test_variants_vs_live_oracle(eng, oracle_port, model_buf, over):
    """Qwen2 biases, rope.dimension_count != n_embd/n_head, tied embeddings,
    GQA: per-token logits and greedy stream against the oracle run live."""
    import oracle
    key = "tiny"
    s = synth.spec(key, **over)
    buf = synth.build_model(s, seed=3)
    prompt = synth.prompt_tokens(5, s.n_vocab, seed=3)
    want = oracle.greedy(oracle_port, buf, prompt, 12)
    m, ctxs = three_stage(eng, buf, s.n_layer)
    assert greedy_stages(ctxs, prompt, 12, s.n_embd) == want
    om = oracle_port.model(buf)
    oe, ol, oh = om.ctx(0), om.ctx(1, 0, s.n_layer - 1), om.ctx(2)
    for c in ctxs:
        c.reset()
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    so = st.copy()
    for t in prompt:
        for g, o in zip(ctxs, (oe, ol, oh)):
            assert g.forward(t, st) == 0 and o.forward(t, so) == 0
        ok, err = vec_close(ctxs[2].logits(), oh.logits(s.n_vocab))
        assert ok, err


def test_forward_errors_and_positions(eng, model_buf):
    s = synth.spec("tiny")
    m = eng.GgufModel(model_buf("tiny"))
    emb = eng.LlmCtx(m, eng.STAGE_EMBED)
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    assert emb.forward(-1, st) == -1 and emb.forward(s.n_vocab, st) == -1
    assert emb.forward(s.n_vocab - 1, st) == 0
    lay = eng.LlmCtx(m, eng.STAGE_LAYERS, 1, 2, 3)
    for i in range(3):
        assert lay.forward(0, st) == 0
    assert lay.forward(0, st) == -1                 # context exhausted
    assert lay.step_layers(0, st) == -1
    lay.reset()
    assert lay.pos == 0 and lay.step_layers(1, st) == 0 and lay.pos == 1
    assert lay.layer_once(2, st) == -1 and lay.layer_once(1, st) == 0 and lay.pos == 1
    full = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=4)
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    assert full.forward(4096, out) == -1
    with pytest.raises(eng.EngineError):
        full.generate([5, 6, 7], 3)                 # 3 + 3 - 1 > 4 positions
    assert full.generate([5, 6], 3) is not None


def test_partial_step_layers_matches_oracle(eng, oracle_port, model_buf):
    """llm_step_layers with n < all layers (eager path) and layer_once."""
    s = synth.spec("mini-q4")
    buf = model_buf("mini-q4")
    m = eng.GgufModel(buf)
    g = eng.LlmCtx(m, eng.STAGE_LAYERS, 0, 1)
    o = oracle_port.model(buf).ctx(1, 0, 1)
    rng = np.random.default_rng(0)
    for _ in range(3):
        x = rng.standard_normal(s.n_embd).astype(np.float32)
        a, b = x.copy(), x.copy()
        assert g.step_layers(1, a) == 0 and o.step_layers(1, b) == 0
        ok, err = vec_close(a, b)
        assert ok, err


def test_repacked_weights_bit_exact(eng, oracle_port, model_buf):
    """Every uploaded tensor read back through its device layout (SPLIT4/
    SPLIT8 rows, fused Q/K/V, interleaved gate/up) equals the oracle's
    dequant of the file bytes."""
    for key in ("mini-q4", "mini-q8", "tiny"):
        s = synth.spec(key)
        buf = model_buf(key)
        m = eng.GgufModel(buf)
        c = eng.LlmCtx(m, eng.STAGE_FULL)
        tab = G.read_tensor_table(buf)
        for name, dims, gt in synth.tensor_list(s):
            if name.endswith("norm.weight"):
                continue
            total = int(np.prod(dims))
            got = c.dequant_tensor(name, 0, total)
            rc, want = oracle_port.dequant(gt, np.frombuffer(tab[name][2], np.uint8), total, 0, total)
            assert rc == 0
            assert bits_equal(got, want), name


def test_context_from_mapped_file(eng, oracle_port, model_buf, tmp_path, monkeypatch):
    """A model opened from a GGUF file (ecu_model_open_file: mapped, a
    stage's context pages in its tensors only), its weights uploaded in small
    pinned chunks (ECU_UPLOAD_MB=1: every matrix in several chunks): the
    oracle's greedy tokens, and a LAYERS stage's state within 1e-3."""
    import oracle
    key = "mini-q4"
    s = synth.spec(key)
    buf = model_buf(key)
    path = tmp_path / "m.gguf"
    path.write_bytes(buf.tobytes())
    monkeypatch.setenv("ECU_UPLOAD_MB", "1")
    m = eng.GgufModel(path=str(path))
    prompt = synth.prompt_tokens(5, s.n_vocab, seed=8)
    want = oracle.greedy(oracle_port, buf, prompt, 8)
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=32)
    assert c.generate(prompt, 8) == want
    lay = eng.LlmCtx(m, eng.STAGE_LAYERS, 1, 1, n_ctx=32)
    o = oracle_port.model(buf).ctx(1, 1, 1)
    x = np.random.default_rng(2).standard_normal(s.n_embd).astype(np.float32)
    a, b = x.copy(), x.copy()
    assert lay.forward(0, a) == 0 and o.forward(0, b) == 0
    ok, err = vec_close(a, b)
    assert ok, err
    c.close()
    lay.close()
    m.close()
