"""The C-ABI library on the CPU: it loads, exports every entry point the
header declares, and its host-side GGUF view follows the reference reader's
acceptance rules.  No kernel runs here."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from distcomp_b200 import engine, synth
from distcomp_b200 import gguf as G

HEADER = Path(__file__).resolve().parents[1] / "include" / "engine_cuda.h"


def declared_functions():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ecu_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported():
    L = engine.lib()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    bound = {n for n, _, _ in engine.SIGNATURES}
    assert set(names) <= bound, set(names) - bound


def test_version_and_counters():
    assert b"sm_100a" in engine.lib().ecu_version()
    assert engine.kernel_launches() >= 0


def test_model_open_reads_metadata(model_buf):
    buf = model_buf("tiny")
    m = engine.GgufModel(buf)
    s = synth.spec("tiny")
    assert m.n_tensors() == len(synth.tensor_list(s))
    t, dims, ptr, nb = m.tensor("blk.0.attn_q.weight")
    assert t == G.Q8_0 and dims == [256, 256] and nb == 256 * 256 // 32 * 34
    assert ptr >= buf.ctypes.data and ptr + nb <= buf.ctypes.data + buf.nbytes
    t, dims, _, _ = m.tensor("blk.0.ffn_down.weight")
    assert t == G.F32 and dims == [688, 256]
    with pytest.raises(KeyError):
        m.tensor("nope")
    # the bytes it points at are the builder's
    tab = G.read_tensor_table(buf)
    mv = tab["output.weight"][2]
    _, _, ptr, nb = m.tensor("output.weight")
    assert bytes(mv) == C.string_at(ptr, nb)


def _mutations(buf):
    """Malformed variants of a valid image: (description, bytes)."""
    out = []
    b = buf.copy(); b[:4] = np.frombuffer(b"GGUX", np.uint8); out.append(("magic", b))
    b = buf.copy(); b[4] = 4; out.append(("version 4", b))
    b = buf.copy(); b[4] = 1; out.append(("version 1", b))
    out.append(("truncated header", buf[:20].copy()))
    out.append(("truncated data", buf[: buf.nbytes - 1000].copy()))
    b = buf.copy(); b[8:16] = np.frombuffer(np.uint64(0).tobytes(), np.uint8); out.append(("no tensors", b))
    b = buf.copy(); b[8:16] = np.frombuffer(np.uint64(5000).tobytes(), np.uint8); out.append(("too many tensors", b))
    b = buf.copy(); b[16:24] = np.frombuffer(np.uint64(1 << 40).tobytes(), np.uint8); out.append(("huge kv count", b))
    return out


def test_model_open_rejects_like_the_reference(model_buf, oracle_port):
    buf = model_buf("tiny")
    engine.GgufModel(buf)
    oracle_port.model(buf)
    for what, b in _mutations(buf):
        with pytest.raises(engine.EngineError):
            engine.GgufModel(b)
        with pytest.raises(ValueError):
            oracle_port.model(b)


def test_model_open_error_message():
    bad = np.zeros(100, dtype=np.uint8)
    with pytest.raises(engine.EngineError, match="magic"):
        engine.GgufModel(bad)
    with pytest.raises(engine.EngineError, match="too small"):
        engine.GgufModel(np.zeros(10, dtype=np.uint8))


def test_model_from_views_like_dcd():
    """dcd assembles a gguf_file from received tensors (src/daemon.c:963-
    1019); ecu_model_new/add_tensor/set_* do the same."""
    L = engine.lib()
    h = L.ecu_model_new()
    assert h
    w = np.ones(64 * 32, dtype=np.float32)
    dims = (C.c_uint64 * 2)(64, 32)
    assert L.ecu_model_add_tensor(h, b"token_embd.weight", 2, dims, 0, w.ctypes.data, w.nbytes) == 0
    assert L.ecu_model_add_tensor(h, b"bad", 2, dims, 0, w.ctypes.data, 10) == -1   # too few bytes
    assert L.ecu_model_set_str(h, b"general.architecture", b"llama") == 0
    assert L.ecu_model_set_u32(h, b"llama.embedding_length", 64) == 0
    assert L.ecu_model_n_tensors(h) == 1
    L.ecu_model_close(h)


def test_ctx_bytes_host_only(model_buf):
    """Device footprint planning (llm_ctx_floats' counterpart) needs no GPU."""
    m = engine.GgufModel(model_buf("tiny"))
    lay = engine.ctx_bytes(m, engine.STAGE_LAYERS, 0, 3, 256)
    half = engine.ctx_bytes(m, engine.STAGE_LAYERS, 0, 1, 256)
    assert lay > half > 0
    assert engine.ctx_bytes(m, engine.STAGE_LAYERS, 0, 7, 256) == 0      # outside the model
    assert engine.ctx_bytes(m, engine.STAGE_HEAD) > 0
    kv = 2 * 4 * 256 * 256 * 4
    assert lay >= kv


def test_ctx_open_without_gpu_fails_loudly(model_buf):
    from conftest import HAS_GPU
    if HAS_GPU:
        pytest.skip("a GPU is present")
    m = engine.GgufModel(model_buf("tiny"))
    with pytest.raises(engine.EngineError, match="CUDA device"):
        engine.LlmCtx(m, engine.STAGE_FULL)


def test_ctx_open_geometry_errors(model_buf):
    """The reference's open-time checks run before any device work."""
    m = engine.GgufModel(model_buf("tiny"))
    with pytest.raises(engine.EngineError, match="outside the model"):
        engine.LlmCtx(m, engine.STAGE_LAYERS, 2, 9)
    with pytest.raises(engine.EngineError, match="unknown stage"):
        engine.LlmCtx(m, 7)
    # spans: a range inside the model, known flags, something to do
    with pytest.raises(engine.EngineError, match="outside the model"):
        engine.LlmCtx(m, engine.STAGE_SPAN, 1, 5, span=engine.SPAN_HEAD)
    with pytest.raises(engine.EngineError, match="span flags"):
        engine.LlmCtx(m, engine.STAGE_SPAN, 0, 0, span=16)
    with pytest.raises(engine.EngineError, match="needs the embedding or the head"):
        engine.LlmCtx(m, engine.STAGE_SPAN, 1, 0, span=0)
    with pytest.raises(engine.EngineError, match="neither its attention nor its FFN half"):
        engine.LlmCtx(m, engine.STAGE_SPAN, 1, 1, span=engine.SPAN_FFN_FIRST | engine.SPAN_ATTN_LAST)


def test_ctx_bytes_q4k_segments_host_only(model_buf):
    """Q4_K weights in their device layout (18 bytes per 32 weights, the GGUF
    size) and an ffn_down wider than one column segment cost exactly their
    file bytes on the device: the footprint is the layers' tensor bytes plus
    the KV cache and bounded work buffers."""
    from distcomp_b200 import gguf as G
    from distcomp_b200 import synth
    s = synth.spec("wide-q4k")
    m = engine.GgufModel(model_buf("wide-q4k"))
    n_ctx = 96
    got = engine.ctx_bytes(m, engine.STAGE_LAYERS, 0, s.n_layer - 1, n_ctx)
    w = sum(G.type_nbytes(gt, int(np.prod(dims))) for name, dims, gt in synth.tensor_list(s)
            if name.startswith("blk.") and "norm" not in name)
    hd = s.n_embd // s.n_head
    kv = 2 * s.n_layer * n_ctx * s.n_head_kv * hd * 4
    assert w + kv <= got <= w + kv + (8 << 20)


def test_model_open_file_maps_the_same_tensors(model_buf, tmp_path):
    """ecu_model_open_file maps a GGUF file: the same tensor table as the
    in-memory open, every tensor's bytes the file's."""
    buf = model_buf("mini-q4")
    path = tmp_path / "m.gguf"
    path.write_bytes(buf.tobytes())
    a = engine.GgufModel(buf)
    b = engine.GgufModel(path=str(path))
    assert a.n_tensors() == b.n_tensors()
    for name, dims, gt in synth.tensor_list(synth.spec("mini-q4")):
        ta, da, _, na = a.tensor(name)
        tb, db, pb, nb = b.tensor(name)
        assert (ta, da, na) == (tb, db, nb)
        assert bytes(G.read_tensor_table(buf)[name][2]) == C.string_at(pb, nb), name
    b.close()
    with pytest.raises(engine.EngineError, match="cannot open"):
        engine.GgufModel(path=str(tmp_path / "missing.gguf"))
