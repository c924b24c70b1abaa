"""ctypes access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two interchangeable back ends with one interface:
  kind="port"  oracle/liboracle.so    -- the C restatement in dc_oracle.c
  kind="ref"   oracle/_ref/libdcref.so -- the reference engine compiled from
                                          its own sources by oracle/Makefile
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  The product (distcomp_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT = HERE / "liboracle.so"
REF = HERE / "_ref" / "libdcref.so"

_cache: dict = {}


def build(ref: bool = True) -> None:
    """make -C oracle (the reference part only where its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"] + (["ref"] if ref else []), check=True,
                   stdout=subprocess.DEVNULL)


def available(kind: str) -> bool:
    return (PORT if kind == "port" else REF).exists()


class OracleLib:
    def __init__(self, kind: str = "port"):
        self.kind = kind
        path = PORT if kind == "port" else REF
        if not path.exists():
            if kind == "port":
                build(ref=False)
            if not path.exists():
                raise FileNotFoundError(path)
        L = C.CDLL(str(path))
        p = "orc_" if kind == "port" else "refw_"
        self.p = p
        vp, i, sz, fp = C.c_void_p, C.c_int, C.c_size_t, C.c_void_p
        sig = {
            "model_open": (vp, [vp, sz, C.c_char_p, sz]),
            "model_close": (None, [vp]),
            "ctx_open": (vp, [vp, i, i, i, i, C.c_char_p, sz]),
            "ctx_close": (None, [vp]),
            "forward": (i, [vp, i, fp]),
            "layer_once": (i, [vp, i, fp]),
            "step_layers": (i, [vp, i, fp]),
            "pick": (i, [vp]),
            "reset": (None, [vp]),
            "set_pos": (None, [vp, i]),
            "logits": (C.POINTER(C.c_float), [vp]),
            "dequant": (i, [C.c_uint, vp, sz, sz, sz, fp]),
        }
        for k, (res, args) in sig.items():
            f = getattr(L, p + k)
            f.restype = res
            f.argtypes = args
            setattr(self, "_" + k, f)
        if kind == "port":
            L.orc_matvec.restype = None
            L.orc_matvec.argtypes = [C.c_uint, vp, i, i, fp, fp]
            L.orc_matvec_f64.restype = None
            L.orc_matvec_f64.argtypes = [C.c_uint, vp, i, i, fp, fp]
            L.orc_f16.restype = C.c_float
            L.orc_f16.argtypes = [C.c_uint16]
        else:
            L.refw_set_threads.restype = None
            L.refw_set_threads.argtypes = [i]
            L.refw_threads.restype = i
        self.L = L

    # ------------------------------------------------------------------
    def model(self, buf: np.ndarray) -> "OModel":
        return OModel(self, buf)

    def dequant(self, gtype: int, raw: np.ndarray, total: int, off: int, n: int):
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        # the reference writes whole blocks past n (src/gguf.c:769-783): room for one more
        out = np.zeros(n + 256, dtype=np.float32)
        rc = self._dequant(gtype, raw.ctypes.data, total, off, n, out.ctypes.data)
        return int(rc), out[:n]

    def matvec(self, gtype, raw, n_in, n_out, x):
        y = np.empty(n_out, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        self.L.orc_matvec(gtype, raw.ctypes.data, n_in, n_out, x.ctypes.data, y.ctypes.data)
        return y

    def matvec_f64(self, gtype, raw, n_in, n_out, x):
        y = np.empty(n_out, dtype=np.float64)
        x = np.ascontiguousarray(x, dtype=np.float32)
        self.L.orc_matvec_f64(gtype, raw.ctypes.data, n_in, n_out, x.ctypes.data, y.ctypes.data)
        return y

    def set_threads(self, n: int) -> None:
        if self.kind == "ref":
            self.L.refw_set_threads(int(n))


def get(kind: str = "port") -> OracleLib:
    if kind not in _cache:
        _cache[kind] = OracleLib(kind)
    return _cache[kind]


class OModel:
    def __init__(self, lib: OracleLib, buf: np.ndarray):
        self.lib = lib
        self.buf = buf      # keep alive: tensors point into it
        err = C.create_string_buffer(512)
        self.h = lib._model_open(buf.ctypes.data, buf.nbytes, err, 512)
        if not self.h:
            raise ValueError(err.value.decode(errors="replace"))

    def ctx(self, stage: int, first: int = 0, last: int = 0, n_ctx: int = 0) -> "OCtx":
        return OCtx(self, stage, first, last, n_ctx)

    def close(self):
        if self.h:
            self.lib._model_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OCtx:
    def __init__(self, model: OModel, stage, first, last, n_ctx):
        self.model = model
        self.lib = model.lib
        err = C.create_string_buffer(512)
        self.h = self.lib._ctx_open(model.h, stage, first, last, n_ctx, err, 512)
        if not self.h:
            raise ValueError(err.value.decode(errors="replace"))

    def forward(self, token: int, out: np.ndarray) -> int:
        return int(self.lib._forward(self.h, int(token), out.ctypes.data))

    def layer_once(self, idx: int, out: np.ndarray) -> int:
        return int(self.lib._layer_once(self.h, int(idx), out.ctypes.data))

    def step_layers(self, n: int, out: np.ndarray) -> int:
        return int(self.lib._step_layers(self.h, int(n), out.ctypes.data))

    def pick(self) -> int:
        return int(self.lib._pick(self.h))

    def reset(self) -> None:
        self.lib._reset(self.h)

    def set_pos(self, pos: int) -> None:
        self.lib._set_pos(self.h, int(pos))

    def logits(self, n_vocab: int) -> np.ndarray:
        p = self.lib._logits(self.h)
        return np.ctypeslib.as_array(p, shape=(n_vocab,)).copy()

    def close(self):
        if self.h:
            self.lib._ctx_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def greedy(lib: OracleLib, buf: np.ndarray, prompt, n_gen: int, n_ctx: int = 0):
    """The reference's three-stage local run (src/shard.c:470-505): embed ->
    layers -> head per token, prompt token by token, then greedy decode.
    Returns the n_gen generated tokens."""
    m = lib.model(buf)
    emb, lay, head = m.ctx(0), None, m.ctx(2)
    lay = m.ctx(1, 0, _n_layer(buf) - 1, n_ctx)
    n_embd = _n_embd(buf)
    state = np.zeros(n_embd + 8, dtype=np.float32)
    out = []
    tok = None
    for t in prompt:
        assert emb.forward(t, state) == 0 and lay.forward(t, state) == 0 and head.forward(t, state) == 0
        tok = int(state[n_embd])
    for _ in range(n_gen):
        out.append(tok)
        if len(out) == n_gen:
            break
        assert emb.forward(tok, state) == 0 and lay.forward(tok, state) == 0 and head.forward(tok, state) == 0
        tok = int(state[n_embd])
    return out


def _meta(buf):
    from distcomp_b200.gguf import read_tensor_table
    return read_tensor_table(buf)["__meta__"]


def _n_layer(buf):
    m = _meta(buf)
    return int(m[m["general.architecture"] + ".block_count"])


def _n_embd(buf):
    m = _meta(buf)
    return int(m[m["general.architecture"] + ".embedding_length"])


if os.environ.get("ORACLE_AUTOBUILD") == "1":
    build()
