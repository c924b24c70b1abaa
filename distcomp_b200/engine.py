"""Python host mirror of the reference engine API over the CUDA library.

The classes mirror src/engine.h:72-101 and src/gguf.h:52-90 name for name:

    GgufModel(buf)                 gguf_open            (gguf.h:52)
    LlmCtx(model, stage, first, last, n_ctx, device)
                                   llm_ctx_open         (engine.h:79)
    ctx.forward(token, out)        llm_forward          (engine.h:88)
    ctx.reset()                    llm_reset            (engine.h:90)
    ctx.layer_once(i, out)         llm_layer_once       (engine.h:94)
    ctx.step_layers(n, out)        llm_step_layers      (engine.h:98)
    ctx.pick()                     llm_pick             (engine.h:101)
    ctx_floats(...) / ctx_bytes    llm_ctx_floats       (engine.h:74)
    dequant(type, raw, total, off, n)
                                   gguf_dequant         (gguf.h:86)

Errors follow the reference: open raises EngineError with the message the C
side wrote into `err`; forward/step/layer_once return 0 or -1.  Everything
runs in libdcb200.so on the GPU: there is no CPU path here, and loading
fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

STAGE_EMBED, STAGE_LAYERS, STAGE_HEAD, STAGE_FULL, STAGE_SPAN = 0, 1, 2, 3, 4
SPAN_EMBED, SPAN_HEAD, SPAN_FFN_FIRST, SPAN_ATTN_LAST = 1, 2, 4, 8

_LIB = None
_LIB_PATH = Path(__file__).resolve().parent / "libdcb200.so"


class EngineError(RuntimeError):
    pass


class EcuInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_head", "n_head_kv", "n_ff", "head_dim",
                                       "n_vocab", "n_rep", "n_ctx", "stage", "first", "last", "pos",
                                       "device")] + [("rms_eps", C.c_float), ("rope_base", C.c_float),
                                                     ("device_bytes", C.c_size_t)]


class EcuKprof(C.Structure):
    _fields_ = [("kind", C.c_char * 32), ("launches", C.c_int), ("total_ms", C.c_double),
                ("bytes_per_launch", C.c_double)]


# (name, restype, argtypes) of every symbol include/engine_cuda.h declares
SIGNATURES = [
    ("ecu_model_open", C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t]),
    ("ecu_model_open_file", C.c_int, [C.POINTER(C.c_void_p), C.c_char_p, C.c_char_p, C.c_size_t]),
    ("ecu_model_new", C.c_void_p, []),
    ("ecu_model_set_str", C.c_int, [C.c_void_p, C.c_char_p, C.c_char_p]),
    ("ecu_model_set_u32", C.c_int, [C.c_void_p, C.c_char_p, C.c_ulong]),
    ("ecu_model_set_f32", C.c_int, [C.c_void_p, C.c_char_p, C.c_float]),
    ("ecu_model_add_tensor", C.c_int, [C.c_void_p, C.c_char_p, C.c_uint, C.POINTER(C.c_uint64), C.c_uint,
                                       C.c_void_p, C.c_size_t]),
    ("ecu_model_close", None, [C.c_void_p]),
    ("ecu_model_n_tensors", C.c_size_t, [C.c_void_p]),
    ("ecu_model_tensor", C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint), C.POINTER(C.c_uint),
                                   C.POINTER(C.c_uint64), C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]),
    ("ecu_ctx_bytes", C.c_size_t, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]),
    ("ecu_ctx_open", C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                               C.c_char_p, C.c_size_t]),
    ("ecu_ctx_close", None, [C.c_void_p]),
    ("ecu_ctx_info", C.c_int, [C.c_void_p, C.POINTER(EcuInfo)]),
    ("ecu_ctx_path", C.c_char_p, [C.c_void_p]),
    ("ecu_forward", C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_reset", None, [C.c_void_p]),
    ("ecu_layer_once", C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_step_layers", C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_pick", C.c_int, [C.c_void_p]),
    ("ecu_get_logits", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    ("ecu_set_pos", C.c_int, [C.c_void_p, C.c_int]),
    ("ecu_state_ptr", C.c_void_p, [C.c_void_p]),
    ("ecu_forward_dev", C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_token_ptr", C.c_void_p, [C.c_void_p]),
    ("ecu_step_dev", C.c_int, [C.c_void_p, C.c_void_p]),
    ("ecu_ctx_fork", C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_char_p, C.c_size_t]),
    ("ecu_ctx_open_span", C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_int, C.c_int, C.c_uint, C.c_int,
                                    C.c_int, C.c_char_p, C.c_size_t]),
    ("ecu_link_handle", C.c_int, [C.c_void_p, C.c_char_p]),
    ("ecu_link_next", C.c_int, [C.c_void_p, C.c_char_p]),
    ("ecu_link_next_local", C.c_int, [C.c_void_p, C.c_void_p]),
    ("ecu_link_input", C.c_int, [C.c_void_p]),
    ("ecu_link_feed", C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_ctx_open_tp", C.c_int, [C.POINTER(C.c_void_p), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_char_p, C.c_size_t]),
    ("ecu_tp_handle", C.c_int, [C.c_void_p, C.c_char_p]),
    ("ecu_tp_connect", C.c_int, [C.c_void_p, C.c_char_p]),
    ("ecu_tp_slice", C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    ("ecu_prefill", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    ("ecu_prefill_rows", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("ecu_generate", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    ("ecu_decode_async", C.c_int, [C.c_void_p, C.c_int]),
    ("ecu_sync", C.c_int, [C.c_void_p]),
    ("ecu_stream", C.c_void_p, [C.c_void_p]),
    ("ecu_dequant", C.c_int, [C.c_uint, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p, C.c_int]),
    ("ecu_dequant_tensor", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.c_size_t, C.c_void_p]),
    ("ecu_matvec", C.c_int, [C.c_uint, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int]),
    ("ecu_matvec_argmax_noalloc", C.c_int, [C.c_uint, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                            C.c_void_p, C.c_void_p]),
    ("ecu_set_wait_ns", C.c_int, [C.c_int, C.c_ulonglong]),
    ("ecu_inject_wait_timeout", C.c_int, [C.c_void_p]),
    ("ecu_matvec_bench", C.c_int, [C.c_uint, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_int, C.c_int, C.POINTER(C.c_double)]),
    ("ecu_matvec_stream_bench", C.c_int, [C.c_uint, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    ("ecu_profile_steps", C.c_int, [C.c_void_p, C.c_int, C.POINTER(EcuKprof), C.c_int]),
    ("ecu_profile_cta_ns", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_int), C.c_char_p,
                                     C.c_size_t]),
    ("ecu_last_error", C.c_char_p, []),
    ("ecu_kernel_launches", C.c_uint64, []),
    ("ecu_version", C.c_char_p, []),
]


def lib() -> C.CDLL:
    """Load libdcb200.so (building it first if the sources are newer)."""
    global _LIB
    if _LIB is None:
        if os.environ.get("DCB200_NO_BUILD") != "1":
            from . import build
            build.build()
        if not _LIB_PATH.exists():
            raise EngineError(f"{_LIB_PATH} is missing: run python -m distcomp_b200.build")
        L = C.CDLL(str(_LIB_PATH))
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def last_error() -> str:
    return (lib().ecu_last_error() or b"").decode(errors="replace")


def kernel_launches() -> int:
    return int(lib().ecu_kernel_launches())


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


class GgufModel:
    """Host view of a GGUF image (the buffer must outlive every LlmCtx opened
    from it until the open call returns; weights are copied to the device)."""

    def __init__(self, buf=None, path: str | None = None):
        """buf: a GGUF image in host memory; or path: a GGUF file, mapped
        (ecu_model_open_file: a stage's context pages in its tensors only)."""
        self.h = C.c_void_p()
        err = C.create_string_buffer(512)
        if path is not None:
            self._buf = None
            rc = lib().ecu_model_open_file(C.byref(self.h), str(path).encode(), err, 512)
        else:
            self._buf = np.frombuffer(buf, dtype=np.uint8) if not isinstance(buf, np.ndarray) else buf
            rc = lib().ecu_model_open(C.byref(self.h), _ptr(self._buf), self._buf.nbytes, err, 512)
        if rc != 0:
            raise EngineError(err.value.decode(errors="replace"))

    def tensor(self, name: str):
        t, nd = C.c_uint(), C.c_uint()
        dims = (C.c_uint64 * 4)()
        data, nb = C.c_void_p(), C.c_size_t()
        if lib().ecu_model_tensor(self.h, name.encode(), C.byref(t), C.byref(nd), dims, C.byref(data),
                                  C.byref(nb)) != 0:
            raise KeyError(name)
        return int(t.value), [int(dims[i]) for i in range(nd.value)], int(data.value), int(nb.value)

    def n_tensors(self) -> int:
        return int(lib().ecu_model_n_tensors(self.h))

    def close(self):
        if self.h:
            lib().ecu_model_close(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ctx_bytes(model: GgufModel, stage: int, first: int = 0, last: int = 0, n_ctx: int = 0) -> int:
    return int(lib().ecu_ctx_bytes(model.h, stage, first, last, n_ctx))


class LlmCtx:
    """One engine stage resident on one GPU (llm_ctx, src/engine.h:46-70)."""

    def __init__(self, model: GgufModel | None, stage: int, first: int = 0, last: int = 0, n_ctx: int = 0,
                 device: int = 0, fork_of: "LlmCtx | None" = None, tp: tuple[int, int] | None = None,
                 span: int = 0):
        """tp = (rank, world): a tensor-parallel FULL context (ecu_ctx_open_tp);
        connect the ranks with tp_handle / tp_connect before the first step.
        stage STAGE_SPAN: layers first..last (first > last: none) with the
        embedding / head by span = SPAN_EMBED | SPAN_HEAD (ecu_ctx_open_span)."""
        self.h = C.c_void_p()
        err = C.create_string_buffer(512)
        if fork_of is not None:
            rc = lib().ecu_ctx_fork(C.byref(self.h), fork_of.h, err, 512)
            span = fork_of.span
        elif stage == STAGE_SPAN:
            rc = lib().ecu_ctx_open_span(C.byref(self.h), model.h, first, last, span, n_ctx, device, err, 512)
        elif tp is not None:
            rc = lib().ecu_ctx_open_tp(C.byref(self.h), model.h, n_ctx, device, int(tp[0]), int(tp[1]), err, 512)
        else:
            rc = lib().ecu_ctx_open(C.byref(self.h), model.h, stage, first, last, n_ctx, device, err, 512)
        if rc != 0:
            raise EngineError(err.value.decode(errors="replace") or last_error())
        i = EcuInfo()
        lib().ecu_ctx_info(self.h, C.byref(i))
        self.info = i
        self.n_embd, self.n_vocab, self.n_ctx = i.n_embd, i.n_vocab, i.n_ctx
        self.stage = i.stage
        self.span = span if i.stage == STAGE_SPAN else 0
        self.has_head = i.stage in (STAGE_HEAD, STAGE_FULL) or bool(self.span & SPAN_HEAD)
        self.device = i.device
        sl = (C.c_int * 4)()
        lib().ecu_tp_slice(self.h, sl)
        self.tp_rank, self.tp_world, self.vocab0, self.vocab1 = (int(v) for v in sl)

    # --- reference API ---------------------------------------------------
    def forward(self, token: int, out: np.ndarray) -> int:
        assert out.dtype == np.float32 and out.flags.c_contiguous
        return int(lib().ecu_forward(self.h, int(token), _ptr(out)))

    def reset(self) -> None:
        lib().ecu_reset(self.h)

    def layer_once(self, idx: int, out: np.ndarray) -> int:
        return int(lib().ecu_layer_once(self.h, int(idx), _ptr(out)))

    def step_layers(self, n: int, out: np.ndarray) -> int:
        return int(lib().ecu_step_layers(self.h, int(n), _ptr(out)))

    def pick(self) -> int:
        return int(lib().ecu_pick(self.h))

    # --- extras ----------------------------------------------------------
    def logits(self) -> np.ndarray:
        """The last step's logits (a tensor-parallel rank: rows vocab0..vocab1)."""
        n = self.vocab1 - self.vocab0
        out = np.empty(n, dtype=np.float32)
        if lib().ecu_get_logits(self.h, _ptr(out), n) != 0:
            raise EngineError(last_error())
        return out

    # --- pipeline links ---------------------------------------------------
    def link_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        if lib().ecu_link_handle(self.h, buf) != 0:
            raise EngineError(last_error())
        return buf.raw

    def link_next(self, nxt: "LlmCtx | bytes") -> None:
        """Send this stage's output to the next stage: a context of this
        process, or another process's link_handle()."""
        if isinstance(nxt, LlmCtx):
            rc = lib().ecu_link_next_local(self.h, nxt.h)
        else:
            rc = lib().ecu_link_next(self.h, bytes(nxt))
        if rc != 0:
            raise EngineError(last_error())

    def link_input(self) -> None:
        if lib().ecu_link_input(self.h) != 0:
            raise EngineError(last_error())

    def link_feed(self, token: int, stream: int | None = None) -> None:
        if lib().ecu_link_feed(self.h, int(token), C.c_void_p(stream) if stream else None) != 0:
            raise EngineError(last_error())

    def cta_times(self):
        """One persistent step with every CTA's phase start/end times:
        (phase names, int64 array [phases + 1, grid] of ns)."""
        buf = np.zeros(4096 * 1024, dtype=np.uint64)
        kinds = C.create_string_buffer(65536)
        grid = C.c_int(0)
        n = lib().ecu_profile_cta_ns(self.h, _ptr(buf), buf.size, C.byref(grid), kinds, 65536)
        if n < 0:
            raise EngineError(last_error())
        names = kinds.value.decode().split(",")
        g = grid.value
        return names, buf[: (n + 1) * g].reshape(n + 1, g).astype(np.int64)

    def tp_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        if lib().ecu_tp_handle(self.h, buf) != 0:
            raise EngineError(last_error())
        return buf.raw

    def tp_connect(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        if lib().ecu_tp_connect(self.h, blob) != 0:
            raise EngineError(last_error())

    def set_pos(self, pos: int) -> None:
        if lib().ecu_set_pos(self.h, int(pos)) != 0:
            raise EngineError("bad position")

    @property
    def pos(self) -> int:
        i = EcuInfo()
        lib().ecu_ctx_info(self.h, C.byref(i))
        return int(i.pos)

    def generate(self, prompt, n_gen: int) -> list[int]:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_gen, 1), dtype=np.int32)
        if lib().ecu_generate(self.h, _ptr(p), len(p), int(n_gen), _ptr(out)) != 0:
            raise EngineError(last_error())
        return [int(t) for t in out[:n_gen]]

    def prefill(self, tokens, out: np.ndarray | None = None) -> int:
        """The prompt at once (ecu_prefill); returns the picked next token."""
        p = np.ascontiguousarray(tokens, dtype=np.int32)
        if out is None:
            out = np.zeros(self.n_embd + 1, dtype=np.float32)
        assert out.dtype == np.float32 and out.size >= self.n_embd + 1
        if lib().ecu_prefill(self.h, _ptr(p), len(p), _ptr(out)) != 0:
            raise EngineError(last_error())
        return int(out[self.n_embd])

    def prefill_rows(self, x_ptr: int, n: int, tokens=None, out: np.ndarray | None = None) -> int | None:
        """One pipeline stage's batched prompt over n device rows at x_ptr
        (ecu_prefill_rows); a stage with the head returns the picked token."""
        tk = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        if out is None and self.has_head:
            out = np.zeros(self.n_embd + 1, dtype=np.float32)
        rc = lib().ecu_prefill_rows(self.h, None if tk is None else _ptr(tk), int(n), C.c_void_p(int(x_ptr)),
                                    None if out is None else _ptr(out))
        if rc != 0:
            raise EngineError(last_error())
        return int(out[self.n_embd]) if self.has_head else None

    def decode_async(self, n: int) -> None:
        if lib().ecu_decode_async(self.h, int(n)) != 0:
            raise EngineError(last_error())

    def sync(self) -> None:
        if lib().ecu_sync(self.h) != 0:
            raise EngineError(last_error())

    def forward_dev(self, token: int, stream: int | None = None) -> None:
        if lib().ecu_forward_dev(self.h, int(token), C.c_void_p(stream or 0)) != 0:
            raise EngineError(last_error())

    def fork(self) -> "LlmCtx":
        """A context of the same stage sharing this one's weights, with its
        own KV cache and stream (one per concurrent sequence)."""
        return LlmCtx(None, self.stage, fork_of=self)

    def token_ptr(self) -> int:
        return int(lib().ecu_token_ptr(self.h) or 0)

    def step_dev(self, stream: int | None = None) -> None:
        """One step from device-resident input (ecu_step_dev)."""
        if lib().ecu_step_dev(self.h, C.c_void_p(stream or 0)) != 0:
            raise EngineError(last_error())

    def inject_wait_timeout(self) -> None:
        """The next persistent step waits for an input word no phase writes
        (ecu_inject_wait_timeout): failure-path testing."""
        if lib().ecu_inject_wait_timeout(self.h) != 0:
            raise EngineError(last_error())

    def path(self) -> str:
        """"persistent" or "kernels: <why not>" (ecu_ctx_path)."""
        return (lib().ecu_ctx_path(self.h) or b"").decode()

    def state_ptr(self) -> int:
        return int(lib().ecu_state_ptr(self.h) or 0)

    def stream(self) -> int:
        return int(lib().ecu_stream(self.h) or 0)

    def profile_steps(self, n_steps: int) -> dict:
        """{kind: (launches, total_ms, bytes_per_launch)} over n_steps eager
        decode steps with CUDA events around every kernel."""
        arr = (EcuKprof * 128)()
        k = lib().ecu_profile_steps(self.h, int(n_steps), arr, 128)
        if k < 0:
            raise EngineError(last_error())
        return {arr[i].kind.decode(): (arr[i].launches, arr[i].total_ms, arr[i].bytes_per_launch)
                for i in range(k)}

    def dequant_tensor(self, name: str, off: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        if lib().ecu_dequant_tensor(self.h, name.encode(), off, n, _ptr(out)) != 0:
            raise EngineError(last_error())
        return out

    def close(self) -> None:
        if self.h:
            lib().ecu_ctx_close(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequant(gtype: int, raw: np.ndarray, total: int, off: int, n: int, device: int = 0) -> tuple[int, np.ndarray]:
    """gguf_dequant on the GPU: (rc, values)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(max(n, 1), dtype=np.float32)
    rc = lib().ecu_dequant(gtype, _ptr(raw), total, off, n, _ptr(out), device)
    return int(rc), out[:n]


def matvec(gtype: int, raw: np.ndarray, n_in: int, n_out: int, x: np.ndarray, device: int = 0) -> np.ndarray:
    """y = W x for a raw GGUF weight (uploads per call)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n_out, dtype=np.float32)
    if lib().ecu_matvec(gtype, _ptr(raw), n_in, n_out, _ptr(x), _ptr(y), device) != 0:
        raise EngineError(last_error())
    return y


def matvec_bench(gtype: int, raw: np.ndarray, n_in: int, n_out: int, x: np.ndarray, copies: int, rounds: int,
                 device: int = 0):
    """Device time per launch (ms) of y = W x over `copies` rotated device
    copies of the matrix, and the last launch's y (ecu_matvec_bench)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n_out, dtype=np.float32)
    ms = C.c_double(0.0)
    if lib().ecu_matvec_bench(gtype, _ptr(raw), n_in, n_out, _ptr(x), _ptr(y), device, copies, rounds,
                              C.byref(ms)) != 0:
        raise EngineError(last_error())
    return ms.value, y


def set_wait_ns(ns: int, device: int = 0) -> None:
    """The limit after which every bounded wait in the kernels gives up."""
    if lib().ecu_set_wait_ns(device, int(ns)) != 0:
        raise EngineError(last_error())


def matvec_stream_bench(gtype: int, raw: np.ndarray, n_in: int, n_out: int, x: np.ndarray, copies: int,
                        rounds: int, device: int = 0):
    """Device time per matvec (ms) with the copies streamed through the
    persistent step's GEMV phases, and the last phase's y
    (ecu_matvec_stream_bench)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n_out, dtype=np.float32)
    ms = C.c_double(0.0)
    if lib().ecu_matvec_stream_bench(gtype, _ptr(raw), n_in, n_out, _ptr(x), _ptr(y), device, copies, rounds,
                                     C.byref(ms)) != 0:
        raise EngineError(last_error())
    return ms.value, y
