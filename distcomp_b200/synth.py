"""Seeded synthetic llama-shaped GGUF models and prompts.

Weights are N(0, 0.02) per tensor (the generator is seeded by the model seed
and the CRC-32 of the tensor name, so any subset of tensors can be rebuilt
independently), quantised to the requested GGUF block type; norm weights
are 1.0 in F32.  Tensors whose input length is not a whole number of blocks
are stored as F32 (the tiny shape's 688-wide ffn_down cannot be Q8_0: the
reference matvec would return zeros for it, src/engine.c:317-320).

Two generation paths with the same quantisation rule:
  * ``device="cpu"``: numpy PCG64 normals, quantised by gguf-py (the
    reference's scripts use the same package); stable across machines, used
    for the fixtures and CPU-checkable models.
  * ``device="cuda"``: torch normals on the GPU and the torch restatement of
    the same Q4_0/Q8_0 rule in ``quantize_torch``; used for the 4.6 GB
    8B-shaped model, which would take minutes on the host.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass, replace

import numpy as np

from . import gguf as G


@dataclass(frozen=True)
class LlamaSpec:
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    n_ff: int
    n_vocab: int
    n_ctx: int
    rope_base: float = 10000.0
    eps: float = 1e-5
    wtype: int = G.Q8_0          # attention / FFN weights
    emb_type: int = G.Q8_0       # token_embd
    out_type: int = G.Q8_0       # output
    arch: str = "llama"
    tied: bool = False           # no output.weight: the head reuses token_embd
    qkv_bias: bool = False       # qwen2-style attention biases
    head_dim: int | None = None  # writes rope.dimension_count when set
    sigma: float = 0.02


SPECS = {
    # single-node CPU shape: dim 256, 4 layers, 8 heads, FFN 688, vocab 4096
    "tiny": LlamaSpec(4, 256, 8, 8, 688, 4096, 256, 10000.0),
    # Llama-3-8B shape, Q4_0 layers, Q8_0 embedding and head
    "llama3-8b": LlamaSpec(32, 4096, 32, 8, 14336, 128256, 4096, 500000.0, wtype=G.Q4_0),
    # Llama-2-70B shape (Q4_K layers)
    "llama2-70b": LlamaSpec(80, 8192, 64, 8, 28672, 32000, 8448, 10000.0, wtype=G.Q4_K),
    # small shapes that still exercise the fast Q4_0/Q8_0 GEMV path (n_in % 1024 == 0)
    "mini-q4": LlamaSpec(2, 1024, 8, 2, 2048, 2048, 128, 500000.0, wtype=G.Q4_0),
    "mini-q8": LlamaSpec(2, 1024, 16, 4, 3072, 1536, 96, 10000.0, wtype=G.Q8_0),
    # Q4_K layers on the fast path; "wide-q4k" has an FFN wider than one
    # column segment (ffn_down kept as two segments of 10240 inputs)
    "mini-q4k": LlamaSpec(2, 1024, 8, 2, 2048, 2048, 128, 500000.0, wtype=G.Q4_K),
    "wide-q4k": LlamaSpec(2, 1024, 8, 1, 20480, 2048, 96, 10000.0, wtype=G.Q4_K),
    # one layer of the 70B shape (n_embd 8192, 64/8 heads, ffn 28672), small vocab
    "l70-1": LlamaSpec(1, 8192, 64, 8, 28672, 2048, 64, 10000.0, wtype=G.Q4_K),
}


def spec(name: str, **over) -> LlamaSpec:
    return replace(SPECS[name], **over)


def tensor_list(s: LlamaSpec):
    """[(name, dims, ggml type)] in file order; dims are ggml's [n_in, n_out]."""
    hd = s.head_dim or s.n_embd // s.n_head
    qd, kvd = s.n_head * hd, s.n_head_kv * hd

    def wt(n_in, t):
        if t in (G.F32, G.F16):
            return t
        return t if n_in % G.BLOCK[t][0] == 0 else G.F32

    out = [("token_embd.weight", (s.n_embd, s.n_vocab), wt(s.n_embd, s.emb_type))]
    for i in range(s.n_layer):
        p = f"blk.{i}."
        out += [
            (p + "attn_norm.weight", (s.n_embd,), G.F32),
            (p + "attn_q.weight", (s.n_embd, qd), wt(s.n_embd, s.wtype)),
            (p + "attn_k.weight", (s.n_embd, kvd), wt(s.n_embd, s.wtype)),
            (p + "attn_v.weight", (s.n_embd, kvd), wt(s.n_embd, s.wtype)),
            (p + "attn_output.weight", (qd, s.n_embd), wt(qd, s.wtype)),
            (p + "ffn_norm.weight", (s.n_embd,), G.F32),
            (p + "ffn_gate.weight", (s.n_embd, s.n_ff), wt(s.n_embd, s.wtype)),
            (p + "ffn_up.weight", (s.n_embd, s.n_ff), wt(s.n_embd, s.wtype)),
            (p + "ffn_down.weight", (s.n_ff, s.n_embd), wt(s.n_ff, s.wtype)),
        ]
        if s.qkv_bias:
            out += [(p + "attn_q.bias", (qd,), G.F32), (p + "attn_k.bias", (kvd,), G.F32),
                    (p + "attn_v.bias", (kvd,), G.F32)]
    out.append(("output_norm.weight", (s.n_embd,), G.F32))
    if not s.tied:
        out.append(("output.weight", (s.n_embd, s.n_vocab), wt(s.n_embd, s.out_type)))
    return out


def name_seed(seed: int, name: str) -> list[int]:
    return [int(seed), zlib.crc32(name.encode()) & 0xFFFFFFFF]


# ------------------------------------------------------------ quantisation --

def quantize_numpy(w: np.ndarray, gtype: int) -> np.ndarray:
    """float32 [.., n_in] -> GGUF block bytes (gguf-py, the ggml rule)."""
    if gtype == G.F32:
        return np.ascontiguousarray(w, dtype=np.float32).view(np.uint8).reshape(-1)
    if gtype == G.F16:
        return np.ascontiguousarray(w, dtype=np.float16).view(np.uint8).reshape(-1)
    from gguf import quants, GGMLQuantizationType as QT
    qt = {G.Q4_0: QT.Q4_0, G.Q8_0: QT.Q8_0, G.Q4_1: QT.Q4_1, G.Q5_0: QT.Q5_0, G.Q5_1: QT.Q5_1}[gtype]
    return np.ascontiguousarray(quants.quantize(w.astype(np.float32), qt)).view(np.uint8).reshape(-1)


def quantize_torch(w, gtype: int):
    """Torch restatement of the same rule (runs on CUDA).  Returns uint8.

    Q4_0 (ggml quantize_row_q4_0_ref, as gguf-py states it): per 32-block,
    m = the element of largest magnitude (first one on ties), d = m / -8,
    id = 1/d (0 when d == 0), q = min(15, trunc(x*id + 8.5)); bytes =
    fp16(d), then q[i] | q[i+16] << 4 for i < 16.
    Q8_0: d = max|x| / 127, id = 1/d (0 when d == 0), q = round-half-away(x*id)
    as int8; bytes = fp16(d), q[0..31].
    Every step is a single fp32 operation (and the first maximum is picked
    explicitly), so the result is bit-identical to gguf-py's numpy code on
    the CPU and on the GPU (checked in tests/test_synth.py)."""
    import torch
    x = w.reshape(-1, 32).to(torch.float32)
    nblk = x.shape[0]
    if gtype == G.Q4_0:
        # the first element of largest magnitude, spelled out: torch.argmax
        # on CUDA does not promise the first index on ties (x and -x both at
        # the block maximum happen in about one block in 30,000 of N(0,1)
        # draws), and the sign of m decides the whole block
        ax = x.abs()
        amax = ax.amax(dim=1, keepdim=True)
        pos = torch.arange(32, device=x.device, dtype=torch.int64).expand_as(ax)
        idx = torch.where(ax == amax, pos, torch.full_like(pos, 32)).amin(dim=1, keepdim=True)
        m = torch.gather(x, 1, idx)
        d = m / torch.full_like(m, -8.0)
        inv = torch.where(d == 0, torch.zeros_like(d), torch.ones_like(d) / d)
        q = torch.trunc(x * inv + 8.5).clamp(0, 15).to(torch.uint8)
        packed = q[:, :16] | (q[:, 16:] << 4)
        dh = d.to(torch.float16).view(torch.uint8).reshape(nblk, 2)
        return torch.cat([dh, packed], dim=1).reshape(-1)
    if gtype == G.Q8_0:
        # a tensor divisor: torch's CUDA kernel for tensor / python-scalar
        # multiplies by the scalar's reciprocal, which is not 1/127 exactly
        amax = x.abs().amax(dim=1, keepdim=True)
        d = amax / torch.full_like(amax, 127.0)
        inv = torch.where(d == 0, torch.zeros_like(d), torch.ones_like(d) / d)
        v = x * inv
        a = v.abs()
        fl = a.floor()
        r = (fl + (2.0 * (a - fl)).floor()) * v.sign()
        q = r.to(torch.int8).view(torch.uint8)
        dh = d.to(torch.float16).view(torch.uint8).reshape(nblk, 2)
        return torch.cat([dh, q], dim=1).reshape(-1)
    raise ValueError(f"quantize_torch: type {gtype} not supported")


def quantize_q4_k_torch(w):
    """float32 weights (a multiple of 256) -> Q4_K super-blocks, 144 bytes
    per 256 weights, as torch uint8 on w's device.

    A plain min/max rule (any byte pattern is a valid block; this one makes
    the dequantised weights follow w): per 32-weight sub-block j, lo = min(0,
    min x), scale_j = (max x - lo) / 15, min_j = -lo; per super-block d =
    fp16(max scale_j / 63), dmin = fp16(max min_j / 63), 6-bit sc_j =
    round(scale_j / d), m_j = round(min_j / dmin); codes q = round((x +
    dmin*m_j) / (d*sc_j)) clamped to 0..15.  Bytes: d, dmin, the 12 packed
    scale bytes (sc/m of sub-blocks 0-3 in the low 6 bits of bytes 0-3 / 4-7,
    the low nibbles of sub-blocks 4-7 in bytes 8-11, their high 2 bits in the
    top bits of bytes 0-7), then chunk c's 32 code bytes with sub-block 2c in
    the low nibbles and 2c+1 in the high ones -- the layout src/gguf.c:558-590
    decodes."""
    import torch
    x = w.reshape(-1, 8, 32).to(torch.float32)
    nb = x.shape[0]
    lo = torch.clamp(x.amin(dim=2), max=0.0)
    sc_f = (x.amax(dim=2) - lo) / 15.0
    mn_f = -lo
    d = (sc_f.amax(dim=1) / 63.0).to(torch.float16)
    dm = (mn_f.amax(dim=1) / 63.0).to(torch.float16)
    df, dmf = d.float()[:, None], dm.float()[:, None]
    inv_d = torch.where(df > 0, 1.0 / df, torch.zeros_like(df))
    inv_dm = torch.where(dmf > 0, 1.0 / dmf, torch.zeros_like(dmf))
    sc = torch.clamp(torch.round(sc_f * inv_d), 0, 63).to(torch.int32)
    mn = torch.clamp(torch.round(mn_f * inv_dm), 0, 63).to(torch.int32)
    dl = (df * sc.float())[..., None]
    ml = (dmf * mn.float())[..., None]
    inv_dl = torch.where(dl > 0, 1.0 / dl, torch.zeros_like(dl))
    q = torch.clamp(torch.round((x + ml) * inv_dl), 0, 15).to(torch.uint8).reshape(nb, 4, 2, 32)
    qs = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    sb = torch.empty((nb, 12), dtype=torch.int32, device=x.device)
    sb[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    sb[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    sb[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    head = torch.cat([d.view(torch.uint8).reshape(nb, 2), dm.view(torch.uint8).reshape(nb, 2),
                      sb.to(torch.uint8)], dim=1)
    return torch.cat([head, qs], dim=1).reshape(-1)


def microbench_blocks(rng: np.random.Generator, gtype: int, n_in: int, n_out: int) -> np.ndarray:
    """The quantised-matvec microbenchmark's weights (Q4_0 or Q8_0): codes
    uniform over the format's range, fp16 scales |N(0, 0.02)| / max_code
    (max_code 8 and 127)."""
    nblk = n_in * n_out // 32
    if gtype == G.Q4_0:
        blk = np.empty((nblk, 18), dtype=np.uint8)
        d = (np.abs(rng.standard_normal(nblk)) * 0.02 / 8).astype(np.float16)
        blk[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
        blk[:, 2:] = rng.integers(0, 256, size=(nblk, 16), dtype=np.uint8)
    elif gtype == G.Q8_0:
        blk = np.empty((nblk, 34), dtype=np.uint8)
        d = (np.abs(rng.standard_normal(nblk)) * 0.02 / 127).astype(np.float16)
        blk[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
        blk[:, 2:] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    else:
        raise ValueError(f"microbench_blocks: type {gtype}")
    return blk.reshape(-1)


def random_kquant_blocks(rng: np.random.Generator, gtype: int, nblk: int, sigma: float = 0.02):
    """Random K-quant blocks: uniform code/scale bytes, fp16 super-block scales
    drawn as |N(0, sigma)| / 64 so that weights land around sigma.  (gguf-py
    cannot quantise K-quants; any bytes are valid blocks.)"""
    be, bb = G.BLOCK[gtype]
    raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    scale = (np.abs(rng.standard_normal((nblk, 2))) * sigma / 64).astype(np.float16)
    if gtype in (G.Q4_K, G.Q5_K):
        raw[:, 0:4] = scale.view(np.uint8)
    elif gtype == G.Q2_K:
        raw[:, 80:84] = scale.view(np.uint8)
    elif gtype == G.Q3_K:
        raw[:, 108:110] = scale[:, :1].view(np.uint8)
    elif gtype == G.Q6_K:
        raw[:, 208:210] = scale[:, :1].view(np.uint8)
    elif gtype == G.Q8_K:
        # the reference's Q8_K reads 32 fp16 scales at bytes 256..319 of a
        # 292-byte block (src/gguf.c:650-659), i.e. 28 of them overlap the
        # next block; only the first 18 lie inside the block
        s = (np.abs(rng.standard_normal((nblk, 18))) * sigma / 64).astype(np.float16)
        raw[:, 256:292] = s.view(np.uint8).reshape(nblk, 36)
    return raw.reshape(-1)


# --------------------------------------------------------------- builders --

def _meta(b: G.GGUFBuilder, s: LlamaSpec):
    a = s.arch
    b.add_kv("general.architecture", G.T_STR, a)
    b.add_kv("general.alignment", G.T_U32, G.ALIGN)
    b.add_kv(f"{a}.block_count", G.T_U32, s.n_layer)
    b.add_kv(f"{a}.context_length", G.T_U32, s.n_ctx)
    b.add_kv(f"{a}.embedding_length", G.T_U32, s.n_embd)
    b.add_kv(f"{a}.feed_forward_length", G.T_U32, s.n_ff)
    b.add_kv(f"{a}.attention.head_count", G.T_U32, s.n_head)
    b.add_kv(f"{a}.attention.head_count_kv", G.T_U32, s.n_head_kv)
    b.add_kv(f"{a}.attention.layer_norm_rms_epsilon", G.T_F32, s.eps)
    b.add_kv(f"{a}.rope.freq_base", G.T_F32, s.rope_base)
    if s.head_dim:
        b.add_kv(f"{a}.rope.dimension_count", G.T_U32, s.head_dim)
    b.add_kv(f"{a}.vocab_size", G.T_U32, s.n_vocab)


def stage_tensors(s: LlamaSpec, first: int, last: int, embed: bool, head: bool) -> set[str]:
    """Names of the tensors a pipeline stage opens: layers first..last, plus
    the embedding and/or the head (output norm and matrix)."""
    names = set()
    for name, _dims, _gt in tensor_list(s):
        if name.startswith("blk."):
            if first <= int(name.split(".")[1]) <= last:
                names.add(name)
        elif name == "token_embd.weight":
            if embed or (head and s.tied):
                names.add(name)
        elif head:
            names.add(name)
    return names


def build_model(s: LlamaSpec, seed: int = 0, device: str = "cpu", threads: int = 1,
                quant_device: str | None = None, only: set[str] | None = None) -> np.ndarray:
    """The whole GGUF image as a numpy uint8 array.

    only: the image holds just these tensors (the same bytes as in the whole
    model: every tensor's generator is seeded by its name), with the whole
    model's metadata -- a pipeline rank builds its stage's part alone.

    device="cpu": numpy normals (the same bytes whatever ``threads`` and
    ``quant_device`` are: with threads > 1 the tensors are generated in
    parallel and quantised by ``quantize_torch``, bit-identical to gguf-py's
    rule, on ``quant_device`` (default the CPU)).  device="cuda:N": torch's
    CUDA generator (a different stream of normals)."""
    b = G.GGUFBuilder()
    _meta(b, s)
    tl = [t for t in tensor_list(s) if only is None or t[0] in only]
    for name, dims, gt in tl:
        b.add_tensor(name, dims, gt)
    b.finalize()
    if device != "cpu":
        import torch
        dev = torch.device(device)

    def cpu_tensor(name, dims, gt):
        view = b.tensor_view(name)
        n = int(np.prod(dims))
        rng = np.random.default_rng(name_seed(seed, name))
        w = (rng.standard_normal(n, dtype=np.float32) * np.float32(s.sigma)).reshape(dims[::-1])
        if gt == G.Q4_K or ((threads > 1 or quant_device) and gt in (G.Q4_0, G.Q8_0)):
            import torch
            t = torch.from_numpy(w.reshape(-1))
            if quant_device:
                t = t.to(quant_device)
            qb = quantize_q4_k_torch(t) if gt == G.Q4_K else quantize_torch(t, gt)
            view[:] = qb.cpu().numpy()
        else:
            view[:] = quantize_numpy(w, gt)

    jobs = []
    for name, dims, gt in tl:
        view = b.tensor_view(name)
        n = int(np.prod(dims))
        if name.endswith("norm.weight"):
            view[:] = np.ones(n, dtype=np.float32).view(np.uint8)
            continue
        if gt in (G.Q2_K, G.Q3_K, G.Q5_K, G.Q6_K, G.Q8_K):
            rng = np.random.default_rng(name_seed(seed, name))
            view[:] = random_kquant_blocks(rng, gt, n // G.BLOCK[gt][0], s.sigma)
            continue
        if device == "cpu":
            if threads > 1:
                jobs.append((name, dims, gt))
            else:
                cpu_tensor(name, dims, gt)
        else:
            import torch
            gen = torch.Generator(device=dev)
            ns = name_seed(seed, name)
            gen.manual_seed(ns[0] * 1_000_003 + ns[1])
            w = torch.randn(n, generator=gen, device=dev, dtype=torch.float32) * s.sigma
            if gt == G.F32:
                qb = w.view(torch.uint8)
            elif gt == G.F16:
                qb = w.to(torch.float16).view(torch.uint8)
            elif gt == G.Q4_K:
                qb = quantize_q4_k_torch(w)
            else:
                qb = quantize_torch(w, gt)
            torch.from_numpy(view).copy_(qb.cpu())
            del w, qb
    if jobs:
        from concurrent.futures import ThreadPoolExecutor
        # largest tensors first, so that the embedding and head overlap the rest
        jobs.sort(key=lambda j: -int(np.prod(j[1])))
        with ThreadPoolExecutor(threads) as ex:
            for f in [ex.submit(cpu_tensor, *j) for j in jobs]:
                f.result()
    return b.buf


def prompt_tokens(n: int, n_vocab: int, seed: int = 0) -> list[int]:
    """Uniform token ids in [3, n_vocab)."""
    rng = np.random.default_rng([int(seed), 0x70726F6D])
    return [int(t) for t in rng.integers(3, n_vocab, size=n)]
