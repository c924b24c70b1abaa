#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ (run in a container where
the reference tree is mounted; the GPU box never runs this).

    python tests/golden/make_golden.py --ref PATH_TO_REFERENCE_CHECKOUT

(or set DC_REFERENCE to that path)

Sources, all of them the reference's own code or tests:
  * kquant_blocks.json   the fixed Q2_K/Q3_K/Q4_K/Q6_K blocks and the 64
                         expected weights per block that tests/quant_test.c
                         carries (parsed as text, values unchanged)
  * llama_ref_tiny.gguf  the F32 model written by scripts/llama_ref.py, and
    llama_ref_tiny.json  its numpy forward (logits, argmax) for the
                         script's default prompt, plus the reference C
                         engine's logits for token 1 and its greedy stream
                         (what tests/engine_test.c prints)
  * dequant_blocks.npz   random blocks of every format gguf_dequant
                         supports, with the reference C decoder's output
  * tiny_q8.npz          the seeded tiny llama (dim 256, Q8_0, F32
                         ffn_down) run by the reference C engine: greedy
                         tokens for a 16-token prompt, first-step logits,
                         per-layer states for the first token
  * mini_q4.npz          the same for a small Q4_0 model with GQA
The reference C engine is oracle/_ref/libdcref.so, built by oracle/Makefile
from the reference sources in place.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

from distcomp_b200 import gguf as G  # noqa: E402
from distcomp_b200 import synth  # noqa: E402


def parse_quant_test(path: Path) -> dict:
    """Byte and float arrays of tests/quant_test.c."""
    src = path.read_text()
    out = {}
    for m in re.finditer(r"static const unsigned char blk_(\w+)\[2\]\[(\d+)\] = \{(.*?)\};", src, re.S):
        name, size, body = m.group(1), int(m.group(2)), m.group(3)
        rows = re.findall(r"\{([^{}]*)\}", body)
        out.setdefault(name, {})["blocks"] = [[int(v, 16) for v in re.findall(r"0x[0-9A-Fa-f]+", r)] for r in rows]
        assert all(len(r) == size for r in out[name]["blocks"])
    for m in re.finditer(r"static const float exp_(\w+)\[2\]\[64\] = \{(.*?)\};", src, re.S):
        name, body = m.group(1), m.group(2)
        rows = re.findall(r"\{([^{}]*)\}", body)
        out[name]["expect"] = [[float(v.rstrip("f")) for v in re.findall(r"-?[0-9.]+(?:e-?[0-9]+)?f", r)] for r in rows]
        assert all(len(r) == 64 for r in out[name]["expect"])
    types = {"Q2_K": G.Q2_K, "Q3_K": G.Q3_K, "Q4_K": G.Q4_K, "Q6_K": G.Q6_K}
    for k in out:
        out[k]["type"] = types[k]
    return out


def sha(buf) -> str:
    return hashlib.sha256(np.ascontiguousarray(buf).view(np.uint8)).hexdigest()


def ref_lib():
    import oracle
    oracle.build(ref=True)
    return oracle.get("ref")


def run_engine(lib, buf, prompt, n_gen, layers_dump=True):
    """Three-stage run like tests/engine_test.c + per-layer states of the
    first prompt token like tests/engine_stages.c."""
    meta = G.read_tensor_table(buf)["__meta__"]
    a = meta["general.architecture"]
    n_layer, n_embd = int(meta[a + ".block_count"]), int(meta[a + ".embedding_length"])
    n_vocab = int(meta.get(a + ".vocab_size", 0)) or None
    m = lib.model(buf)
    emb, lay, head = m.ctx(0), m.ctx(1, 0, n_layer - 1, 0), m.ctx(2)
    st = np.zeros(n_embd + 8, dtype=np.float32)
    res = {}
    if layers_dump:
        assert emb.forward(prompt[0], st) == 0
        states = [st[:n_embd].copy()]
        for li in range(n_layer):
            assert lay.layer_once(li, st) == 0
            states.append(st[:n_embd].copy())
        res["layer_states"] = np.stack(states)
        lay.reset()
    gen, first_logits = [], None
    tok = None
    for i, t in enumerate(prompt):
        assert emb.forward(t, st) == 0 and lay.forward(t, st) == 0 and head.forward(t, st) == 0
        tok = int(st[n_embd])
        if i == 0:
            res["logits_tok0"] = head.logits(n_vocab or lib_vocab(buf))
    res["logits_last_prompt"] = head.logits(n_vocab or lib_vocab(buf))
    while len(gen) < n_gen:
        gen.append(tok)
        if len(gen) == n_gen:
            break
        assert emb.forward(tok, st) == 0 and lay.forward(tok, st) == 0 and head.forward(tok, st) == 0
        tok = int(st[n_embd])
    res["greedy"] = np.array(gen, dtype=np.int32)
    res["prompt"] = np.array(prompt, dtype=np.int32)
    return res


def lib_vocab(buf):
    t = G.read_tensor_table(buf)
    return int(t["token_embd.weight"][1][1])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DC_REFERENCE"),
                    help="the reference checkout (default: $DC_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set DC_REFERENCE")
    ref = Path(args.ref)

    # 1. quant_test.c vectors
    kq = parse_quant_test(ref / "tests" / "quant_test.c")
    (OUT / "kquant_blocks.json").write_text(json.dumps(kq, indent=0))
    print("kquant_blocks.json:", {k: len(v["blocks"]) for k, v in kq.items()})

    lib = ref_lib()

    # 2. llama_ref.py tiny F32 model
    with tempfile.TemporaryDirectory() as td:
        gpath, jpath = Path(td) / "m.gguf", Path(td) / "m.json"
        subprocess.run([sys.executable, str(ref / "scripts" / "llama_ref.py"), str(gpath), "--json", str(jpath)],
                       check=True, stdout=subprocess.DEVNULL)
        data = json.loads(jpath.read_text())
        gbytes = gpath.read_bytes()
    (OUT / "llama_ref_tiny.gguf").write_bytes(gbytes)
    buf = np.frombuffer(gbytes, dtype=np.uint8).copy()
    r = run_engine(lib, buf, [1], 4, layers_dump=False)
    data["c_engine_token1_logits8"] = [float(v) for v in r["logits_tok0"][:8]]
    data["c_engine_greedy_from_token1"] = [int(v) for v in r["greedy"]]
    data["sha256"] = sha(buf)
    (OUT / "llama_ref_tiny.json").write_text(json.dumps(data, indent=1))
    print("llama_ref_tiny:", data["c_engine_greedy_from_token1"], "numpy greedy", data["greedy"])

    # 3. random blocks of every supported format through gguf_dequant
    rng = np.random.default_rng(1234)
    arrs = {}
    for gt in (G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q8_0, G.Q2_K, G.Q3_K, G.Q4_K, G.Q5_K, G.Q6_K, G.Q8_K):
        be, bb = G.BLOCK[gt]
        nblk = 24
        raw = rng.integers(0, 256, size=nblk * bb, dtype=np.uint8)
        # fp16 scales: mostly normal finite values, plus subnormals, zeros, inf and NaN
        sc_off = {G.Q4_0: [0], G.Q4_1: [0, 2], G.Q5_0: [0], G.Q5_1: [0, 2], G.Q8_0: [0], G.Q2_K: [80, 82],
                  G.Q3_K: [108], G.Q4_K: [0, 2], G.Q5_K: [0, 2], G.Q6_K: [208], G.Q8_K: []}[gt]
        specials = [0x0000, 0x8000, 0x0001, 0x03FF, 0x8200, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00]
        for b in range(nblk):
            for o in sc_off:
                if b < len(specials):
                    h = specials[b]
                else:
                    h = int(np.float16(rng.standard_normal() * 0.05).view(np.uint16))
                raw[b * bb + o] = h & 0xFF
                raw[b * bb + o + 1] = h >> 8
        total = nblk * be
        n = total - (be if gt == G.Q8_K else 0)   # Q8_K reads past its last block
        rc, vals = lib.dequant(gt, raw, total, 0, n)
        assert rc == 0
        arrs[f"raw_{gt}"] = raw
        arrs[f"out_{gt}"] = vals
        arrs[f"n_{gt}"] = np.array([total, n])
    # F16 / F32 element streams
    h = rng.integers(0, 65536, size=4096, dtype=np.uint16)
    h[:16] = [0, 0x8000, 1, 0x3FF, 0x400, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x7D01, 0x8001, 0x83FF, 0x3C00, 0xC000, 0x3555, 0x0200]
    rc, vals = lib.dequant(G.F16, h.view(np.uint8), 4096, 0, 4096)
    arrs[f"raw_{G.F16}"], arrs[f"out_{G.F16}"], arrs[f"n_{G.F16}"] = h.view(np.uint8), vals, np.array([4096, 4096])
    np.savez_compressed(OUT / "dequant_blocks.npz", **arrs)
    print("dequant_blocks.npz written")

    # 4/5. seeded llama models through the reference engine
    for key, name, n_prompt, n_gen in (("tiny", "tiny_q8", 16, 128), ("mini-q4", "mini_q4", 8, 32),
                                       ("mini-q8", "mini_q8", 8, 24)):
        s = synth.spec(key)
        buf = synth.build_model(s, seed=0)
        prompt = synth.prompt_tokens(n_prompt, s.n_vocab, seed=0)
        r = run_engine(lib, buf, prompt, n_gen)
        r["model_sha256"] = np.frombuffer(sha(buf).encode(), dtype=np.uint8)
        np.savez_compressed(OUT / f"{name}.npz", **r)
        print(f"{name}: greedy[:12] {list(r['greedy'][:12])}")


if __name__ == "__main__":
    main()
