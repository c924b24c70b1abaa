#!/usr/bin/env python3
"""Golden outputs of the reference engine on the 8B-shaped Q4_0 model.

    python tests/golden/make_golden_8b.py [--threads N]

The model is the seeded Llama-3-8B shape (synth.spec("llama3-8b"), seed 0:
dim 4096, 32 layers, 32/8 heads, FFN 14336, vocab 128256, Q4_0 layers,
Q8_0 embedding and head) built on the host from numpy's seeded normals
(synth.build_model(device="cpu"), the same bytes with any thread count;
the GPU test rebuilds it and checks its sha256).  The engine is the
reference itself, oracle/_ref/libdcref.so (src/engine.c, src/gguf.c,
src/thread.c compiled from their sources by oracle/Makefile), run as
src/shard.c's local three-stage loop (EMBED, LAYERS 0..31, HEAD), one token
at a time.  Written to tests/golden/llama3_8b_q4_0.npz:

  model_sha256        sha256 of the GGUF image
  prompt              the 512 prompt tokens (synth.prompt_tokens(512, vocab, 0))
  greedy16            64 greedy tokens after the prompt's first 16 tokens
  layer_states        token prompt[0] at position 0: the state after EMBED
                      and after each layer (llm_layer_once), [33][4096]
  top_idx0, top_val0  the 256 largest logits of that first step (HEAD),
  logits0_absmax      and the largest |logit|
  greedy512           16 greedy tokens after the whole 512-token prompt
  top_idx512, top_val512  the 256 largest logits of the last prompt step

Takes about 20 minutes on 8 host cores (the reference streams the 4.5 GB
of weights at 2-4 GB/s per token).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

from distcomp_b200 import synth  # noqa: E402

KEY = "llama3-8b"
N_PROMPT, N_SHORT, N_GEN_SHORT, N_GEN_LONG, TOPK = 512, 16, 64, 16, 256


def topk(v: np.ndarray, k: int):
    idx = np.argsort(-v.astype(np.float64), kind="stable")[:k]
    return idx.astype(np.int32), v[idx].astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    import oracle
    if not oracle.available("ref"):
        raise SystemExit("oracle/_ref/libdcref.so is not built (make -C oracle ref with DC_REFERENCE set)")
    lib = oracle.get("ref")
    lib.set_threads(min(64, args.threads))

    s = synth.spec(KEY)
    t0 = time.time()
    buf = synth.build_model(s, seed=0, threads=args.threads)
    sha = hashlib.sha256(buf.view(np.uint8)).hexdigest()
    print(f"model built in {time.time() - t0:.0f} s, {buf.size} bytes, sha256 {sha}", flush=True)
    prompt = synth.prompt_tokens(N_PROMPT, s.n_vocab, seed=0)

    m = lib.model(buf)
    emb, lay, head = m.ctx(0), m.ctx(1, 0, s.n_layer - 1, 0), m.ctx(2)
    st = np.zeros(s.n_embd + 8, dtype=np.float32)
    res = {"model_sha256": np.frombuffer(sha.encode(), dtype=np.uint8), "prompt": np.array(prompt, np.int32)}

    # per-layer states of the first prompt token at position 0
    assert emb.forward(prompt[0], st) == 0
    states = [st[:s.n_embd].copy()]
    for li in range(s.n_layer):
        assert lay.layer_once(li, st) == 0
        states.append(st[:s.n_embd].copy())
    res["layer_states"] = np.stack(states)
    lay.reset()

    def step(t, with_head=True):
        assert emb.forward(t, st) == 0 and lay.forward(t, st) == 0
        if with_head:
            assert head.forward(t, st) == 0
            return int(st[s.n_embd])
        return None

    # short prompt, 64 greedy tokens
    t0 = time.time()
    tok = None
    for i, t in enumerate(prompt[:N_SHORT]):
        tok = step(t)
        if i == 0:
            lg = head.logits(s.n_vocab)
            res["top_idx0"], res["top_val0"] = topk(lg, TOPK)
            res["logits0_absmax"] = np.array([np.max(np.abs(lg))], np.float32)
    gen = []
    while len(gen) < N_GEN_SHORT:
        gen.append(tok)
        if len(gen) < N_GEN_SHORT:
            tok = step(tok)
    res["greedy16"] = np.array(gen, np.int32)
    print(f"greedy after {N_SHORT} tokens ({time.time() - t0:.0f} s): {gen}", flush=True)

    # the whole prompt (the HEAD stage only for its last token), 16 tokens
    lay.reset()
    t0 = time.time()
    for i, t in enumerate(prompt):
        tok = step(t, with_head=i + 1 == len(prompt))
        if (i + 1) % 64 == 0:
            print(f"  prompt {i + 1}/{len(prompt)} ({time.time() - t0:.0f} s)", flush=True)
    lg = head.logits(s.n_vocab)
    res["top_idx512"], res["top_val512"] = topk(lg, TOPK)
    gen = []
    while len(gen) < N_GEN_LONG:
        gen.append(tok)
        if len(gen) < N_GEN_LONG:
            tok = step(tok)
    res["greedy512"] = np.array(gen, np.int32)
    print(f"greedy after {N_PROMPT} tokens ({time.time() - t0:.0f} s): {gen}", flush=True)
    np.savez_compressed(OUT / "llama3_8b_q4_0.npz", **res)
    print("written", OUT / "llama3_8b_q4_0.npz")


if __name__ == "__main__":
    main()
