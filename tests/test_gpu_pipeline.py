"""The layer pipeline on real kernels.

On one GPU, the stages of a 2-, 3- and 4-way split run as separate stage
runtimes in one process (their messages are device copies between the
stages' streams); the interleaved sequences must produce exactly the
greedy tokens and final logits of a FULL context fed the same prompt: a
stage boundary moves the state between buffers but changes no arithmetic.
With two or more GPUs, the same check runs as torchrun ranks over NCCL.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from distcomp_b200 import pipeline as P
from distcomp_b200 import synth

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def full_greedy(eng, m, prompt, n_gen, n_ctx):
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    toks = c.generate(prompt, n_gen)
    logits = c.logits()
    c.close()
    return toks, logits


def full_prefill_greedy(eng, m, s, prompt, n_gen, n_ctx):
    """A FULL context: the prompt as one batch (ecu_prefill), then greedy
    steps; the tokens and the last step's logits."""
    c = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    toks = [c.prefill(prompt)]
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    while len(toks) < n_gen:
        assert c.forward(toks[-1], out) == 0
        toks.append(int(out[s.n_embd]))
    logits = c.logits()
    c.close()
    return toks, logits


@pytest.mark.parametrize("n_ranks,n_seq,head_alone", [(2, 1, False), (2, 3, False), (3, 2, False),
                                                       (4, 4, False), (3, 3, True)])
def test_loopback_pipeline_matches_full_context(eng, model_buf, n_ranks, n_seq, head_alone):
    """head_alone: the last stage holds the output head and no layer."""
    key, over = "mini-q4", {"n_layer": 4}
    s = synth.spec(key, **over)
    buf = model_buf(key, **over)
    m = eng.GgufModel(buf)
    n_prompt, n_gen, n_ctx = 5, 12, 64
    prompts = [synth.prompt_tokens(n_prompt, s.n_vocab, seed=11 + q) for q in range(n_seq)]
    plan = P.split_stages(s.n_layer, n_ranks)
    if head_alone:
        plan = P.split_stages(s.n_layer, n_ranks - 1) + [(s.n_layer, s.n_layer - 1)]
    stages = {r: P.GpuStage(m, r, n_ranks, a, b, s.n_layer, n_seq, n_ctx, 0, prompts=prompts)
              for r, (a, b) in enumerate(plan)}
    n_steps = n_prompt + n_gen - 1
    stages[n_ranks - 1].record_tokens(n_steps)
    S = P.Schedule(n_ranks, n_seq, n_steps, n_prompt=n_prompt)
    P.run_ticks(S, stages, P.LoopbackExchanger())
    for st in stages.values():
        st.sync()
    hist = stages[n_ranks - 1].history.cpu().numpy()
    last = stages[n_ranks - 1]
    for q in range(n_seq):
        want, want_logits = full_greedy(eng, m, prompts[q], n_gen, n_ctx)
        got = [int(t) for t in hist[q, n_prompt - 1:]]
        assert got == want, (q, got, want)
        got_logits = last.chains[q][-1].logits()
        assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
    for st in stages.values():
        st.close()


def test_step_dev_rejects_bad_device_token(eng, model_buf):
    """A token outside the vocabulary that arrives in device memory (not
    through the host checks) is reported by ecu_sync instead of read."""
    buf = model_buf("mini-q4")
    m = eng.GgufModel(buf)
    c = eng.LlmCtx(m, eng.STAGE_EMBED, n_ctx=16)
    tok = P.device_view(c.token_ptr(), 1, "<i4", 0)
    tok.fill_(10 ** 6)
    torch.cuda.synchronize()
    c.step_dev()
    with pytest.raises(eng.EngineError, match="vocabulary"):
        c.sync()
    tok.fill_(7)
    torch.cuda.synchronize()
    c.step_dev()
    c.sync()
    c.close()


def test_fork_shares_weights_and_keeps_own_cache(eng, model_buf):
    s = synth.spec("mini-q4")
    m = eng.GgufModel(model_buf("mini-q4"))
    a = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=32)
    b = a.fork()
    assert b.info.device_bytes < a.info.device_bytes / 2
    pa, pb = synth.prompt_tokens(4, s.n_vocab, seed=1), synth.prompt_tokens(4, s.n_vocab, seed=2)
    ta = a.generate(pa, 6)
    tb = b.generate(pb, 6)
    a.close()                       # the fork keeps the shared weights alive
    assert b.generate(pa, 6) != [] and b.pos == 18
    ref = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=32)
    assert ref.generate(pb, 6) == tb
    ref.reset()
    assert ref.generate(pa, 6) == ta
    b.close()
    ref.close()


@pytest.mark.parametrize("n_ranks,n_seq,layout", [(2, 1, "ref"), (2, 3, "ref"), (3, 4, "ref"),
                                                   (3, 2, "head_alone"), (3, 3, "half")])
def test_linked_loopback_pipeline(eng, model_buf, n_ranks, n_seq, layout):
    """Linked stages (each step writes its output into the next stage's
    tagged words, the last stage's head its token into the first stage's) on
    one GPU, all stages on one stream in tick order: the prompts through the
    stages as batches (prefill_local), then greedy steps with no exchange
    between ticks -- the FULL context's tokens and final logits bit for bit,
    and again after a reset."""
    key, over = "mini-q4", {"n_layer": 4}
    s = synth.spec(key, **over)
    m = eng.GgufModel(model_buf(key, **over))
    n_prompt, n_gen, n_ctx = 6, 10, 64
    prompts = [synth.prompt_tokens(n_prompt, s.n_vocab, seed=41 + q) for q in range(n_seq)]
    plan = [(a, b, 0) for a, b in P.split_stages(s.n_layer, n_ranks)]
    if layout == "head_alone":
        plan = [(a, b, 0) for a, b in P.split_stages(s.n_layer, n_ranks - 1)] + [(s.n_layer, s.n_layer - 1, 0)]
    if layout == "half":                       # layers 1 and 2 each cut between two GPUs
        plan = [(0, 1, eng.SPAN_ATTN_LAST), (1, 2, eng.SPAN_FFN_FIRST | eng.SPAN_ATTN_LAST),
                (2, 3, eng.SPAN_FFN_FIRST)]
    stream = torch.cuda.Stream()
    stages = {r: P.GpuStage(m, r, n_ranks, a, b, s.n_layer, n_seq, n_ctx, 0, prompts=prompts, stream=stream,
                            halves=h)
              for r, (a, b, h) in enumerate(plan)}
    P.link_local(stages)
    last = stages[n_ranks - 1]
    wants = [full_prefill_greedy(eng, m, s, prompts[q], n_gen, n_ctx) for q in range(n_seq)]
    for _run in range(2):
        firsts = [P.prefill_local(stages, q, prompts[q]) for q in range(n_seq)]
        n_steps = n_gen - 1
        last.record_tokens(n_prompt + n_steps)
        S = P.Schedule(n_ranks, n_seq, n_steps, n_prompt=0, first_step=n_prompt)
        P.run_ticks(S, stages, P.LinkedExchanger())
        for st in stages.values():
            st.sync()
        hist = last.history.cpu().numpy()
        for q in range(n_seq):
            want, want_logits = wants[q]
            got = [firsts[q]] + [int(t) for t in hist[q, n_prompt: n_prompt + n_steps]]
            assert got == want, (q, got, want)
            got_logits = last.chains[q][-1].logits()
            assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
        for st in stages.values():
            st.reset()
    for st in stages.values():
        st.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_pipeline_two_gpus(tmp_path):
    """bench.py's pipeline path at a small size over two real ranks: NCCL
    hops with the prompts through the ticks, then linked steps after the
    prompts as batches."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29531", str(ROOT / "tests" / "pipeline_ranks.py"),
           str(tmp_path)]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert (tmp_path / "ok").exists()
    assert (tmp_path / "ok_linked").exists(), r.stdout[-2000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_pipeline_two_gpus_70b_shape(tmp_path):
    """Two 70B-shape layers, one per GPU, each rank building only its stage's
    tensors: the prompt as a batch per stage, then linked greedy steps; the
    tokens the oracle's and a FULL context's, the logits bit for bit."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", str(ROOT / "tests" / "pipeline_ranks_70b.py"),
           str(tmp_path)]
    r = subprocess.run(["timeout", "-k", "30", "900"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert (tmp_path / "ok").exists(), r.stdout[-2000:]


def test_prefill_through_stages_matches_full_context(eng, oracle_port, model_buf):
    """Two layers of the 70B shape (n_embd 8192, 64/8 heads, FFN 28672,
    Q4_K) as two pipeline stages in one process -- EMBED + layer 0 | layer
    1 + HEAD -- the prompt as one batch per stage (ecu_prefill_rows), then
    greedy decode through the tick schedule: tokens and final logits bit for
    bit a FULL context's (ecu_prefill + per-token decode), and the oracle's
    greedy tokens."""
    import oracle
    key, over = "l70-1", {"n_layer": 2}
    s = synth.spec(key, **over)
    buf = model_buf(key, **over)
    m = eng.GgufModel(buf)
    n_prompt, n_gen, n_ctx = 8, 4, s.n_ctx
    prompt = synth.prompt_tokens(n_prompt, s.n_vocab, seed=21)
    full = eng.LlmCtx(m, eng.STAGE_FULL, n_ctx=n_ctx)
    want = [full.prefill(prompt)]
    out = np.zeros(s.n_embd + 1, dtype=np.float32)
    while len(want) < n_gen:
        assert full.forward(want[-1], out) == 0
        want.append(int(out[s.n_embd]))
    want_logits = full.logits()
    full.close()
    assert want == oracle.greedy(oracle_port, buf, prompt, n_gen)

    # two stages, then three with the head alone on the last
    for plan in ([(0, 0), (1, 1)], [(0, 0), (1, 1), (2, 1)]):
        k = len(plan)
        stages = {r: P.GpuStage(m, r, k, a, b, s.n_layer, 1, n_ctx, 0) for r, (a, b) in enumerate(plan)}
        tok = P.prefill_local(stages, 0, prompt)
        assert tok == want[0]
        stages[k - 1].record_tokens(n_prompt + n_gen)
        S = P.Schedule(k, 1, n_gen - 1, n_prompt=n_prompt, first_step=n_prompt)
        P.run_ticks(S, stages, P.LoopbackExchanger())
        for st in stages.values():
            st.sync()
        hist = stages[k - 1].history.cpu().numpy()[0]
        got = [tok] + [int(t) for t in hist[n_prompt: n_prompt + n_gen - 1]]
        assert got == want, plan
        got_logits = stages[k - 1].chains[0][-1].logits()
        assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
        for st in stages.values():
            st.close()
