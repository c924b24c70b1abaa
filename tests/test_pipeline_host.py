"""Host-side logic of the layer pipeline, on the CPU.

* split_stages restates src/shard.c:384-413 (the LAYERS part of
  split_stages); the cases below follow that loop by hand.
* split_by_bytes is checked against brute force on small inputs.
* The tick schedule is checked for the properties the ranks rely on, and
  then run for real: ranks as gloo processes (world size 2 and 3) and as one
  process with a loopback exchanger, each stage a stand-in whose "layers"
  are cheap deterministic functions, compared with the same functions
  applied in plain order (the answer a single node gives).
"""
import itertools
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from distcomp_b200 import pipeline as P


# ------------------------------------------------------------------ split --

def test_split_stages_reference_rule():
    assert P.split_stages(32, 1) == [(0, 31)]
    assert P.split_stages(32, 2) == [(0, 15), (16, 31)]
    assert P.split_stages(32, 8) == [(4 * i, 4 * i + 3) for i in range(8)]
    # ceil(32/3) = 11, then ceil(21/2) = 11, then 10
    assert P.split_stages(32, 3) == [(0, 10), (11, 21), (22, 31)]
    # 80 layers on 8: 10 each; 5 layers on 8 stages: one each, three idle
    assert P.split_stages(80, 8) == [(10 * i, 10 * i + 9) for i in range(8)]
    assert P.split_stages(5, 8) == [(i, i) for i in range(5)]


def test_split_stages_capacity():
    cost = lambda a, b: (b - a + 1) * 10          # 10 bytes a layer
    # stage 0 holds 2 layers, stage 1 holds 10: 2 + 8 -> the rest fits
    assert P.split_stages(10, 2, cost, [25, 100]) == [(0, 1), (2, 9)]
    with pytest.raises(ValueError):
        P.split_stages(10, 2, cost, [5, 100])      # no layer fits stage 0
    with pytest.raises(ValueError):
        P.split_stages(10, 2, cost, [25, 30])      # layers left over


def _brute(layer_bytes, k, head, emb, head_alone=False):
    n = len(layer_bytes)
    best = None
    splits = list(itertools.combinations(range(1, n), k - 1))
    if head_alone and head > 0:                # the head's stage may hold no layer
        splits += [c + (n,) for c in itertools.combinations(range(1, n), k - 2)]
    for cuts in splits:
        b = (0,) + cuts + (n,)
        c = []
        for i in range(k):
            x = sum(layer_bytes[b[i]:b[i + 1]])
            x += emb if i == 0 else 0
            x += head if i == k - 1 else 0
            c.append(x)
        if best is None or max(c) < best:
            best = max(c)
    return best


def _cost(plan, layer_bytes, head, emb):
    c = []
    for i, (a, b) in enumerate(plan):
        x = sum(layer_bytes[a:b + 1]) + (emb if i == 0 else 0) + (head if i == len(plan) - 1 else 0)
        c.append(x)
    return max(c)


@pytest.mark.parametrize("seed", range(6))
def test_split_by_bytes_optimal(seed):
    g = torch.Generator().manual_seed(seed)
    n = 9
    lb = [int(x) for x in torch.randint(1, 50, (n,), generator=g)]
    head = int(torch.randint(0, 120, (1,), generator=g))
    for k in range(2, 6):
        plan = P.split_by_bytes(lb, k, head_bytes=head, embed_bytes=3)
        assert len(plan) == k and plan[0][0] == 0 and plan[-1][1] == n - 1
        assert all(a <= b for a, b in plan)
        assert all(plan[i][1] + 1 == plan[i + 1][0] for i in range(k - 1))
        assert _cost(plan, lb, head, 3) == _brute(lb, k, head, 3)


@pytest.mark.parametrize("seed", range(6))
def test_split_by_bytes_head_alone_optimal(seed):
    g = torch.Generator().manual_seed(100 + seed)
    n = 9
    lb = [int(x) for x in torch.randint(1, 50, (n,), generator=g)]
    head = int(torch.randint(1, 150, (1,), generator=g))
    for k in range(2, 6):
        plan = P.split_by_bytes(lb, k, head_bytes=head, embed_bytes=3, head_alone=True)
        assert len(plan) == k and plan[0][0] == 0 and plan[-1][1] == n - 1
        assert all(a <= b for a, b in plan[:-1]) and plan[-1][0] <= plan[-1][1] + 1
        assert all(plan[i][1] + 1 == plan[i + 1][0] for i in range(k - 1))
        assert _cost(plan, lb, head, 3) == _brute(lb, k, head, 3, head_alone=True)
        assert _cost(plan, lb, head, 3) <= _brute(lb, k, head, 3)


def test_split_by_bytes_8b_shape():
    # 32 equal layers of 122.7 MB, 558 MB head: the head counts as ~4.5 layers
    lb = [122_683_392] * 32
    head = 558_170_112 + 16_384
    plan = P.split_by_bytes(lb, 8, head_bytes=head, embed_bytes=4352)
    sizes = [b - a + 1 for a, b in plan]
    assert sum(sizes) == 32 and sizes[-1] < sizes[0]
    assert P.split_by_bytes(lb, 2, head_bytes=558_170_112)[0] == (0, 17)
    # the head alone on the 8th GPU: no stage above 5 layers' bytes
    alone = P.split_by_bytes(lb, 8, head_bytes=head, embed_bytes=4352, head_alone=True)
    assert alone[-1] == (32, 31)
    assert _cost(alone, lb, head, 4352) == 5 * lb[0] < _cost(plan, lb, head, 4352)
    # where it does not pay, the split is the same as without the option
    assert P.split_by_bytes(lb, 2, head_bytes=head, head_alone=True) == P.split_by_bytes(lb, 2, head_bytes=head)
    assert P.split_by_bytes(lb, 4, head_bytes=head, head_alone=True)[-1][0] <= 31


# --------------------------------------------------------------- schedule --

@pytest.mark.parametrize("n_ranks,n_seq,n_steps,n_prompt", [(2, 1, 5, 2), (2, 8, 4, 3), (3, 2, 6, 1),
                                                            (4, 4, 3, 0), (8, 8, 3, 2), (8, 3, 4, 4)])
def test_schedule_properties(n_ranks, n_seq, n_steps, n_prompt):
    S = P.Schedule(n_ranks, n_seq, n_steps, n_prompt=n_prompt)
    when = {}
    for t in range(S.n_ticks + 5):
        for r in range(n_ranks):
            w = S.work(r, t)
            if w is not None:
                assert (r, w) not in when
                when[(r, w)] = t
    # every rank does every (sequence, step) exactly once, all inside n_ticks
    assert len(when) == n_ranks * n_seq * n_steps
    assert max(when.values()) == S.n_ticks - 1
    for s in range(n_seq):
        for k in range(n_steps):
            for r in range(1, n_ranks):
                # a stage works on (s, k) the tick after the stage before it
                assert when[(r, (s, k))] == when[(r - 1, (s, k))] + 1
            if k + 1 < n_steps:
                # the token of step k+1 exists (last stage, step k) before
                # the first stage needs it
                assert when[(n_ranks - 1, (s, k))] < when[(0, (s, k + 1))]
    # messages: state hops for every (s, k); tokens only for argmax-fed steps
    n_state = n_token = 0
    for t in range(S.n_ticks):
        for m in S.messages(t):
            assert S.work(m.src, t) is not None and S.work(m.src, t)[0] == m.seq
            if m.kind == "state":
                assert m.dst == m.src + 1
                n_state += 1
            else:
                assert (m.src, m.dst) == (n_ranks - 1, 0)
                n_token += 1
    assert n_state == (n_ranks - 1) * n_seq * n_steps
    assert n_token == n_seq * max(0, n_steps - max(n_prompt, 1))


# ------------------------------------------------------- stand-in stages --

D, V = 8, 1000


def f_embed(tok):
    i = torch.arange(D, dtype=torch.float64)
    return torch.sin(tok * 0.37 + i)


def f_layer(l, x, pos):
    return torch.tanh(x * (1.0 + 0.01 * l) + 0.05 * l + 0.001 * pos)


def f_head(x):
    return int(abs(float(x.sum())) * 1e4) % V


class FakeStage:
    """Stand-in with the buffers and calls of GpuStage."""

    def __init__(self, rank, n_ranks, first, last, n_layer, n_seq, prompts):
        self.first, self.last = first, last
        self.has_embed, self.has_head = first == 0, last == n_layer - 1
        self.tok_in = [torch.zeros(1, dtype=torch.int32) for _ in range(n_seq)]
        self.tok_out = [torch.zeros(1, dtype=torch.int32) for _ in range(n_seq)]
        self.x_in = [torch.zeros(D, dtype=torch.float64) for _ in range(n_seq)]
        self.x_out = [torch.zeros(D, dtype=torch.float64) for _ in range(n_seq)]
        self.pos = [0] * n_seq
        self.prompts = prompts
        self.history = [[] for _ in range(n_seq)]

    def send_buf(self, s, kind):
        return self.tok_out[s] if kind == "token" else self.x_out[s]

    def recv_buf(self, s, kind):
        return self.tok_in[s] if kind == "token" else self.x_in[s]

    def set_token(self, s, k):
        self.tok_in[s][0] = self.prompts[s][k]

    def run(self, s, k):
        assert self.pos[s] == k                  # steps of a sequence in order
        x = f_embed(int(self.tok_in[s][0])) if self.has_embed else self.x_in[s].clone()
        for l in range(self.first, self.last + 1):
            x = f_layer(l, x, self.pos[s])
        self.pos[s] += 1
        if self.has_head:
            t = f_head(x)
            self.tok_out[s][0] = t
            self.history[s].append(t)
        else:
            self.x_out[s].copy_(x)


def reference_tokens(prompts, n_layer, n_steps):
    out = []
    for p in prompts:
        toks, tok = [], p[0]
        for k in range(n_steps):
            x = f_embed(tok)
            for l in range(n_layer):
                x = f_layer(l, x, k)
            t = f_head(x)
            toks.append(t)
            tok = p[k + 1] if k + 1 < len(p) else t
        out.append(toks)
    return out


def _prompts(n_seq, n_prompt):
    return [[(7 * s + 13 * k + 3) % V for k in range(n_prompt)] for s in range(n_seq)]


def test_loopback_matches_plain_order():
    n_layer, n_steps, n_prompt = 7, 9, 3
    for n_ranks, n_seq in [(2, 1), (2, 3), (3, 3), (4, 2), (5, 8)]:
        prompts = _prompts(n_seq, n_prompt)
        plan = P.split_stages(n_layer, n_ranks)
        stages = {r: FakeStage(r, n_ranks, a, b, n_layer, n_seq, prompts) for r, (a, b) in enumerate(plan)}
        S = P.Schedule(n_ranks, n_seq, n_steps, n_prompt=n_prompt)
        P.run_ticks(S, stages, P.LoopbackExchanger())
        assert stages[n_ranks - 1].history == reference_tokens(prompts, n_layer, n_steps)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, n_layer, n_seq, n_steps, n_prompt, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = _prompts(n_seq, n_prompt)
        a, b = P.split_stages(n_layer, world)[rank]
        st = FakeStage(rank, world, a, b, n_layer, n_seq, prompts)
        S = P.Schedule(world, n_seq, n_steps, n_prompt=n_prompt)
        # two halves, as bench.py runs warm-up and timed ticks separately
        mid = S.n_ticks // 2
        P.run_ticks(S, {rank: st}, P.DistExchanger(rank), t0=0, t1=mid)
        dist.barrier()
        P.run_ticks(S, {rank: st}, P.DistExchanger(rank), t0=mid)
        if rank == world - 1:
            torch.save(st.history, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_seq", [(2, 1), (2, 4), (3, 5)])
def test_gloo_pipeline_matches_plain_order(tmp_path, world, n_seq):
    n_layer, n_steps, n_prompt = 6, 7, 2
    out = str(tmp_path / "hist.pt")
    mp.start_processes(_gloo_rank, args=(world, _free_port(), n_layer, n_seq, n_steps, n_prompt, out),
                       nprocs=world, join=True, start_method="spawn")
    hist = torch.load(out)
    assert hist == reference_tokens(_prompts(n_seq, n_prompt), n_layer, n_steps)


def test_split_half_layers():
    """Ranges of layer halves: contiguous, every half placed once, optimal
    against brute force on the units, and the 8B shape on 8 GPUs no slower
    than whole layers (one layer's halves may sit on two GPUs)."""
    from distcomp_b200 import engine as E
    n, A, F, H, Em = 5, 3.0, 5.0, 7.0, 1.0
    for k in range(2, 5):
        plan = P.split_half_layers(A, F, n, k, H, Em)
        assert len(plan) == k
        units = []
        for a, b, fl in plan:
            if a > b:
                continue
            u0 = 2 * a + (1 if fl & E.SPAN_FFN_FIRST else 0)
            u1 = 2 * b + (0 if fl & E.SPAN_ATTN_LAST else 1)
            units.append((u0, u1))
        assert units[0][0] == 0 and units[-1][1] == 2 * n - 1
        assert all(units[i][1] + 1 == units[i + 1][0] for i in range(len(units) - 1))
        costs = [int(A * 1000), int(F * 1000)] * n
        got = _cost([(u0, u1) for u0, u1 in units] + ([(2 * n, 2 * n - 1)] if plan[-1][0] > plan[-1][1] else []),
                    costs, int(H * 1000), int(Em * 1000))
        assert got == _brute(costs, k, int(H * 1000), int(Em * 1000), head_alone=True)
    half = P.split_half_layers(22.4, 29.9, 32, 8, 98.0, 5.0)
    t = lambda p: (0 if p[0] > p[1] else
                   sum(22.4 * (not (i == p[0] and p[2] & E.SPAN_FFN_FIRST)) +
                       29.9 * (not (i == p[1] and p[2] & E.SPAN_ATTN_LAST)) for i in range(p[0], p[1] + 1)))
    worst = max(t(p) + (98.0 if i == 7 else 0) + (5.0 if i == 0 else 0) for i, p in enumerate(half))
    assert worst < 5 * (22.4 + 29.9)
    assert P.stage_text((4, 8, E.SPAN_FFN_FIRST)) == "4:ffn-8" and P.stage_text((32, 31, 0)) == "head"
