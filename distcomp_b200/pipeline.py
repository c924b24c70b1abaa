"""Layer-pipelined decode over the GPUs of one node.

The reference splits a model over nodes by contiguous layer ranges
(split_stages, src/shard.c:358-437): an EMBED node, LAYERS nodes with
ceil(remaining layers / remaining nodes) layers each, a HEAD node, with the
fp32 state forwarded node to node over UDP and the argmax token sent back
to the entry node (src/shard.c:865-966).  Here every GPU is one stage: the
embedding folds into the first GPU and the head into the last (the
reference's separate EMBED/HEAD nodes are a memory policy,
src/shard.c:369-370, that 180 GB per GPU does not need), and the hops are
NCCL send/recv over NVLink of the n_embd fp32 state (16 KB for dim 4096)
and of the 4-byte token.

Several independent sequences can be interleaved to keep every stage busy:
each stage keeps one KV cache per sequence (ecu_ctx_fork shares the
weights).  All ranks follow one tick schedule: in tick t, rank r works on
sequence (t - r) mod P, P = max(n_seq, n_ranks), then every rank exchanges
the messages the schedule names for that tick as one NCCL group.  The
schedule is pure host arithmetic, identical on every rank, so sends and
receives always pair up and no rank waits for a message nobody sends.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


# ----------------------------------------------------------------- layout --

def split_stages(n_layer: int, n_nodes: int, cost=None, cap=None) -> list[tuple[int, int]]:
    """Contiguous layer ranges for n_nodes LAYERS stages, by the rule of
    src/shard.c:384-413: each stage takes ceil(remaining layers / remaining
    stages), at most what leaves one layer for every later stage, shrunk
    while cost(first, last) exceeds that stage's cap[k].  Raises ValueError
    where the reference returns its errors (a stage that holds no layer,
    layers left over)."""
    if n_nodes < 1:
        raise ValueError("need at least one stage")
    out, l = [], 0
    for k in range(n_nodes):
        if l >= n_layer:
            break
        rem_layers, rem_nodes = n_layer - l, n_nodes - k
        give = -(-rem_layers // rem_nodes)
        give = min(give, rem_layers - (rem_nodes - 1))
        give = max(give, 1)
        if cost is not None and cap is not None:
            while give >= 1 and cost(l, l + give - 1) > cap[k]:
                give -= 1
            if give < 1:
                raise ValueError(f"stage {k} cannot hold layer {l}")
        out.append((l, l + give - 1))
        l += give
    if l < n_layer:
        raise ValueError(f"{l} of {n_layer} layers placed: add devices")
    return out


# The output head's share of a stage's time per byte, relative to a layer's:
# one persistent step streams the head (one GEMV phase, ~5.7 TB/s on B200)
# about 2.4 times faster per byte than a layer (five phases and their
# boundaries, ~2.4 TB/s), measured on the 8B shape (head 98 us for 558 MB,
# layer 51.8 us for 123 MB).  The benches balance stages by time: head bytes
# x HEAD_COST against layer bytes.
HEAD_COST = 0.42


def split_by_bytes(layer_bytes: list[int], n_stages: int, head_bytes: int = 0,
                   embed_bytes: int = 0, head_alone: bool = False) -> list[tuple[int, int]]:
    """Contiguous layer ranges for n_stages GPUs that minimise the largest
    per-token byte stream of a stage, when the first stage also reads the
    embedding row and the last the output head.  Every stage gets at least
    one layer, except that with head_alone the last stage may hold the head
    only (an empty range (n, n - 1)): where the head weighs about as much as
    a stage's share of the layers (the 8B shape on 8 GPUs: 558 MB against
    5 x 123 MB), one more layer on the head's GPU would set the pace.  (The
    reference's rule balances layer counts; with the head folded into the
    last GPU, balancing bytes keeps that GPU from setting the pipeline's
    pace.)"""
    n = len(layer_bytes)
    if not 1 <= n_stages <= n:
        raise ValueError(f"{n_stages} stages for {n} layers")
    pre = [0]
    for b in layer_bytes:
        pre.append(pre[-1] + b)

    def stage_cost(k, a, b):            # layers a..b-1 on stage k
        c = pre[b] - pre[a]
        if k == 0:
            c += embed_bytes
        if k == n_stages - 1:
            c += head_bytes
        return c

    empty_last = head_alone and head_bytes > 0 and n_stages > 1

    def feasible(limit):
        cuts, a = [], 0
        for k in range(n_stages):
            # stages after this one, one layer each at least (the head's
            # stage none when it may stand alone)
            left = n_stages - k - 1 - (1 if empty_last and k < n_stages - 1 else 0)
            if k == n_stages - 1:
                b = n
                if (b <= a and not empty_last) or stage_cost(k, a, b) > limit:
                    return None
            else:
                b = a + 1
                if b > n or stage_cost(k, a, b) > limit:
                    return None
                while b + 1 <= n - left and stage_cost(k, a, b + 1) <= limit:
                    b += 1
            cuts.append((a, b - 1))
            a = b
        return cuts if a == n else None

    lo = max(max(layer_bytes), head_bytes)
    hi = pre[n] + head_bytes + embed_bytes
    best = feasible(hi)
    while lo < hi:                        # smallest feasible limit (integer bytes)
        mid = (lo + hi) // 2
        f = feasible(mid)
        if f is not None:
            best, hi = f, mid
        else:
            lo = mid + 1
    f = feasible(lo)
    return f if f is not None else best


def stage_text(p) -> str:
    """A stage's range for the bench line: layers a-b, 'a:ffn' / 'b:attn' for
    a layer the stage holds half of, 'head' for the head alone."""
    from . import engine as E
    a, b, flags = p
    if a > b:
        return "head"
    lo = f"{a}:ffn" if flags & E.SPAN_FFN_FIRST else str(a)
    hi = f"{b}:attn" if flags & E.SPAN_ATTN_LAST else str(b)
    return f"{lo}-{hi}"


def split_half_layers(attn_cost: float, ffn_cost: float, n_layer: int, n_stages: int, head_cost: float = 0,
                      embed_cost: float = 0, scale: float = 1000.0) -> list[tuple[int, int, int]]:
    """Contiguous ranges of layer halves (each layer = its attention half,
    then its FFN half) for n_stages GPUs, minimising the largest per-token
    cost of a stage (split_by_bytes over the halves, the head alone allowed
    on the last GPU).  Returns (first, last, flags) per stage: layers
    first..last, flags SPAN_FFN_FIRST when layer `first` contributes its FFN
    half only and SPAN_ATTN_LAST when layer `last` contributes its attention
    half only (first > last: no layer).  A layer whose attention half ends one
    GPU's range and whose FFN half starts the next one's is cut between
    them; the residual stream is the only state that crosses."""
    from . import engine as E
    units = []
    for _ in range(n_layer):
        units += [int(round(attn_cost * scale)), int(round(ffn_cost * scale))]
    plan = split_by_bytes(units, n_stages, head_bytes=int(round(head_cost * scale)),
                          embed_bytes=int(round(embed_cost * scale)), head_alone=True)
    out = []
    for u0, u1 in plan:
        if u0 > u1:                                   # the head alone
            out.append((n_layer, n_layer - 1, 0))
            continue
        flags = (E.SPAN_FFN_FIRST if u0 % 2 else 0) | (E.SPAN_ATTN_LAST if u1 % 2 == 0 else 0)
        out.append((u0 // 2, u1 // 2, flags))
    return out


# Per-token time of a layer's attention half (Q/K/V, attention, O) and FFN
# half (gate/up, down), of the head and of the embedding row, in us, as the
# persistent step spends them on one B200 (8B shape at positions 520-780).
HALF_COSTS = {"llama3-8b": (22.4, 29.9, 98.0, 5.0)}


# --------------------------------------------------------------- schedule --

@dataclass(frozen=True)
class Msg:
    src: int
    dst: int
    seq: int
    kind: str            # "state" (rank r -> r+1) or "token" (last -> 0)


class Schedule:
    """Tick schedule of n_seq sequences through n_ranks stages, n_steps
    tokens each (the first n_prompt of them fed from the prompt)."""

    def __init__(self, n_ranks: int, n_seq: int, n_steps: int, n_prompt: int = 0, first_step: int = 0):
        if n_ranks < 2:
            raise ValueError("a pipeline needs at least two stages")
        self.n_ranks, self.n_seq, self.n_steps = n_ranks, n_seq, n_steps
        self.n_prompt, self.first_step = n_prompt, first_step
        self.period = max(n_seq, n_ranks)
        self.n_ticks = (n_steps - 1) * self.period + (n_seq - 1) + (n_ranks - 1) + 1 if n_steps > 0 else 0

    def work(self, rank: int, tick: int):
        """(seq, step) rank works on in this tick, or None."""
        u = tick - rank
        if u < 0:
            return None
        k, s = divmod(u, self.period)
        if s >= self.n_seq or k >= self.n_steps:
            return None
        return s, self.first_step + k

    def messages(self, tick: int) -> list[Msg]:
        out = []
        last = self.n_ranks - 1
        for r in range(self.n_ranks):
            w = self.work(r, tick)
            if w is None:
                continue
            s, k = w
            if r < last:
                out.append(Msg(r, r + 1, s, "state"))
            elif self.n_prompt <= k + 1 < self.first_step + self.n_steps:
                # the next input token of s is this argmax (not a prompt token)
                out.append(Msg(last, 0, s, "token"))
        return out

    def step_ticks(self, step: int) -> tuple[int, int]:
        """Ticks [t0, t1) in which the ranks do `step` of every sequence in
        steady state (P ticks per step)."""
        t0 = (step - self.first_step) * self.period
        return t0, t0 + self.period


# ---------------------------------------------------------------- runtime --

class Exchanger:
    """Carries one tick's messages between stage runtimes."""

    def exchange(self, msgs: list[Msg], stages: dict) -> None:
        raise NotImplementedError


class LoopbackExchanger(Exchanger):
    """All ranks in this process: a message is a copy between their buffers."""

    def exchange(self, msgs, stages):
        for m in msgs:
            src, dst = stages[m.src], stages[m.dst]
            ss, ds = getattr(src, "stream", None), getattr(dst, "stream", None)
            if ss is None:
                dst.recv_buf(m.seq, m.kind).copy_(src.send_buf(m.seq, m.kind))
                continue
            import torch
            # the receiver's stream copies once the sender's output is
            # written; the sender reuses its buffer only after the copy
            ds.wait_stream(ss)
            with torch.cuda.stream(ds):
                dst.recv_buf(m.seq, m.kind).copy_(src.send_buf(m.seq, m.kind))
            ss.wait_stream(ds)


class LinkedExchanger(Exchanger):
    """Linked stages (ecu_link_*): the steps hand the state and the token to
    the next stage themselves, so a tick has nothing to carry."""

    def exchange(self, msgs, stages):
        return


class DistExchanger(Exchanger):
    """One rank per process over torch.distributed (NCCL between GPUs, gloo
    on the host): the tick's sends and receives of this rank as one group."""

    def __init__(self, rank: int):
        self.rank = rank

    def exchange(self, msgs, stages):
        import torch.distributed as dist
        me = stages[self.rank]
        ops = []
        for m in msgs:
            if m.src == self.rank:
                ops.append(dist.P2POp(dist.isend, me.send_buf(m.seq, m.kind), m.dst))
            elif m.dst == self.rank:
                ops.append(dist.P2POp(dist.irecv, me.recv_buf(m.seq, m.kind), m.src))
        if not ops:
            return
        stream = getattr(me, "stream", None)
        if stream is None:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            return
        import torch
        # NCCL orders itself after the current stream and w.wait() orders the
        # current stream after NCCL: make the stage's stream the current one
        with torch.cuda.stream(stream):
            for w in dist.batch_isend_irecv(ops):
                w.wait()


def run_ticks(sched: Schedule, stages: dict, exchanger: Exchanger, prompts=None, t0: int = 0,
              t1: int | None = None, on_tick=None) -> None:
    """Drive the local stages through ticks [t0, t1) of the schedule.
    stages: {rank: runtime} for the ranks of this process.  prompts[s][k] is
    fed as input token of step k of sequence s while k < sched.n_prompt."""
    t1 = sched.n_ticks if t1 is None else t1
    for t in range(t0, t1):
        for r, st in stages.items():
            w = sched.work(r, t)
            if w is None:
                continue
            s, k = w
            if r == 0 and k < sched.n_prompt:
                st.set_token(s, k)
            st.run(s, k)
        exchanger.exchange(sched.messages(t), stages)
        if on_tick is not None:
            on_tick(t)


class GpuStage:
    """One rank's stage on one GPU: per sequence one engine context -- a span
    of layers first..last with the embedding folded in on the first rank and
    the head on the last (ecu_ctx_open_span: the reference's EMBED / LAYERS /
    HEAD stages of one node, src/shard.c:358-437, as one persistent step) --
    forks of sequence 0's, all enqueued on one torch stream.  Input/output
    buffers are zero-copy torch views of the contexts' device state
    (ecu_state_ptr / ecu_token_ptr).

    Linked (link_local / link_dist): each context sends its output straight
    into the next stage's context of the same sequence from inside its step
    (the last stage its token into the first stage's), so a tick launches
    the steps and carries nothing.  Stages that share one GPU must then
    share one stream (`stream`), which runs their steps in tick order: a
    step never waits there for one that has not run.  Across processes, a
    rank synchronises its device before any collective: a persistent step
    holds every SM, so a collective's kernel waiting on this GPU for another
    rank would keep this rank's next step from launching while the other
    rank's step waits for that step's output."""

    def __init__(self, model, rank: int, n_ranks: int, first: int, last: int, n_layer: int, n_seq: int,
                 n_ctx: int, device: int, prompts=None, stream=None, halves: int = 0):
        import torch
        from . import engine as E
        self.rank, self.n_ranks, self.device = rank, n_ranks, device
        self.torch = torch
        self.dev = torch.device("cuda", device)
        # the first rank embeds, the last runs the head (first > last: the
        # head's GPU holds no layer, and the rank before it ends at the last
        # layer without the head)
        self.has_embed, self.has_head = rank == 0, rank == n_ranks - 1
        # halves: SPAN_FFN_FIRST / SPAN_ATTN_LAST, a range cut inside a layer
        flags = (E.SPAN_EMBED if self.has_embed else 0) | (E.SPAN_HEAD if self.has_head else 0) | halves
        base = [E.LlmCtx(model, E.STAGE_SPAN, first, last, n_ctx, device, span=flags)]
        self.chains = [base] + [[c.fork() for c in base] for _ in range(n_seq - 1)]
        self.n_embd = base[0].n_embd
        self.stream = stream if stream is not None else torch.cuda.Stream(device=self.dev)
        self.linked = False
        self._state = [[device_view(c.state_ptr(), self.n_embd + 1, "<f4", device) for c in ch]
                       for ch in self.chains]
        self._token = [[device_view(c.token_ptr(), 1, "<i4", device) for c in ch] for ch in self.chains]
        self.prompts = self.host_prompts = None
        if prompts is not None:
            self.prompts = torch.tensor(prompts, dtype=torch.int32, device=self.dev)
            self.host_prompts = [list(map(int, q)) for q in prompts]
        self.history = None

    def record_tokens(self, n_steps: int):
        """Keep every argmax in a device table [n_seq, n_steps] (last stage)."""
        self.history = self.torch.zeros((len(self.chains), n_steps), dtype=self.torch.int32, device=self.dev)

    # buffers the exchanger reads and writes
    def send_buf(self, s: int, kind: str):
        return self._token[s][-1] if kind == "token" else self._state[s][-1][: self.n_embd]

    def recv_buf(self, s: int, kind: str):
        return self._token[s][0] if kind == "token" else self._state[s][0][: self.n_embd]

    def set_token(self, s: int, k: int):
        if self.linked:
            self.feed(s, self.host_prompts[s][k])
            return
        with self.torch.cuda.stream(self.stream):
            self._token[s][0].copy_(self.prompts[s, k: k + 1])

    def feed(self, s: int, token: int):
        """Sequence s's next input token from the host (first stage)."""
        if self.linked:
            self.chains[s][0].link_feed(int(token), self.stream.cuda_stream)
        else:
            with self.torch.cuda.stream(self.stream):
                self._token[s][0].fill_(int(token))

    def run(self, s: int, k: int):
        torch = self.torch
        ch = self.chains[s]
        sp = self.stream.cuda_stream
        with torch.cuda.stream(self.stream):
            for i, c in enumerate(ch):
                if i > 0:
                    self._state[s][i][: self.n_embd].copy_(self._state[s][i - 1][: self.n_embd])
                c.step_dev(sp)
            if self.has_head and self.history is not None and k < self.history.shape[1]:
                self.history[s, k: k + 1].copy_(self._token[s][-1])

    def reset(self):
        for ch in self.chains:
            for c in ch:
                c.reset()

    def sync(self):
        self.stream.synchronize()
        for ch in self.chains:
            for c in ch:
                c.sync()

    def close(self):
        for ch in reversed(self.chains):
            for c in ch:
                c.close()


def link_local(stages: dict) -> None:
    """Link the stages of this process into a ring (rank r's contexts send
    to rank r + 1's of the same sequence, the last rank's head its token to
    rank 0): ecu_link_next_local / ecu_link_input."""
    ranks = sorted(stages)
    for i, r in enumerate(ranks):
        nxt = stages[ranks[(i + 1) % len(ranks)]]
        for s, ch in enumerate(stages[r].chains):
            ch[0].link_next(nxt.chains[s][0])
    for st in stages.values():
        for ch in st.chains:
            ch[0].link_input()
        st.linked = True


def link_dist(st: "GpuStage", rank: int, world: int) -> None:
    """link_local across processes (one rank per GPU): every rank's context
    handles to every rank (torch.distributed), then each rank maps the next
    rank's (ecu_link_handle / ecu_link_next)."""
    import torch.distributed as dist
    mine = [ch[0].link_handle() for ch in st.chains]
    every = [None] * world
    dist.all_gather_object(every, mine)
    nxt = every[(rank + 1) % world]
    for s, ch in enumerate(st.chains):
        ch[0].link_next(nxt[s])
        ch[0].link_input()
    st.linked = True
    dist.barrier()


def prefill_local(stages: dict, seq: int, prompt, send_rows=None, recv_rows=None, share_token=None) -> int | None:
    """The prompt of sequence `seq` through the pipeline as one batch per
    stage (ecu_prefill_rows): the reference's token-by-token prompt feed
    (src/shard.c:911-917) becomes one hop of n rows per stage boundary.
    stages: {rank: GpuStage} of this process, run in rank order on one row
    buffer; with one rank per process, recv_rows(r, rows) / send_rows(r,
    rows) carry the rows from rank r-1 / to rank r+1, and share_token(tok)
    brings the last stage's picked token to every rank.  The first stage's
    device token of the sequence is set to it, ready for the first decode
    step.  Returns the token."""
    import torch
    n = len(prompt)
    rows, tok = None, None
    for r in sorted(stages):
        st = stages[r]
        if rows is None:
            rows = torch.empty((n, st.n_embd), dtype=torch.float32, device=st.dev)
        if recv_rows is not None and r > 0:
            recv_rows(r, rows)
            torch.cuda.current_stream(st.dev).synchronize()
        for c in st.chains[seq]:
            t = c.prefill_rows(rows.data_ptr(), n, tokens=prompt)
            if t is not None:
                tok = t
        if send_rows is not None and r + 1 < st.n_ranks:
            send_rows(r, rows)
    if share_token is not None:
        tok = share_token(tok)
    if 0 in stages:
        stages[0].feed(seq, int(tok))
    return tok


def device_view(ptr: int, n: int, typestr: str, device: int):
    """A torch tensor over n elements of device memory owned by the engine
    (no copy, no ownership)."""
    import torch

    class _View:
        __cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (int(ptr), False),
                                    "version": 3, "strides": None}

    if not ptr:
        raise ValueError("null device pointer")
    return torch.as_tensor(_View(), device=torch.device("cuda", device))


# ------------------------------------------------------------------ bench --

def bench_main(args, rank: int, world: int, local: int, B) -> int:
    """bench.py at N > 1: the 8B decode pipelined over `world` GPUs.  B is
    the bench module (metric, config, clock sampler, byte counts)."""
    import datetime
    import json
    import time
    import torch
    import torch.distributed as dist
    from . import engine as E
    from . import synth

    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=180))
    try:
        spec = synth.spec(B.CONFIG, **({"n_layer": args.layers} if args.layers else {}))
        buf = B.build_model_gpu(spec, args.seed, local)
        model = E.GgufModel(buf)
        lb = layer_bytes(spec)
        head_b = tensor_bytes(spec, "output.weight") + tensor_bytes(spec, "output_norm.weight")
        emb_row = tensor_bytes(spec, "token_embd.weight") // spec.n_vocab
        if args.split == "ref":
            plan = [(a, b, 0) for a, b in split_stages(spec.n_layer, world)]
        elif args.split == "half" and B.CONFIG in HALF_COSTS and not args.layers:
            plan = split_half_layers(*HALF_COSTS[B.CONFIG][:2], spec.n_layer, world, *HALF_COSTS[B.CONFIG][2:])
        else:
            plan = [(a, b, 0) for a, b in
                    split_by_bytes(lb, world, head_bytes=int(head_b * HEAD_COST), embed_bytes=emb_row, head_alone=True)]
        first, last, halves = plan[rank]
        n_seq = args.seqs
        prompts = [synth.prompt_tokens(args.prompt, spec.n_vocab, seed=args.seed + 1 + s) for s in range(n_seq)]
        n_tok = args.prompt + args.warmup + 2 * args.steps + 2
        if n_tok > args.n_ctx:
            raise SystemExit(f"prompt + steps need {n_tok} positions > n_ctx {args.n_ctx}")
        st = GpuStage(model, rank, world, first, last, spec.n_layer, n_seq, args.n_ctx, local,
                      prompts=prompts if rank == 0 else None, halves=halves)
        del buf
        torch.cuda.empty_cache()
        linked = getattr(args, "hops", "link") == "link"
        if linked:
            # every step hands its output to the next GPU itself: no
            # exchange between ticks, the hosts only launch
            link_dist(st, rank, world)
            ex = LinkedExchanger()
        else:
            ex = DistExchanger(rank)
        stages = {rank: st}
        dev = st.dev
        dist.barrier()

        def send_rows(r, rows):
            dist.send(rows, r + 1)

        def recv_rows(r, rows):
            dist.recv(rows, r - 1)

        def share_token(tok):
            t = torch.tensor([tok if rank == world - 1 else 0], dtype=torch.int64, device=dev)
            dist.broadcast(t, world - 1)
            return int(t.item())

        def prefill(seqs):
            """Each sequence's prompt through the stages as one batch per
            stage; returns the first generated tokens."""
            firsts = []
            for q in seqs:
                firsts.append(prefill_local(stages, q, prompts[q], send_rows, recv_rows, share_token))
                torch.cuda.synchronize(local)
            dist.barrier()
            return firsts

        def timed(sched, t0, t1, host_tokens=False):
            """Device time of ticks [t0, t1) on this rank, max over ranks (ms)."""
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # (linked steps still in flight finish before any collective: a
            # collective's kernel holding an SM would keep this GPU's next
            # step, which another GPU's step waits for, from launching)
            torch.cuda.synchronize(local)
            dist.barrier()
            h0 = time.perf_counter()
            ev0.record(st.stream)
            if host_tokens and st.has_head:
                pinned = torch.zeros(n_seq, dtype=torch.int32, pin_memory=True)

                def tick(t):
                    w = sched.work(rank, t)
                    if w is not None and w[0] == n_seq - 1:      # a step of every sequence done
                        with torch.cuda.stream(st.stream):
                            for s in range(n_seq):
                                pinned[s: s + 1].copy_(st._token[s][-1], non_blocking=True)
                        st.stream.synchronize()
                run_ticks(sched, stages, ex, t0=t0, t1=t1, on_tick=tick)
            else:
                run_ticks(sched, stages, ex, t0=t0, t1=t1)
            ev1.record(st.stream)
            torch.cuda.synchronize(local)
            host_s = time.perf_counter() - h0
            dist.barrier()
            ms = torch.tensor([ev0.elapsed_time(ev1), host_s * 1e3], dtype=torch.float64, device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            return float(ms[0]), float(ms[1])

        n = args.prompt
        # (1) one sequence alone: the batch-1 latency through all stages
        t_pf = time.perf_counter()
        prefill([0])
        pf_s = time.perf_counter() - t_pf
        s1 = Schedule(world, 1, args.warmup + args.steps, n_prompt=0, first_step=n)
        w0 = s1.step_ticks(n + args.warmup)[0]
        run_ticks(s1, stages, ex, t0=0, t1=w0)
        ms1, _ = timed(s1, w0, s1.n_ticks)
        b1_tps = args.steps / (ms1 / 1e3)
        st.sync()
        st.reset()

        # (2) n_seq interleaved sequences: prompts, warm-up, timed, end-to-end
        dec = args.warmup + 2 * args.steps
        firsts = prefill(range(n_seq))
        sched = Schedule(world, n_seq, dec, n_prompt=0, first_step=n)
        if st.has_head:
            st.record_tokens(n + dec)
        ta = sched.step_ticks(n + args.warmup)[0]
        tb = sched.step_ticks(n + args.warmup + args.steps)[0]
        run_ticks(sched, stages, ex, t0=0, t1=ta)
        l0 = E.kernel_launches()
        clocks = B.ClockSampler(local)
        if rank == 0:
            clocks.start()
        ms, _ = timed(sched, ta, tb)
        launches = E.kernel_launches() - l0
        clk = clocks.stop() if rank == 0 else None
        _, e2e_ms = timed(sched, tb, sched.n_ticks, host_tokens=True)
        st.sync()
        lt = torch.tensor([launches], dtype=torch.int64, device=dev)
        dist.all_reduce(lt)
        tps = n_seq * args.steps / (ms / 1e3)
        # tokens completed in the end-to-end window: every step after tb
        e2e_steps = dec - (args.warmup + args.steps)
        e2e = n_seq * e2e_steps / (e2e_ms / 1e3)
        # sequence 0's greedy tokens through the pipeline (the first from the
        # staged prompt, then the last stage's record) against one GPU's FULL
        # context on the same prompt (ecu_prefill, then per-token steps)
        hist = st.history[0].clone() if st.has_head else torch.zeros(n + dec, dtype=torch.int32, device=dev)
        dist.broadcast(hist, src=world - 1)
        dist.barrier()             # every rank's steps are over: no link writes into freed memory
        st.close()
        pp_check = None
        if rank == 0:
            n_gen = dec + 1
            ref = B.one_gpu_tokens(model, spec, args, local, n_gen, prompts[0], prefill=True)
            got = [int(firsts[0])] + [int(t) for t in hist[n: n + dec].cpu().tolist()]
            pp_check = {"tokens_match_one_gpu": got == ref, "tokens_checked": n_gen, "sequence": 0}
        dist.barrier()
        # (3) the other partition on the same GPUs: batch-1 tensor parallel
        from . import tensor_parallel
        tp_prompt = synth.prompt_tokens(args.prompt, spec.n_vocab, seed=args.seed)
        tp_ref = B.one_gpu_tokens(model, spec, args, local, 32, tp_prompt) if rank == 0 else None
        tp = tensor_parallel.measure(args, rank, world, local, B, model, spec, ref_tokens=tp_ref)

        if rank == 0:
            peak, peak_kind = B.peaks()
            bpt = B.algorithmic_bytes_per_token(spec, args.prompt + args.warmup + (args.steps - 1) / 2)
            line = {
                "metric": B.METRIC, "value": round(tps, 2), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
                "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "q4_0 codes x int8 digit planes, fp32 accumulate",
                "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_0/Q8_0 on the GPU, random prompts",
                "config": {"workload": f"llama3-8b-shape Q4_0 decode, layer pipeline over {world} GPUs "
                                       f"(one span context per GPU and sequence, "
                                       + ("linked steps: each writes its output into the next GPU's step "
                                          "over NVLink" if linked else "NCCL send/recv hops between steps")
                                       + f"), {n_seq} interleaved sequences; a step = one token of every "
                                         f"sequence; prompts {n} tokens each as one batch per stage",
                           "hops": "link" if linked else "nccl",
                           "stages": [stage_text(p) for p in plan], "split": args.split,
                           "sequences": n_seq, "prompt_tokens": args.prompt, "n_ctx": args.n_ctx,
                           "l2": "inputs larger than L2 (4.49 GB of weights per token)"},
                "token_roofline": {"bytes_per_token": bpt, "achieved_gbs": round(bpt * tps / 1e9, 1),
                                   "peak_gbs": peak * world, "frac": round(bpt * tps / 1e9 / (peak * world), 4),
                                   "peak_kind": peak_kind},
                "pp_batch1": {"value": round(b1_tps, 2), "unit": "tokens/s",
                              "frac": round(bpt * b1_tps / 1e9 / peak, 4),
                              "note": "one sequence: one stage busy at a time"},
                "prefill_one_sequence": {"tokens": n, "s": round(pf_s, 3),
                                         "note": "ecu_prefill_rows per stage, rows over NCCL send/recv; wall "
                                                 "time with barriers"},
                "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 4 * n_seq,
                        "api": "ecu_step_dev per stage and sequence (the token fed back on the devices); the "
                               "last stage copies every step's tokens to the host and waits for them"},
                "gpu_launches": int(lt.item()),
                "clocks": clk,
                "pp_parity": pp_check,
                "tp": tp,
            }
            print(json.dumps(line), flush=True)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0


def bench_long_main(args, rank: int, world: int, local: int, B) -> int:
    """bench.py --model llama2-70b at N > 1: the 70B shape (Q4_K layers,
    Q8_0 embedding and head) layer-pipelined over `world` GPUs, batch 1.
    Each rank generates only its stage's tensors (synth.stage_tensors; the
    same bytes as the whole model's); the prompt goes through the stages as
    one batch per stage (ecu_prefill_rows, the rows handed on by NCCL
    send/recv); then K greedy decode steps of the one sequence, one stage
    busy at a time (the tick schedule of the 8B pipeline with one sequence).
    B is the bench module."""
    import datetime
    import json
    import time
    import torch
    import torch.distributed as dist
    from . import engine as E
    from . import synth

    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=600))
    try:
        spec = synth.spec(args.model, **({"n_layer": args.layers} if args.layers else {}))
        lb = layer_bytes(spec)
        head_b = tensor_bytes(spec, "output.weight") + tensor_bytes(spec, "output_norm.weight")
        emb_row = tensor_bytes(spec, "token_embd.weight") // spec.n_vocab
        plan = split_stages(spec.n_layer, world) if args.split == "ref" else \
            split_by_bytes(lb, world, head_bytes=int(head_b * HEAD_COST), embed_bytes=emb_row, head_alone=True)
        first, last = plan[rank]
        need = args.prompt + args.warmup + args.steps + 2
        if need > args.n_ctx:
            raise SystemExit(f"prompt + steps need {need} positions > n_ctx {args.n_ctx}")
        t_b = time.perf_counter()
        only = synth.stage_tensors(spec, first, last, rank == 0, rank == world - 1)
        torch.cuda.set_device(local)
        buf = synth.build_model(spec, seed=args.seed, device=f"cuda:{local}", only=only)
        torch.cuda.empty_cache()
        model = E.GgufModel(buf)
        st = GpuStage(model, rank, world, first, last, spec.n_layer, 1, args.n_ctx, local)
        del buf
        t_b = time.perf_counter() - t_b
        prompt = synth.prompt_tokens(args.prompt, spec.n_vocab, seed=args.seed)
        dev = torch.device("cuda", local)

        def send_rows(r, rows):
            dist.send(rows, r + 1)

        def recv_rows(r, rows):
            dist.recv(rows, r - 1)

        def share_token(tok):
            t = torch.tensor([tok if rank == world - 1 else 0], dtype=torch.int64, device=dev)
            dist.broadcast(t, world - 1)
            return int(t.item())

        linked = getattr(args, "hops", "link") == "link"
        if linked:
            link_dist(st, rank, world)
        dist.barrier()
        t0 = time.perf_counter()
        first_tok = prefill_local({rank: st}, 0, prompt, send_rows, recv_rows, share_token)
        dist.barrier()
        pf_s = time.perf_counter() - t0

        n = len(prompt)
        sched = Schedule(world, 1, args.warmup + 2 * args.steps, n_prompt=0, first_step=n)
        ex = LinkedExchanger() if linked else DistExchanger(rank)
        stages = {rank: st}
        ta = sched.step_ticks(n + args.warmup)[0]
        tb = sched.step_ticks(n + args.warmup + args.steps)[0]
        run_ticks(sched, stages, ex, t0=0, t1=ta)
        clocks = B.ClockSampler(local)
        if rank == 0:
            clocks.start()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(local)          # (no collective while linked steps are in flight)
        dist.barrier()
        l0 = E.kernel_launches()
        ev0.record(st.stream)
        run_ticks(sched, stages, ex, t0=ta, t1=tb)
        ev1.record(st.stream)
        torch.cuda.synchronize(local)
        launches = E.kernel_launches() - l0
        clk = clocks.stop() if rank == 0 else None
        ms_t = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
        tps = args.steps / (ms / 1e3)
        # end to end: the last stage copies every step's token to the host
        pinned = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        toks = []

        def tick(t):
            w = sched.work(rank, t)
            if w is not None and st.has_head:
                with torch.cuda.stream(st.stream):
                    pinned.copy_(st._token[0][-1], non_blocking=True)
                st.stream.synchronize()
                toks.append(int(pinned.item()))

        torch.cuda.synchronize(local)
        dist.barrier()
        h0 = time.perf_counter()
        run_ticks(sched, stages, ex, t0=tb, t1=sched.n_ticks, on_tick=tick)
        st.sync()
        e2e_t = torch.tensor([time.perf_counter() - h0], dtype=torch.float64, device=dev)
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e = args.steps / float(e2e_t.item())
        lt = torch.tensor([launches], dtype=torch.int64, device=dev)
        dist.all_reduce(lt)
        tk = torch.tensor(toks[:8] + [0] * (8 - len(toks[:8])), dtype=torch.int64, device=dev)
        dist.broadcast(tk, world - 1)
        if rank == 0:
            peak, peak_kind = B.peaks()
            bpt = B.algorithmic_bytes_per_token(spec, n + args.warmup + (args.steps - 1) / 2)
            pf_flops = 2.0 * n * B.prefill_params(spec)
            line = {
                "metric": B.metric_for(args.model), "value": round(tps, 2), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": B.dtype_text(spec),
                "data": "synthetic: seeded N(0,0.02) weights quantised on the GPU, each rank its stage's tensors; "
                        "random prompt",
                "config": {"workload": B.workload_text(spec, args.model) + f", KV fp32 {args.n_ctx}, layer pipeline "
                                       f"over {world} GPUs, batch 1, "
                                       + ("linked steps over NVLink" if linked else "NCCL send/recv hops"),
                           "hops": "link" if linked else "nccl",
                           "stages": [list(p_) for p_ in plan], "split": args.split, "prompt_tokens": n,
                           "decode_positions": [n + args.warmup, n + args.warmup + args.steps - 1],
                           "l2": f"inputs larger than L2 ({bpt / 1e9:.1f} GB per token)"},
                "token_roofline": {"bytes_per_token": bpt, "achieved_gbs": round(bpt * tps / 1e9, 1),
                                   "peak_gbs": peak, "frac": round(bpt * tps / 1e9 / peak, 4),
                                   "frac_of_8tbs_nominal": round(bpt * tps / 1e9 / 8000, 4), "peak_kind": peak_kind,
                                   "note": "batch 1 through a layer pipeline: one stage streams at a time, so the "
                                           "bound is one GPU's HBM bandwidth"},
                "prefill": {"tokens": n, "s": round(pf_s, 3), "tokens_per_s": round(n / pf_s, 1),
                            "tflops_useful": round(pf_flops / pf_s / 1e12, 2),
                            "note": "the prompt as one batch per stage (ecu_prefill_rows), the rows handed on by "
                                    "NCCL send/recv; wall time with barriers", "first_token": first_tok},
                "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
                        "api": "ecu_step_dev chain per stage; the last stage copies each token to the host"},
                "first_decode_tokens": [int(v) for v in tk.cpu().tolist()],
                "gpu_launches": int(lt.item()),
                "clocks": clk,
                "setup_s": {"stage_model_build_and_upload": round(t_b, 1)},
            }
            print(json.dumps(line), flush=True)
        dist.barrier()             # every rank's steps are over: no link writes into freed memory
        st.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0


def layer_bytes(spec) -> list[int]:
    from . import synth
    from . import gguf as G
    per = [0] * spec.n_layer
    for name, dims, gt in synth.tensor_list(spec):
        if name.startswith("blk."):
            i = int(name.split(".")[1])
            per[i] += G.type_nbytes(gt, math.prod(dims))
    return per


def tensor_bytes(spec, name: str) -> int:
    from . import synth
    from . import gguf as G
    for n, dims, gt in synth.tensor_list(spec):
        if n == name:
            return G.type_nbytes(gt, math.prod(dims))
    if name == "output.weight":                # tied: the head reads token_embd
        return tensor_bytes(spec, "token_embd.weight")
    return 0
