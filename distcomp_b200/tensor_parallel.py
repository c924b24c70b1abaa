"""Tensor-parallel decode: one FULL context per GPU, one process per GPU.

The alternative partition to the layer pipeline (src/shard.c:358-437).  Rank
r of w holds, of every layer, query heads [r*n_head/w, ..) with their KV
heads and KV cache, rows [r*n_embd/w, ..) of attn_output and ffn_down, FFN
channels [r*n_ff/w, ..) of the fused gate/up matrix, and a slice of the
vocabulary rows of the head (ecu_ctx_open_tp).  No projection splits its
input, so every output element is computed by one rank with the arithmetic
of the one-GPU step and the ranks' results are bit-identical to it; inside
the persistent step each rank stores its outputs straight into every rank's
copy of the tagged vectors (NVLink peer stores), and the argmax is combined
from one (value, index) pair per rank.

This module is the host side: open a rank, exchange the shareable handles of
the ranks' vector blocks through torch.distributed (any backend), connect.
Every rank must then issue the same steps in the same order.
"""
from __future__ import annotations


def exchange_handles(mine: bytes, world: int) -> list[bytes]:
    """Every rank's handle, in rank order (torch.distributed all_gather)."""
    import torch.distributed as dist
    out: list = [None] * world
    dist.all_gather_object(out, mine)
    for i, h in enumerate(out):
        if not isinstance(h, (bytes, bytearray)) or len(h) != 64:
            raise RuntimeError(f"rank {i} sent a malformed handle")
    return [bytes(h) for h in out]


def open_rank(model, rank: int, world: int, n_ctx: int, device: int):
    """This rank's tensor-parallel FULL context, connected to the others."""
    import torch.distributed as dist
    from . import engine as E
    ctx = E.LlmCtx(model, E.STAGE_FULL, n_ctx=n_ctx, device=device, tp=(rank, world))
    try:
        ctx.tp_connect(exchange_handles(ctx.tp_handle(), world))
    except Exception:
        ctx.close()
        raise
    dist.barrier()                          # every rank mapped before any step
    return ctx


def measure(args, rank: int, world: int, local: int, B, model, spec, ref_tokens=None) -> dict | None:
    """Batch-1 tensor-parallel decode of `model` over the process group
    (already initialised): the prompt token by token, W warm-up and K timed
    steps (device time, max over ranks), K steps end to end through
    ecu_forward, and a greedy check against one GPU's tokens (ref_tokens,
    rank 0: the tokens a FULL context generates after the same prompt).
    Returns rank 0's fields (None on the other ranks)."""
    import time
    import numpy as np
    import torch
    import torch.distributed as dist
    from . import engine as E
    from . import synth

    ctx = open_rank(model, rank, world, args.n_ctx, local)
    try:
        prompt = synth.prompt_tokens(args.prompt, spec.n_vocab, seed=args.seed)
        n_check = len(ref_tokens) if ref_tokens is not None else 0
        n_check = int(_bcast_int(n_check, rank, local))
        got = ctx.generate(prompt, max(1, n_check))
        ctx.decode_async(args.warmup)
        ctx.sync()
        stream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pos0 = ctx.pos
        dist.barrier()
        torch.cuda.synchronize(local)
        l0 = E.kernel_launches()
        e0.record(stream)
        ctx.decode_async(args.steps)
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize(local)
        launches = E.kernel_launches() - l0
        ms_t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
        tps = args.steps / (ms / 1e3)
        prof = ctx.profile_steps(args.profile_steps)

        # end to end through ecu_forward with host buffers, every rank
        out = np.zeros(spec.n_embd + 1, dtype=np.float32)
        tok = ctx.pick()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            if ctx.forward(tok, out) != 0:
                raise SystemExit("ecu_forward failed: " + E.last_error())
            tok = int(out[spec.n_embd])
        e2e_t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e = args.steps / float(e2e_t.item())
        # every rank picked the same tokens (the greedy check's and the last one)
        mine = torch.tensor(got + [tok], dtype=torch.int64, device=f"cuda:{local}")
        allt = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allt, mine)
        same = all(bool(torch.equal(t, mine)) for t in allt)
        lt = torch.tensor([launches], dtype=torch.int64, device=f"cuda:{local}")
        dist.all_reduce(lt)
        path = ctx.path()
    finally:
        ctx.close()
    dist.barrier()
    if rank != 0:
        return None
    peak, peak_kind = B.peaks()
    bpt = B.algorithmic_bytes_per_token(spec, pos0 + (args.steps - 1) / 2)
    step = prof.get("decode_step")
    res = {
        "value": round(tps, 2), "unit": "tokens/s", "ms_per_step": round(ms / args.steps, 4),
        "decode_positions": [pos0, pos0 + args.steps - 1],
        "token_roofline": {"bytes_per_token": bpt, "achieved_gbs": round(bpt * tps / 1e9, 1),
                           "peak_gbs": peak * world, "frac": round(bpt * tps / 1e9 / (peak * world), 4),
                           "peak_kind": peak_kind},
        "rank0_step_us": round(step[1] / step[0] * 1e3, 1) if step else None,
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": (spec.n_embd + 1) * 4,
                "api": "ecu_forward on every rank (tensor-parallel FULL contexts)"},
        "ranks_agree": bool(same),
        "gpu_launches": int(lt.item()),
        "step_path": path,
    }
    if ref_tokens is not None:
        res["tokens_match_one_gpu"] = got[:n_check] == list(ref_tokens)
        res["tokens_checked"] = n_check
    return res


def _bcast_int(v: int, rank: int, local: int) -> int:
    import torch
    import torch.distributed as dist
    t = torch.tensor([v if rank == 0 else 0], dtype=torch.int64, device=f"cuda:{local}")
    dist.broadcast(t, 0)
    return int(t.item())


def bench_main(args, rank: int, world: int, local: int, B) -> int:
    """bench.py at N > 1 with --mode tp: batch-1 decode of the 8B shape, one
    token per step across all ranks.  B is the bench module."""
    import datetime
    import json
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
        need = args.prompt + args.warmup + 2 * args.steps + args.profile_steps + 2
        if need > args.n_ctx:
            raise SystemExit(f"prompt + steps need {need} positions > n_ctx {args.n_ctx}")
        ref = B.one_gpu_tokens(model, spec, args, local, n=32) if rank == 0 else None
        clocks = B.ClockSampler(local)
        if rank == 0:
            clocks.start()
        r = measure(args, rank, world, local, B, model, spec, ref_tokens=ref)
        clk = clocks.stop() if rank == 0 else None
        if rank == 0:
            line = {
                "metric": B.METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "q4_0 codes x int8 digit planes, fp32 accumulate",
                "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_0/Q8_0 on the GPU, random prompt",
                "config": {"workload": f"llama3-8b-shape Q4_0 decode, batch 1, tensor parallel over {world} GPUs "
                                       "(heads / output rows / FFN channels / vocabulary split; outputs "
                                       "exchanged by NVLink peer stores inside the persistent step)",
                           "prompt_tokens": args.prompt, "decode_positions": r["decode_positions"],
                           "n_ctx": args.n_ctx, "l2": "inputs larger than L2 (4.49 GB of weights per token)"},
                "clocks": clk,
            }
            line.update({k: v for k, v in r.items() if k not in ("value", "unit", "ms_per_step",
                                                                  "decode_positions")})
            print(json.dumps(line), flush=True)
            if not r["ranks_agree"]:
                raise SystemExit("tensor-parallel ranks picked different tokens")
    finally:
        dist.destroy_process_group()
    return 0
