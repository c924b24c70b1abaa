#!/usr/bin/env python3
"""Batch-1 greedy decode throughput of the 8B-shaped Q4_0 llama on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the 8B decode configuration): dim 4096, 32 layers, 32/8 heads,
FFN 14336, vocab 128256, RoPE theta 5e5; N(0,0.02) weights quantised to
Q4_0 (embedding and head Q8_0), generated on the GPU from a fixed seed;
KV cache fp32 for 4096 positions.  A 512-token random prompt goes in
first through ecu_prefill (timed once: the `prefill` field), then W untimed
and K timed greedy decode steps.  One step = one
token through embed -> 32 layers -> head -> argmax, the next token fed back
on the device (one persistent-kernel launch per token).  The 4.5 GB of weights
stream from HBM every step, far above the 126 MB L2, so no flush is needed.

One JSON line: value = tokens/s from CUDA events around the K steps; e2e =
the same through ecu_forward with host buffers (token in, state + token
out, pinned copies inside the timed region); roofline = the dominant
kernel from CUDA events of a profiling replay: the persistent whole-step
kernel (one launch per token, the default path), or with ECU_MEGA=0 the
fused gate/up GEMV + SwiGLU of the per-kernel step; cpu_baseline = the
reference engine (oracle/_ref, compiled from the reference's sources) on
this host's cores on a bounded sample.

--impl reference times that reference CPU engine alone (rank 0) on the
same config and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s (batch 1) + % HBM roofline, 8B-shape Q4_0, 1/2/4/8 B200 vs host CPU"
CONFIG = "llama3-8b"
# other shapes (--model): the 70B long-context one, weights in Q4_K
METRICS = {"llama2-70b": "decode tokens/s (batch 1) + % HBM roofline, 70B-shape Q4_K long context, B200"}


def metric_for(key: str) -> str:
    return METRICS.get(key, METRIC)


def workload_text(spec, key: str) -> str:
    from distcomp_b200 import gguf as G
    hd = spec.n_embd // spec.n_head
    return (f"{key}-shape {G.TYPE_NAMES[spec.wtype]} decode, batch 1 (dim {spec.n_embd}, {spec.n_layer} layers, "
            f"{spec.n_head}/{spec.n_head_kv} heads, head_dim {hd}, ffn {spec.n_ff}, vocab {spec.n_vocab}, "
            f"theta {spec.rope_base:g}, embedding {G.TYPE_NAMES[spec.emb_type]}, head {G.TYPE_NAMES[spec.out_type]})")


def dtype_text(spec) -> str:
    from distcomp_b200 import gguf as G
    return f"{G.TYPE_NAMES[spec.wtype].lower()} codes x int8 digit planes, fp32 accumulate"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--n-ctx", type=int, default=4096)
    ap.add_argument("--profile-steps", type=int, default=2)
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--seqs", type=int, default=8,
                    help="N > 1: independent sequences interleaved through the layer pipeline")
    ap.add_argument("--mode", choices=["pp", "tp", "gemv"], default="pp",
                    help="N > 1: layer pipeline with interleaved sequences (pp) or batch-1 tensor "
                         "parallelism (tp); gemv: the quantised-matvec microbenchmark (one GPU)")
    ap.add_argument("--hops", choices=["link", "nccl"], default="link",
                    help="N > 1 pipeline: each step writes its output into the next GPU's step (link), or NCCL "
                         "send/recv between the steps (nccl)")
    ap.add_argument("--split", choices=["half", "bytes", "ref"], default="half",
                    help="N > 1: ranges of layer halves balancing each stage's time (a GPU may hold half a "
                         "layer; 8B interleaved pipeline), whole layers balancing time per stage (bytes, the "
                         "head at its cost per byte), or shard.c's ceil(layers/stages) rule")
    ap.add_argument("--gemv-case", default="",
                    help="--mode gemv: only this case, e.g. Q4_0:14336x4096 (profiler captures)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override n_layer (reduced-depth runs for profiler captures; not a bench line)")
    ap.add_argument("--model", choices=["llama3-8b", "llama2-70b"], default=CONFIG,
                    help="model shape (one GPU): the 8B Q4_0 headline, or the 70B Q4_K long-context shape "
                         "(use --prompt 8192 --n-ctx 8704 --steps 128 for its configuration)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"dcb200_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names[1:], f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def prefill_params(spec) -> int:
    """Weights a prompt token multiplies in the layers (the GEMMs of ecu_prefill)."""
    hd = spec.n_embd // spec.n_head
    qd, kvd = spec.n_head * hd, spec.n_head_kv * hd
    per = spec.n_embd * (qd + 2 * kvd) + qd * spec.n_embd + 3 * spec.n_embd * spec.n_ff
    return per * spec.n_layer


def algorithmic_bytes_per_token(spec, pos_mean: float) -> float:
    """Weights as stored + KV rows read (positions 0..pos) and written."""
    from distcomp_b200 import synth
    from distcomp_b200 import gguf as G
    w = 0
    for name, dims, gt in synth.tensor_list(spec):
        n = 1
        for d in dims:
            n *= d
        if name == "token_embd.weight":
            w += G.type_nbytes(gt, dims[0])        # one embedding row
        else:
            w += G.type_nbytes(gt, n)
    hd = spec.n_embd // spec.n_head
    kv_row = 2 * spec.n_head_kv * hd * 4 * spec.n_layer
    return w + kv_row * (pos_mean + 1) + kv_row


def cpu_reference_tokens_per_s(buf, spec, budget_s: float, max_tokens: int, threads: int | None = None):
    """The reference engine (three stages, as src/shard.c's local run) on the
    host cores: decode tokens from position 0 until the budget is used.
    Returns (tokens/s, tokens timed, threads, kind)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle
    kind = "reference" if oracle.available("ref") else "port"
    lib = oracle.get("ref" if kind == "reference" else "port")
    n_thr = 1
    if kind == "reference":
        n_thr = min(64, threads or os.cpu_count() or 1)
        lib.set_threads(n_thr)
    m = lib.model(buf)
    emb, lay, head = m.ctx(0), m.ctx(1, 0, spec.n_layer - 1, 64), m.ctx(2)
    st = np.zeros(spec.n_embd + 8, dtype=np.float32)
    tok = 3

    def step(t):
        assert emb.forward(t, st) == 0 and lay.forward(t, st) == 0 and head.forward(t, st) == 0
        return int(st[spec.n_embd])

    tok = step(tok)                      # warm-up: thread pool, page-in
    n, t0 = 0, time.perf_counter()
    while n < max_tokens:
        tok = step(tok)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return n / dt, n, n_thr, kind


def build_model_gpu(spec, seed, device):
    from distcomp_b200 import synth
    import torch
    torch.cuda.set_device(device)
    buf = synth.build_model(spec, seed=seed, device=f"cuda:{device}")
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return buf


def one_gpu_tokens(model, spec, args, device: int, n: int, prompt, prefill: bool = False) -> list[int]:
    """n greedy tokens after `prompt` (fed one token at a time, or with
    prefill as one batch through ecu_prefill) from a FULL context on one
    GPU: the reference for the multi-GPU partitions' tokens."""
    import numpy as np
    from distcomp_b200 import engine as E
    c = E.LlmCtx(model, E.STAGE_FULL, n_ctx=args.n_ctx, device=device)
    try:
        if not prefill:
            return c.generate(list(prompt), n)
        toks = [c.prefill(list(prompt))]
        out = np.zeros(spec.n_embd + 1, dtype=np.float32)
        while len(toks) < n:
            if c.forward(toks[-1], out) != 0:
                raise RuntimeError(E.last_error())
            toks.append(int(out[spec.n_embd]))
        return toks
    finally:
        c.close()


def load_traffic(name: str, bytes_per_launch: float):
    """dram bytes per launch of the dominant kernel from the committed ncu
    summary, when one exists: the captured bytes of that launch, or (for a
    capture of a reduced case) the captured traffic / algorithmic-bytes ratio
    applied to this launch's algorithmic bytes."""
    p = ROOT / "profiles" / name
    if p.exists():
        try:
            d = json.loads(p.read_text())
            if d.get("traffic_over_algorithmic"):
                return int(round(float(d["traffic_over_algorithmic"]) * bytes_per_launch)), d.get("scaled_from")
            return d.get("dram_bytes_per_launch"), d.get("scaled_from")
        except Exception:
            pass
    return None, None


def our_arm(args, rank, world, local):
    import numpy as np
    import torch
    from distcomp_b200 import engine as E
    from distcomp_b200 import synth

    if world > 1 and args.mode == "tp":
        from distcomp_b200 import tensor_parallel
        return tensor_parallel.bench_main(args, rank, world, local, sys.modules[__name__])
    if world > 1:
        from distcomp_b200 import pipeline
        if args.model != CONFIG:
            return pipeline.bench_long_main(args, rank, world, local, sys.modules[__name__])
        return pipeline.bench_main(args, rank, world, local, sys.modules[__name__])

    spec = synth.spec(args.model, **({"n_layer": args.layers} if args.layers else {}))
    t_build = time.perf_counter()
    buf = build_model_gpu(spec, args.seed, local)
    t_build = time.perf_counter() - t_build
    model = E.GgufModel(buf)
    t_up = time.perf_counter()
    ctx = E.LlmCtx(model, E.STAGE_FULL, n_ctx=args.n_ctx, device=local)
    t_up = time.perf_counter() - t_up
    prompt = synth.prompt_tokens(args.prompt, spec.n_vocab, seed=args.seed)
    need = args.prompt + args.warmup + 2 * args.steps + args.profile_steps + 2
    if need > args.n_ctx:
        raise SystemExit(f"prompt + steps need {need} positions > n_ctx {args.n_ctx}")

    # the prompt through ecu_prefill (one batch per layer on the tensor
    # cores), timed once after a warm-up prefill of the same prompt
    ctx.prefill(prompt)
    ctx.reset()
    torch.cuda.synchronize(local)
    t_pf = time.perf_counter()
    first_tok = ctx.prefill(prompt)
    t_pf = time.perf_counter() - t_pf
    pf_flops = 2.0 * args.prompt * prefill_params(spec)
    ctx.decode_async(args.warmup)
    ctx.sync()
    stream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    pos0 = ctx.pos
    torch.cuda.synchronize(local)
    l0 = E.kernel_launches()
    e0.record(stream)
    ctx.decode_async(args.steps)
    e1.record(stream)
    ctx.sync()
    torch.cuda.synchronize(local)
    launches = E.kernel_launches() - l0
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    tps = args.steps / (ms / 1e3)

    # dominant-kernel roofline from a profiling replay: the persistent step
    # kernel when the context runs one (events around each launch), else the
    # fused gate/up GEMV (events around every kernel)
    prof = ctx.profile_steps(args.profile_steps)
    peak, peak_kind = peaks()
    if "decode_step" in prof:
        dom = "decode_step"
        kname = (f"k_decode_mega<{spec.n_embd // spec.n_head}, {spec.n_head // spec.n_head_kv}> "
                 "(persistent kernel: the whole token step)")
        tname = "decode_step_mega_8b.json" if args.model == CONFIG and not args.layers else None
    else:
        dom, kname = "gemv_gate_up", "k_gemv_fast<Q4_0, rmsnorm, swiglu> (fused ffn_gate+ffn_up)"
        tname = "gemv_gate_up_q4_0_8b.json"
    n_l, tot_ms, bpl = prof[dom]
    traffic, scaled = load_traffic(tname, bpl) if tname else (None, None)
    avg_ms = tot_ms / n_l
    achieved = bpl / (avg_ms / 1e3) / 1e9

    # end to end through the C ABI with host buffers
    out = np.zeros(spec.n_embd + 1, dtype=np.float32)
    tok = ctx.pick()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        if ctx.forward(tok, out) != 0:
            raise SystemExit("ecu_forward failed: " + E.last_error())
        tok = int(out[spec.n_embd])
    e2e_s = time.perf_counter() - t0
    e2e = args.steps / e2e_s

    bpt = algorithmic_bytes_per_token(spec, pos0 + (args.steps - 1) / 2)
    wbytes = algorithmic_bytes_per_token(spec, -1.0) - 2 * spec.n_head_kv * (spec.n_embd // spec.n_head) * 4 * spec.n_layer
    line = {
        "metric": metric_for(args.model), "value": round(tps, 2), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_text(spec),
        "data": "synthetic: seeded N(0,0.02) weights quantised on the GPU, random prompt",
        "config": {"workload": workload_text(spec, args.model) + f", KV fp32 {args.n_ctx}",
                   "prompt_tokens": args.prompt, "decode_positions": [pos0, pos0 + args.steps - 1],
                   "l2": f"inputs larger than L2 ({wbytes / 1e9:.2f} GB of weights per step)",
                   "n_ctx": args.n_ctx},
        "token_roofline": {"bytes_per_token": bpt, "achieved_gbs": round(bpt * tps / 1e9, 1),
                           "peak_gbs": peak, "frac": round(bpt * tps / 1e9 / peak, 4),
                           "frac_of_8tbs_nominal": round(bpt * tps / 1e9 / 8000, 4), "peak_kind": peak_kind},
        "roofline": {"kernel": kname, "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "bytes_per_launch": bpl, "avg_launch_us": round(avg_ms * 1e3, 2),
                     "peak_kind": peak_kind, "traffic_scaled_from": scaled},
        "kernels_per_token": {k: {"launches": v[0] / args.profile_steps, "us": round(v[1] / args.profile_steps * 1e3, 1),
                                  "gbs": round(v[2] * v[0] / (v[1] / 1e3) / 1e9, 1) if v[1] > 0 else None}
                              for k, v in prof.items()},
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": (spec.n_embd + 1) * 4, "api": "ecu_forward (FULL context)"},
        "gpu_launches": int(launches),
        "prefill": {"tokens": args.prompt, "ms": round(t_pf * 1e3, 2), "tokens_per_s": round(args.prompt / t_pf, 1),
                    "tflops_useful": round(pf_flops / t_pf / 1e12, 2),
                    "note": "ecu_prefill wall time incl. host sync; GEMMs split-fp16 (3 tensor-core "
                            "products per useful one), first token " + str(first_tok)},
        "step_path": ctx.path(),
        "clocks": clk,
        "setup_s": {"model_build": round(t_build, 1), "upload": round(t_up, 1)},
    }
    if not args.no_cpu_baseline:
        v, n, thr, kind = cpu_reference_tokens_per_s(buf, spec, args.cpu_sample_s, 64)
        line["cpu_baseline"] = {"value": round(v, 4), "unit": "tokens/s", "cores": thr, "kind": kind,
                                "sample": f"{n} decode tokens at positions 1..{n} of the same model "
                                          f"(embed+{spec.n_layer} layers+head, three stages like shard.c's "
                                          f"local run); KV reads differ from the timed positions"}
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


GEMV_METRIC = "quantised matvec GB/s (Q4_0/Q8_0 GEMV microbenchmark) + % HBM roofline, B200 vs host CPU"
GEMV_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]      # n_out x n_in


def dequant_np(gtype: int, raw, n_in: int, n_out: int):
    """Q4_0 / Q8_0 blocks -> float64 [n_out, n_in] (the ggml rules: Q4_0
    y[l] = (lo - 8) d, y[l + 16] = (hi - 8) d; Q8_0 y = d q)."""
    import numpy as np
    from distcomp_b200 import gguf as G
    bb = 18 if gtype == G.Q4_0 else 34
    blk = raw.reshape(-1, bb)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float64)
    if gtype == G.Q4_0:
        q = blk[:, 2:]
        v = np.concatenate([(q & 0xF).astype(np.int32) - 8, (q >> 4).astype(np.int32) - 8], axis=1)
    else:
        v = blk[:, 2:].view(np.int8).astype(np.int32)
    return (v * d).reshape(n_out, n_in)


def gemv_arm(args, local):
    """The quantised-matvec microbenchmark: Q4_0 and Q8_0 at 4096x4096,
    14336x4096 and 4096x14336 (n_out x n_in), codes uniform over each
    format's range, fp16 scales |N(0,0.02)|/max_code, x ~ N(0,1).  Each case
    rotates over enough device copies of its matrix to exceed the L2 three
    times, so every launch streams its weights from HBM; CUDA events around
    `rounds` replays of a graph of one launch per copy.  GB/s = (weight
    bytes as stored + x + y) / time per launch.  Every case's output is
    checked against a float64 numpy matvec of the dequantised blocks with
    the tests' bound |y - ref| <= 1e-4 |ref| + 1e-6 ||w_o|| ||x||.  Each
    case is also measured streamed: the copies as consecutive GEMV phases of
    one persistent launch (ecu_matvec_stream_bench), how the decode step
    consumes its matrices, reported under "streamed"."""
    import math
    import numpy as np
    from distcomp_b200 import engine as E
    from distcomp_b200 import gguf as G
    from distcomp_b200 import synth
    peak, peak_kind = peaks()
    l2 = 126e6
    cases = []
    clocks = ClockSampler(local)
    clocks.start()
    l0 = E.kernel_launches()
    for gt in (G.Q4_0, G.Q8_0):
        for n_out, n_in in GEMV_SHAPES:
            if args.gemv_case and args.gemv_case != f"{G.TYPE_NAMES[gt]}:{n_out}x{n_in}":
                continue
            rng = np.random.default_rng([n_out, n_in, gt])
            raw = synth.microbench_blocks(rng, gt, n_in, n_out)
            x = rng.standard_normal(n_in).astype(np.float32)
            wbytes = raw.size
            copies = max(2, math.ceil(3 * l2 / wbytes))
            rounds = max(4, math.ceil(args.steps * 8 / copies))
            ms, y = E.matvec_bench(gt, raw, n_in, n_out, x, copies, rounds, device=local)
            W = dequant_np(gt, raw, n_in, n_out)
            ref = W @ x.astype(np.float64)
            bound = 1e-4 * np.abs(ref) + 1e-6 * np.linalg.norm(W, axis=1) * np.linalg.norm(x.astype(np.float64))
            err = np.abs(y.astype(np.float64) - ref)
            algo = wbytes + 4 * n_in + 4 * n_out
            gbs = algo / (ms / 1e3) / 1e9
            # the same copies streamed through the persistent step's GEMV
            # phases (one cooperative launch per round over every copy)
            ms_s, y_s = E.matvec_stream_bench(gt, raw, n_in, n_out, x, copies, rounds, device=local)
            err_s = np.abs(y_s.astype(np.float64) - ref)
            gbs_s = algo / (ms_s / 1e3) / 1e9
            cases.append({"type": G.TYPE_NAMES[gt], "shape": f"{n_out}x{n_in}", "weight_bytes": int(wbytes),
                          "us_per_launch": round(ms * 1e3, 3), "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4), "frac_of_8tbs_nominal": round(gbs / 8000, 4),
                          "copies": copies, "launches": copies * rounds,
                          "max_err_over_bound": round(float(np.max(err / bound)), 4),
                          "within_tolerance": bool(np.all(err <= bound)),
                          "streamed": {"us_per_matvec": round(ms_s * 1e3, 3), "gbs": round(gbs_s, 1),
                                       "frac": round(gbs_s / peak, 4), "launches": rounds,
                                       "max_err_over_bound": round(float(np.max(err_s / bound)), 4),
                                       "within_tolerance": bool(np.all(err_s <= bound))}})
            del W
    launches = E.kernel_launches() - l0
    clk = clocks.stop()
    gm = math.exp(sum(math.log(c["gbs"]) for c in cases) / len(cases))
    gm_s = math.exp(sum(math.log(c["streamed"]["gbs"]) for c in cases) / len(cases))
    line = {
        "metric": GEMV_METRIC, "value": round(gm, 1), "unit": "GB/s (geometric mean over the 6 cases)",
        "n_gpus": 1, "steps": args.steps, "warmup": 2, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_0/q8_0 codes x int8 digit planes, fp32 accumulate",
        "data": "synthetic: codes uniform over each format's range, fp16 scales |N(0,0.02)|/max_code, x ~ N(0,1)",
        "config": {"workload": "quantised matvec y = W x, Q4_0 and Q8_0 at 4096x4096, 14336x4096, 4096x14336 "
                               "(n_out x n_in)",
                   "l2": "each case rotates over >= 3 x L2 of device copies of its matrix"},
        "peak_gbs": peak, "peak_kind": peak_kind, "cases": cases, "gpu_launches": int(launches), "clocks": clk,
        "streamed": {"value": round(gm_s, 1), "frac": round(gm_s / peak, 4),
                     "how": "every copy one GEMV phase of one persistent cooperative launch (how the decode step "
                            "streams its matrices); time per matvec = launch time / copies"},
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_gemv(cases)
    print(json.dumps(line), flush=True)
    return 0


def cpu_reference_gemv(cases):
    """The reference's own matvec (src/engine.c:348-357 over its thread pool,
    compiled from its sources into oracle/_ref/libdcref_mv.so) on the host
    cores, each case timed for about 2 s."""
    import ctypes as C
    import numpy as np
    from distcomp_b200 import gguf as G
    from distcomp_b200 import synth
    so = ROOT / "oracle" / "_ref" / "libdcref_mv.so"
    if not so.exists():
        return {"unavailable": "oracle/_ref/libdcref_mv.so not built"}
    L = C.CDLL(str(so))
    L.refmv_matvec.restype = C.c_int
    L.refmv_matvec.argtypes = [C.c_uint, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    thr = min(64, os.cpu_count() or 1)
    L.refmv_set_threads(thr)
    out = []
    names = {v: k for k, v in G.TYPE_NAMES.items()}
    for c in cases:
        gt = names[c["type"]]
        n_out, n_in = (int(v) for v in c["shape"].split("x"))
        rng = np.random.default_rng([n_out, n_in, gt])
        raw = synth.microbench_blocks(rng, gt, n_in, n_out)
        x = rng.standard_normal(n_in).astype(np.float32)
        y = np.empty(n_out, np.float32)
        L.refmv_matvec(gt, raw.ctypes.data, raw.size, n_in, n_out, x.ctypes.data, y.ctypes.data)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 2.0:
            L.refmv_matvec(gt, raw.ctypes.data, raw.size, n_in, n_out, x.ctypes.data, y.ctypes.data)
            n += 1
        dt = (time.perf_counter() - t0) / n
        out.append({"type": c["type"], "shape": c["shape"],
                    "gbs": round((raw.size + 4 * n_in + 4 * n_out) / dt / 1e9, 3), "ms": round(dt * 1e3, 3)})
    return {"kind": "reference", "cores": thr, "cases": out,
            "value": round(float(np.exp(np.mean([np.log(o["gbs"]) for o in out]))), 3), "unit": "GB/s",
            "sample": "each case's matvec repeated for ~2 s (weights L2/LLC-resident only for the small cases)"}


def reference_arm(args, rank, world, local):
    if rank != 0:
        return 0
    from distcomp_b200 import synth
    spec = synth.spec(CONFIG)
    buf = build_model_gpu(spec, args.seed, local)
    budget = max(30.0, min(240.0, 2.0 * args.steps))
    v, n, thr, kind = cpu_reference_tokens_per_s(buf, spec, budget, max(1, args.steps))
    line = {
        "metric": METRIC, "value": round(v, 4), "unit": "tokens/s", "n_gpus": world, "steps": n,
        "warmup": 1, "ms_per_step": round(1e3 / v, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (dequantised per block)", "impl": "reference",
        "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_0/Q8_0, random prompt",
        "config": {"workload": "llama3-8b-shape Q4_0 decode, batch 1 (dim 4096, 32 layers, 32/8 heads, "
                               "ffn 14336, vocab 128256, theta 5e5)"},
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": thr, "kind": kind,
                         "sample": f"{n} decode tokens (bounded to {budget:.0f} s) from position 1, "
                                   "reference engine.c/gguf.c/thread.c compiled from its sources"},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if "WORLD_SIZE" not in os.environ:
        world = 1 if args.gpus == 1 else args.gpus
        if world > 1:
            raise SystemExit("launch N>1 with torch.distributed.run (one process per GPU)")
    if args.impl == "reference":
        return reference_arm(args, rank, world, local)
    if args.mode == "gemv":
        return gemv_arm(args, local) if rank == 0 else 0
    return our_arm(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
