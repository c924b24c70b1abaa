"""Rank program for the tensor-parallel test (run under torch.distributed.run,
one GPU per rank).

Each rank builds the same seeded model and opens its tensor-parallel FULL
context; the ranks greedy-decode one prompt together.  Each rank then opens
a one-GPU FULL context on its own GPU and decodes the same prompt: the
tokens must be identical and the rank's slice of the final logits equal
bit for bit (no projection splits its input, so tensor parallelism changes
no arithmetic).  Writes <outdir>/ok.<rank> when everything matches.
"""
import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from distcomp_b200 import engine as E              # noqa: E402
from distcomp_b200 import synth                    # noqa: E402
from distcomp_b200 import tensor_parallel as TP    # noqa: E402


def main():
    out = Path(sys.argv[1])
    key = sys.argv[2] if len(sys.argv) > 2 else "mini-q4"
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=120))
    ok = True
    try:
        s = synth.spec(key, n_layer=4)
        m = E.GgufModel(synth.build_model(s, seed=0))
        n_ctx, n_gen = 96, 64
        prompt = synth.prompt_tokens(7, s.n_vocab, seed=3)
        ctx = TP.open_rank(m, rank, world, n_ctx, local)
        print(f"rank {rank}: {ctx.path()} vocab [{ctx.vocab0}, {ctx.vocab1})", flush=True)
        got = ctx.generate(prompt, n_gen)
        got_logits = ctx.logits()
        v0, v1 = ctx.vocab0, ctx.vocab1
        ctx.sync()
        dist.barrier()
        ctx.close()
        one = E.LlmCtx(m, E.STAGE_FULL, n_ctx=n_ctx, device=local)
        want = one.generate(prompt, n_gen)
        want_logits = one.logits()[v0:v1]
        one.close()
        same_tok = got == want
        same_logits = np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
        print(f"rank {rank}: tokens {'equal' if same_tok else 'DIFFER'}, logits slice "
              f"{'bit-equal' if same_logits else 'DIFFER'}", flush=True)
        if not same_tok:
            print("tp  ", got, "\none ", want, flush=True)
        ok = same_tok and same_logits
        if ok:
            (out / f"ok.{rank}").write_text("ok\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
