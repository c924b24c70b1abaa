"""Rank program for the two-GPU pipeline test (run under torch.distributed.run).

Each rank builds the same seeded model, holds its stage of a 2-way split and
decodes three interleaved sequences over NCCL; the last rank compares every
sequence's greedy tokens with a FULL context on its own GPU and writes
<outdir>/ok when they all match.
"""
import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from distcomp_b200 import engine as E          # noqa: E402
from distcomp_b200 import pipeline as P        # noqa: E402
from distcomp_b200 import synth                # noqa: E402


def main():
    out = Path(sys.argv[1])
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=120))
    ok = True
    try:
        s = synth.spec("mini-q4", n_layer=4)
        m = E.GgufModel(synth.build_model(s, seed=0))
        n_seq, n_prompt, n_gen, n_ctx = 3, 5, 12, 64
        prompts = [synth.prompt_tokens(n_prompt, s.n_vocab, seed=11 + q) for q in range(n_seq)]
        a, b = P.split_stages(s.n_layer, world)[rank]
        st = P.GpuStage(m, rank, world, a, b, s.n_layer, n_seq, n_ctx, local, prompts=prompts)
        n_steps = n_prompt + n_gen - 1
        if st.has_head:
            st.record_tokens(n_steps)
        dist.barrier()
        S = P.Schedule(world, n_seq, n_steps, n_prompt=n_prompt)
        P.run_ticks(S, {rank: st}, P.DistExchanger(rank))
        st.sync()
        if st.has_head:
            hist = st.history.cpu().tolist()
            for q in range(n_seq):
                c = E.LlmCtx(m, E.STAGE_FULL, n_ctx=n_ctx, device=local)
                want = c.generate(prompts[q], n_gen)
                c.close()
                got = hist[q][n_prompt - 1:]
                print(f"seq {q}: pipeline {got} full {want}", flush=True)
                ok = ok and got == want
            if ok:
                (out / "ok").write_text("ok\n")
        st.close()
        dist.barrier()

        # linked: the prompts as one batch per stage (rows over NCCL), then
        # every step hands its output to the other GPU's step itself
        st = P.GpuStage(m, rank, world, a, b, s.n_layer, n_seq, n_ctx, local, prompts=prompts)
        P.link_dist(st, rank, world)
        dev = torch.device("cuda", local)

        def send_rows(r, rows):
            dist.send(rows, r + 1)

        def recv_rows(r, rows):
            dist.recv(rows, r - 1)

        def share_token(tok):
            t = torch.tensor([tok if rank == world - 1 else 0], dtype=torch.int64, device=dev)
            dist.broadcast(t, world - 1)
            return int(t.item())

        firsts = [P.prefill_local({rank: st}, q, prompts[q], send_rows, recv_rows, share_token) for q in range(n_seq)]
        n_dec = n_gen - 1
        if st.has_head:
            st.record_tokens(n_prompt + n_dec)
        dist.barrier()
        S = P.Schedule(world, n_seq, n_dec, n_prompt=0, first_step=n_prompt)
        P.run_ticks(S, {rank: st}, P.LinkedExchanger())
        st.sync()
        if st.has_head:
            hist = st.history.cpu().tolist()
            ok2 = True
            for q in range(n_seq):
                c = E.LlmCtx(m, E.STAGE_FULL, n_ctx=n_ctx, device=local)
                want = [c.prefill(prompts[q])]
                o = torch.zeros(s.n_embd + 1, dtype=torch.float32).numpy()
                while len(want) < n_gen:
                    assert c.forward(want[-1], o) == 0
                    want.append(int(o[s.n_embd]))
                c.close()
                got = [firsts[q]] + hist[q][n_prompt: n_prompt + n_dec]
                print(f"linked seq {q}: pipeline {got} full {want}", flush=True)
                ok2 = ok2 and got == want
            if ok2:
                (out / "ok_linked").write_text("ok\n")
            ok = ok and ok2
        dist.barrier()             # no step writes into another rank's memory any more
        st.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
