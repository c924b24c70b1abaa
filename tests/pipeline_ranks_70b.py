"""Rank program for the two-GPU 70B-shape pipeline test (run under
torch.distributed.run).

Two layers of the 70B shape (n_embd 8192, 64/8 heads, FFN 28672, Q4_K
layers, Q8_0 embedding and head), one layer per GPU: the prompt goes through
the two stages as one batch each (ecu_prefill_rows, the rows over NCCL),
then greedy decoding with the steps linked over NVLink (each step writes its
output into the other GPU's step).  Rank 1 (the head) compares the tokens
with the oracle's (the CPU restatement of the reference engine, fed the same
prompt token by token) and with a FULL context on its own GPU (ecu_prefill,
then per-token steps: bit for bit), and writes <outdir>/ok when both match.
"""
import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
from distcomp_b200 import engine as E          # noqa: E402
from distcomp_b200 import pipeline as P        # noqa: E402
from distcomp_b200 import synth                # noqa: E402


def main():
    out = Path(sys.argv[1])
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=300))
    ok = True
    try:
        s = synth.spec("l70-1", n_layer=2)
        first, last = [(0, 0), (1, 1)][rank]
        # each rank generates only its stage's tensors (the same bytes as
        # the whole model's), as the 70B bench does
        only = synth.stage_tensors(s, first, last, rank == 0, rank == world - 1)
        m = E.GgufModel(synth.build_model(s, seed=0, only=only))
        n_prompt, n_gen, n_ctx = 8, 5, s.n_ctx
        prompt = synth.prompt_tokens(n_prompt, s.n_vocab, seed=21)
        st = P.GpuStage(m, rank, world, first, last, s.n_layer, 1, n_ctx, local)
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

        tok = P.prefill_local({rank: st}, 0, prompt, send_rows, recv_rows, share_token)
        if st.has_head:
            st.record_tokens(n_prompt + n_gen)
        torch.cuda.synchronize(local)
        dist.barrier()
        S = P.Schedule(world, 1, n_gen - 1, n_prompt=0, first_step=n_prompt)
        P.run_ticks(S, {rank: st}, P.LinkedExchanger())
        st.sync()
        dist.barrier()             # no step writes into the other GPU any more
        if st.has_head:
            got = [tok] + [int(t) for t in st.history[0, n_prompt: n_prompt + n_gen - 1].cpu().tolist()]
            got_logits = st.chains[0][0].logits()
        st.close()
        if rank == world - 1:
            import oracle
            oracle.build(ref=False)
            full_buf = synth.build_model(s, seed=0)
            want = oracle.greedy(oracle.get("port"), full_buf, prompt, n_gen)
            fm = E.GgufModel(full_buf)
            c = E.LlmCtx(fm, E.STAGE_FULL, n_ctx=n_ctx, device=local)
            full = [c.prefill(prompt)]
            o = np.zeros(s.n_embd + 1, dtype=np.float32)
            while len(full) < n_gen:
                assert c.forward(full[-1], o) == 0
                full.append(int(o[s.n_embd]))
            full_logits = c.logits()
            c.close()
            same_logits = np.array_equal(got_logits.view(np.uint32), full_logits.view(np.uint32))
            print(f"pipeline {got}\nfull     {full}\noracle   {want}\nlogits bit-equal {same_logits}", flush=True)
            ok = got == want and got == full and same_logits
            if ok:
                (out / "ok").write_text("ok\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
