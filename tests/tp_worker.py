"""One rank of a tensor-parallel decode run, started by tests/test_gpu_tp.py in its own
process (one GPU per rank).  The ranks exchange their setup data over a gloo process group
on 127.0.0.1, decode the same prompt and greedy continuation, and each writes its tokens and
its vocabulary slice of the logits to out_dir/rank<r>.npz."""
import datetime
import os

import numpy as np


def run_rank(rank, world, comm, path, prompt, n_gen, max_seq, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    from mcpm.tp import TPEngine
    e = TPEngine(rank, rank, world, max_seq, comm)
    try:
        e.load(path)
        e.connect(dist)
        toks, logs = [], []
        for p, t in enumerate(prompt):
            tok, lg = e.forward(int(t), p)
            toks.append(tok)
            logs.append(lg)
        for i in range(n_gen):
            tok, lg = e.forward(-1, len(prompt) + i)
            toks.append(tok)
            logs.append(lg)
        chained = e.read_tokens(0, len(prompt) + n_gen)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), tokens=np.array(toks, np.int32),
                 logits=np.stack(logs), lo=e.vocab_lo, hi=e.vocab_hi, log=chained)
    finally:
        dist.barrier()   # no rank frees its receive buffer while a peer may still store into it
        e.close()
        dist.destroy_process_group()
