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


def run_timeout_rank(rank, world, path, wait_us, port, out_dir, recover):
    """Failure detection of the tensor-parallel exchange, with the failure made on the host:
    rank 1 connects and then takes no step, so rank 0's waits for its partial sums run out.
    Rank 0 records the status and duration of two steps and of mcpm_tp_reset.  With `recover`
    (one GPU per rank), every rank then resets and both step together again."""
    import json
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    from mcpm import engine as E
    from mcpm.tp import TPEngine
    device = rank if recover else 0
    e = TPEngine(device, rank, world, 32, "p2p", peer_wait_us=wait_us)
    out = {}
    try:
        e.load(path)
        e.connect(dist)
        dist.barrier()
        if rank == 0:
            for i in range(2):
                t0 = time.perf_counter()
                try:
                    e.forward(11, 0, logits=False)
                    out[f"step{i}"] = "ok"
                except E.MCPMError as ex:
                    out[f"step{i}"] = ex.status
                out[f"step{i}_s"] = time.perf_counter() - t0
            e.reset()
            out["reset"] = "ok"
        dist.barrier()   # rank 1 took no step while rank 0 waited
        if recover:
            if rank != 0:
                e.reset()
            dist.barrier()   # every rank has reset before any rank steps again
            toks = [e.forward(t, p, logits=False)[0] for p, t in enumerate([11, 4242, 7])]
            out["recovered_tokens"] = [int(t) for t in toks]
        with open(os.path.join(out_dir, f"timeout{rank}.json"), "w") as f:
            json.dump(out, f)
    finally:
        dist.barrier()   # no rank frees its receive buffer while a peer may still store into it
        e.close()
        dist.destroy_process_group()
