"""Host-side multi-rank logic of bench.py on CPU: world_size-2 `gloo` process groups.

Batch-1 decode runs as independent replicas (one sequence per GPU, no collective in the data
path); the only cross-rank steps are the start barrier and the max-over-ranks reduction of
the device timings, and the reference arm runs on rank 0 alone.
"""
import json
import os
import socket
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, values, out_dir):
    import torch.distributed as dist
    sys.path.insert(0, REPO)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dist.barrier()
    got = bench.max_over_ranks(values[rank], dist, device="cpu")
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump({"max": got}, f)
    dist.barrier()
    dist.destroy_process_group()


def test_max_over_ranks_gloo(tmp_path):
    import torch.multiprocessing as mp
    values = [3.25, 7.5]
    mp.spawn(_worker, args=(2, _free_port(), values, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert json.load(open(tmp_path / f"r{r}.json"))["max"] == 7.5


def test_max_over_ranks_single_process():
    sys.path.insert(0, REPO)
    import bench
    assert bench.max_over_ranks(1.5, None, device="cpu") == 1.5


def test_reference_arm_runs_on_rank0_only(capsys):
    """Under torchrun the reference CPU arm prints its line on rank 0 and nothing elsewhere."""
    sys.path.insert(0, REPO)
    import bench

    class A:
        gpus, steps, warmup = 2, 4, 3
    bench.run_reference(A, rank=1, world=2)
    assert capsys.readouterr().out == ""
