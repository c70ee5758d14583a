"""Host-side logic of the tensor-parallel engine, without a GPU: argument checks of the C ABI
and the setup exchange of `TPEngine.connect` between two gloo ranks on CPU."""
import ctypes as C
import datetime
import os
import socket

import pytest


def test_tp_create_rejects_bad_config():
    from mcpm import engine as E
    from mcpm.tp import mcpm_tp_config
    lib = E.load_library()
    h = C.c_void_p()
    for dev, rank, world, max_seq, comm in [(0, 0, 3, 16, 0), (0, 2, 2, 16, 0), (0, -1, 2, 16, 0),
                                            (0, 0, 1, 0, 0), (0, 0, 1, 1 << 20, 0), (0, 0, 2, 16, 7)]:
        cfg = mcpm_tp_config(dev, rank, world, max_seq, comm, 0)
        assert lib.mcpm_tp_create(C.byref(cfg), C.byref(h)) == E.BAD_ARG, (rank, world, max_seq, comm)
    assert lib.mcpm_tp_create(None, C.byref(h)) == E.BAD_ARG
    assert lib.mcpm_tp_forward(None, 0, 0, None, None) == E.BAD_ARG
    assert lib.mcpm_tp_nccl_id(None) == E.BAD_ARG


def test_tp_bytes_per_step_partition():
    """Per-GPU bytes of the bench's roofline: the shards of all ranks add up to the whole
    model plus the replicated pieces."""
    import bench
    from mcpm import spec
    one = bench.tp_bytes_per_step(1, 0)
    eight = bench.tp_bytes_per_step(8, 0)
    rb = spec.N_EMBD // 32 * 34
    # KV rows: 8 ranks recompute the 2 KV heads 4 times over
    extra_kv_rows = spec.N_LAYER * 2 * (8 * 128 - 256) * rb
    replicated = 7 * (spec.N_LAYER * 2 * 4 * spec.N_EMBD + 4 * spec.N_EMBD + rb)
    assert 8 * eight == one + extra_kv_rows + replicated


class _FakeEngine:
    def __init__(self, rank, world, comm):
        self.rank, self.world, self.comm = rank, world, comm
        self.got = None

    def ipc_handle(self):
        return bytes([self.rank + 1]) * 64

    def connect_with(self, nccl_id128=None, handles=None):
        self.got = (nccl_id128, handles)


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from mcpm import tp
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    tp.nccl_id = lambda: b"N" * 128   # the id itself comes from libnccl; only its distribution is tested
    res = []
    for comm in ("p2p", "nccl"):
        f = _FakeEngine(rank, world, comm)
        tp.TPEngine.connect(f, dist)
        res.append(f.got)
    dist.destroy_process_group()
    import pickle
    with open(os.path.join(out, f"r{rank}.pkl"), "wb") as fh:
        pickle.dump(res, fh)


def test_connect_exchange_two_gloo_ranks(tmp_path):
    import pickle
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        with open(os.path.join(tmp_path, f"r{r}.pkl"), "rb") as fh:
            p2p, nccl = pickle.load(fh)
        assert p2p == (None, [b"\x01" * 64, b"\x02" * 64])   # every rank's handle, in rank order
        assert nccl == (b"N" * 128, None)                     # rank 0's id on every rank
