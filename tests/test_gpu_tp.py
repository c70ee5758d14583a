"""Tensor-parallel all-Q8_0 decode against the C restatement's all-Q8_0 forward.

One GPU: the same operations in the same order as the restatement, so logits and tokens are
bit-exact.  N GPUs (one process each; skipped when fewer GPUs are visible): o_proj and down
are split by input columns, so their partial sums are added across ranks in another order;
logits within 2e-3 absolute and 1e-3 relative, greedy tokens identical."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def q8_path():
    from mcpm import synth
    return synth.ensure_model("q8_0", 0)


def oracle_run(oracle, path, prompt, n_gen, max_seq):
    import oracle as O
    om = O.OracleModel(oracle, path, max_seq)
    toks, logs = [], []
    ref = np.zeros(130560, np.float32)
    t = None
    try:
        for p in range(len(prompt) + n_gen):
            t = int(prompt[p]) if p < len(prompt) else t
            t = om.forward(t, p, ref)
            toks.append(t)
            logs.append(ref.copy())
    finally:
        om.close()
    return np.array(toks), np.stack(logs)


def test_tp1_bitexact(cuda, oracle, q8_path):
    from mcpm.tp import TPEngine
    prompt = [5, 77, 1234, 130559]
    n_gen = 3
    want_t, want_l = oracle_run(oracle, q8_path, prompt, n_gen, 16)
    e = TPEngine(0, 0, 1, 16)
    try:
        e.load(q8_path)
        e.connect()
        assert (e.vocab_lo, e.vocab_hi) == (0, 130560)
        for p in range(len(prompt) + n_gen):
            tok, lg = e.forward(prompt[p] if p < len(prompt) else -1, p)
            diff = np.sum(lg.view(np.uint32) != want_l[p].view(np.uint32))
            assert diff == 0, f"pos {p}: {diff} logits differ, max {np.max(np.abs(lg - want_l[p]))}"
            assert tok == want_t[p]
        assert list(e.read_tokens(0, len(prompt) + n_gen)) == list(want_t)
        # chained generation on the device continues the same greedy stream
        e.reset()
        for p, t in enumerate(prompt):
            e.forward(t, p, logits=False)
        e.generate_async(n_gen - 1)
        e.sync()
        assert list(e.read_tokens(len(prompt), n_gen - 1)) == list(want_t[len(prompt):len(prompt) + n_gen - 1])
    finally:
        e.close()


def test_tp_rejects_other_mixes(cuda, model_path):
    from mcpm import engine as E
    from mcpm.tp import TPEngine
    e = TPEngine(0, 0, 1, 16)
    try:
        with pytest.raises(E.MCPMError) as ei:
            e.load(model_path)   # Q4_K_M mix
        assert ei.value.status == E.UNSUPPORTED_TYPE
    finally:
        e.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,comm", [(2, "p2p"), (2, "nccl"), (4, "p2p"), (8, "p2p"), (8, "nccl")])
def test_tp_multi_gpu(cuda, oracle, q8_path, tmp_path, world, comm):
    if cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    import tp_worker
    prompt = [11, 4242, 99999, 7]
    n_gen = 4
    mp.spawn(tp_worker.run_rank, args=(world, comm, q8_path, prompt, n_gen, 16, _free_port(), str(tmp_path)),
             nprocs=world, join=True)
    want_t, want_l = oracle_run(oracle, q8_path, prompt, n_gen, 16)
    parts = [np.load(os.path.join(tmp_path, f"rank{r}.npz")) for r in range(world)]
    lg = np.concatenate([p["logits"] for p in parts], axis=1)
    assert [int(p["hi"]) for p in parts][-1] == 130560
    for p in parts:
        assert list(p["tokens"]) == list(want_t)
        assert list(p["log"]) == list(want_t)
    err = np.abs(lg - want_l)
    assert np.all(err <= ATOL + RTOL * np.abs(want_l)), f"max abs err {err.max()}"
