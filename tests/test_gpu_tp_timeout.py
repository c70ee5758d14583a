"""Failure detection of the tensor-parallel exchange (the device-side waits for another rank's
partial sums, include/mcpm.h mcpm_tp_config::peer_wait_us).

The failure is made on the host: rank 1 connects and then takes no step, so the flag rank 0
waits for is never written and no GPU faults or hangs.  Rank 0's step must end with
MCPM_TIMEOUT after about one bound (once one wait has given up, the step's later waits give up
at once), the next step must fail the same way, and mcpm_tp_reset must succeed.  With one GPU
per rank, both ranks then reset, meet at a host barrier and step together again, and their
greedy tokens agree."""
import json
import os

import pytest

pytestmark = pytest.mark.gpu

WAIT_US = 50_000   # 50 ms


def _run(cuda, q8_path, tmp_path, recover):
    import torch.multiprocessing as mp
    import tp_worker
    from test_gpu_tp import _free_port
    mp.spawn(tp_worker.run_timeout_rank, args=(2, q8_path, WAIT_US, _free_port(), str(tmp_path), recover), nprocs=2,
             join=True)
    return [json.load(open(os.path.join(tmp_path, f"timeout{r}.json"))) for r in range(2)]


@pytest.fixture(scope="module")
def q8_path():
    from mcpm import synth
    return synth.ensure_model("q8_0", 0)


def test_peer_wait_times_out_and_reset_succeeds(cuda, q8_path, tmp_path):
    from mcpm import engine as E
    r0, _ = _run(cuda, q8_path, tmp_path, recover=False)
    assert r0["step0"] == E.TIMEOUT and r0["step1"] == E.TIMEOUT
    # one bound (50 ms) plus the kernels that then give up at once; far below the 5 s default
    assert r0["step0_s"] < 1.5 and r0["step1_s"] < 1.5
    assert r0["reset"] == "ok"


def test_ranks_recover_after_timeout(cuda, q8_path, tmp_path):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (ranks that wait on each other never share one GPU)")
    from mcpm import engine as E
    r0, r1 = _run(cuda, q8_path, tmp_path, recover=True)
    assert r0["step0"] == E.TIMEOUT
    assert r0["recovered_tokens"] == r1["recovered_tokens"]
