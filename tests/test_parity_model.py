"""End-to-end pin of the C restatement to the reference build on the parity model (CPU only).

The benchmark model's random weights drive the residual stream into one direction, so its
greedy stream hardly depends on the input; the parity model (same layout and tensor types,
balanced Q4_K mins, smaller per-layer block scales; mcpm.synth.write_model) gives input-
dependent logits and a greedy stream of 63 distinct tokens in 65.  Golden vectors come from
the reference build at one OpenMP thread, where it is deterministic, on BASELINE config 0's
shape: a 128-id prompt, then 64 greedy tokens (tests/golden/make_golden.py --wc).

At more than one thread the reference does not repeat itself: the OpenMP reduction of its
RMSNorm sum (src/ops/ops.cpp:680-685) changes in the last bits from run to run, and the int8
re-quantisation in front of every GEMV (ops.cpp:676-723, ops_avx2.cpp:85-144) turns that into
logit differences of several units after 42 layers.  The fixture records that spread from two
4-thread runs; a position whose 1-thread top-2 margin exceeds it is "decidable".  An
implementation with other (equally valid) rounding -- this project's canonical order -- must
therefore: give the reference's argmax at every decidable position, and stay within the
reference's own spread on average.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

import oracle as O

PARITY_DSCALE = 0.04
N_CHECK = 24   # teacher-forced positions run on the CPU (the GPU test covers all 192)


@pytest.fixture(scope="module")
def parity():
    g = np.load(os.path.join(GOLDEN, "reference_decode_wc.npz"))
    v = json.load(open(os.path.join(GOLDEN, "reference_variability_wc.json")))
    r = np.load(os.path.join(GOLDEN, "restatement_decode_wc.npz"))
    return g, v, r


@pytest.fixture(scope="module")
def parity_model_path():
    from mcpm import synth
    return synth.ensure_model("q4_k_m", 0, dscale=PARITY_DSCALE)


def test_parity_fixture_is_informative(parity):
    g, v, _ = parity
    assert len(g["prompt"]) == 128 and len(g["tokens"]) == 128 + 64
    assert v["distinct_generated_tokens"] >= 10
    assert sum(v["decidable"]) >= 100
    assert np.isfinite(g["top_val"]).all() and np.isfinite(g["full_last_prompt"]).all()


def test_parity_model_file_matches_fixture(parity, parity_model_path):
    _, v, _ = parity
    man = json.load(open(parity_model_path + ".json"))
    assert man["content_digest"] == v["model_manifest"]["content_digest"]


def test_restatement_vs_reference_on_parity_model(parity, parity_model_path, oracle):
    g, v, r = parity
    m = O.OracleModel(oracle, parity_model_path, N_CHECK + 1)
    lg = np.zeros(130560, np.float32)
    am, top = [], []
    for pos in range(N_CHECK):
        am.append(m.forward(int(g["prompt"][pos]), pos, lg))
        top.append(lg[g["top_idx"][pos]].copy())
    am, top = np.array(am), np.array(top)
    # the restatement itself has not moved (the GPU test pins the CUDA engine to this fixture)
    assert np.array_equal(top.view(np.uint32), r["top_val"][:N_CHECK].view(np.uint32))
    assert np.array_equal(am, r["argmax"][:N_CHECK])
    dec = np.array(v["decidable"][:N_CHECK])
    assert np.array_equal(am[dec], g["tokens"][:N_CHECK][dec])
    assert np.abs(top - g["top_val"][:N_CHECK]).mean() <= 1.25 * max(v["mean_abs_top32_4_vs_1"])


def test_restatement_fixture_vs_reference_all_positions(parity):
    """The committed teacher-forced restatement run (all 192 positions) against the reference."""
    g, v, r = parity
    dec = np.array(v["decidable"])
    assert np.array_equal(r["argmax"][dec], g["tokens"][dec])
    assert np.abs(r["top_val"] - g["top_val"]).mean() <= 1.25 * max(v["mean_abs_top32_4_vs_1"])
    # as good as the reference against itself: at least as many argmax agreements
    assert int(np.sum(r["argmax"] == g["tokens"])) >= min(v["argmax_agree_4_vs_1"]) - 4


def test_block_order_fixture_vs_reference_all_positions(parity):
    """The committed teacher-forced restatement run in the block order (the engine's default GEMV
    order; all 192 positions) against the reference, at the same bar as the eight-lane order."""
    g, v, _ = parity
    r = np.load(os.path.join(GOLDEN, "restatement_decode_wc_block.npz"))
    dec = np.array(v["decidable"])
    assert np.array_equal(r["argmax"][dec], g["tokens"][dec])
    assert np.abs(r["top_val"] - g["top_val"]).mean() <= 1.25 * max(v["mean_abs_top32_4_vs_1"])
    assert int(np.sum(r["argmax"] == g["tokens"])) >= min(v["argmax_agree_4_vs_1"]) - 4


def test_batch_order_restatement_vs_reference_on_parity_model(parity, parity_model_path, oracle):
    """The batched path's fp32 order (exact block sums, one fma per block, groups of four
    blocks: the tcgen05 batched GEMM and prefill) against the reference build: the reference's
    argmax at every decidable position and logits within its own thread-count spread."""
    g, v, _ = parity
    m = O.OracleModel(oracle, parity_model_path, N_CHECK + 1)
    m.set_order(O.Oracle.ORDER_BATCH)
    lg = np.zeros(130560, np.float32)
    am, top = [], []
    for pos in range(N_CHECK):
        am.append(m.forward(int(g["prompt"][pos]), pos, lg))
        top.append(lg[g["top_idx"][pos]].copy())
    am, top = np.array(am), np.array(top)
    # the committed block-order fixture is this restatement's own run (the GPU test pins the engine to it)
    rb = np.load(os.path.join(GOLDEN, "restatement_decode_wc_block.npz"))
    assert np.array_equal(top.view(np.uint32), rb["top_val"][:N_CHECK].view(np.uint32))
    assert np.array_equal(am, rb["argmax"][:N_CHECK])
    dec = np.array(v["decidable"][:N_CHECK])
    assert np.array_equal(am[dec], g["tokens"][:N_CHECK][dec])
    assert np.abs(top - g["top_val"][:N_CHECK]).mean() <= 1.25 * max(v["mean_abs_top32_4_vs_1"])
    m.close()
