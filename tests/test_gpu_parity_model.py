"""The CUDA engine on the parity model against the reference build's goldens (BASELINE
config 0's shape: a 128-id prompt, then 64 greedy tokens), teacher-forced with the
reference's own tokens.  See test_parity_model.py for the model and for the reference's own
run-to-run spread, which bounds what any implementation with other rounding can match.

Checks, over all 192 positions, in both GEMV orders of the engine (the default block order
against the restatement's ORC_ORDER_BATCH fixture, MCPM_GEMM_MMA against the eight-lane one):
  * the engine equals the C restatement bit for bit (logits at the reference's top-32 indices
    and the argmax), so every parity statement about the restatement holds for the engine;
  * at every position where the reference decides its argmax against its own spread, the
    engine's argmax is the reference's;
  * the engine's logits stay within the reference's own average spread.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

PARITY_DSCALE = 0.04


@pytest.mark.parametrize("order", ["block", "avx2"])
def test_engine_vs_reference_on_parity_model(cuda, order):
    from mcpm import engine as E, synth
    g = np.load(os.path.join(GOLDEN, "reference_decode_wc.npz"))
    v = json.load(open(os.path.join(GOLDEN, "reference_variability_wc.json")))
    r = np.load(os.path.join(GOLDEN, "restatement_decode_wc_block.npz" if order == "block" else
                             "restatement_decode_wc.npz"))
    path = synth.ensure_model("q4_k_m", 0, dscale=PARITY_DSCALE)
    assert json.load(open(path + ".json"))["content_digest"] == v["model_manifest"]["content_digest"]
    toks, prompt = g["tokens"], g["prompt"]
    n = len(toks)
    inputs = list(prompt) + list(toks[len(prompt) - 1:n - 1])
    eng = E.MiniCPM5Engine(device=0, max_seq=n + 8, batch_gemm=E.GEMM_TCGEN05 if order == "block" else E.GEMM_MMA)
    assert eng.load_model(path)
    am, top = [], []
    full = None
    for pos in range(n):
        lg = eng.forward(int(inputs[pos]), pos)
        am.append(eng.last_argmax)
        top.append(lg[g["top_idx"][pos]].copy())
        if pos == len(prompt) - 1:
            full = lg.copy()
    eng.close()
    am, top = np.array(am), np.array(top)
    assert np.array_equal(top.view(np.uint32), r["top_val"].view(np.uint32))
    assert np.array_equal(am, r["argmax"])
    dec = np.array(v["decidable"])
    assert np.array_equal(am[dec], toks[dec])
    bound = 1.25 * max(v["mean_abs_top32_4_vs_1"])
    assert np.abs(top - g["top_val"]).mean() <= bound
    assert np.abs(full - g["full_last_prompt"]).mean() <= bound
    assert int(np.argmax(full)) == int(toks[len(prompt) - 1]) or not dec[len(prompt) - 1]
