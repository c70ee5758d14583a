"""Regenerates the golden fixtures from the reference build (run in a container that has the
reference tree; the fixtures are committed and the tests only read them).

    python tests/golden/make_golden.py

Fixtures:
  metadata_digest.json        digest of the reference's tensor table (include/minicpm_metadata.h)
  reference_kernels.npz       reference-build outputs on seeded inputs: quantize_row_q8_K_avx2,
                              gemv_q4_K_q8_K_avx2, gemv_q6_K_q8_K_avx2, rmsnorm_and_quantize_q8k
                              (integer-valued input so the sum is order-free)
  reference_decode_q4km.npz   MiniCPM5Engine::forward of the reference build at OMP_NUM_THREADS=1
                              on the seed-0 synthetic Q4_K_M model: greedy tokens, top-32
                              logits per step and every 256th logit
  reference_variability.json  reference at 1 vs 4 OpenMP threads on the same steps
  reference_decode_wc.npz     MiniCPM5Engine::forward of the reference build at OMP_NUM_THREADS=1
                              on the seed-0 parity model (same layout and types, balanced Q4_K
                              mins, per-layer block scales x PARITY_DSCALE): the config-0 shape,
                              a 128-id prompt (seed 1234) then 64 greedy tokens; argmax at every
                              position, top-32 logits and every 256th logit per position, all
                              logits at the last prompt position
  reference_variability_wc.json  the reference's own spread on the parity run: eight teacher-forced
                              runs at 4 OpenMP threads against the 1-thread run (per position)
  restatement_decode_wc.npz   the C restatement on the same teacher-forced inputs (eight-lane order)
  restatement_decode_wc_block.npz  the same in the block order (the engine's default GEMV order)
  reference_q8_0.npz          gemv_q8_0 of the reference build (fp32 activations) on seeded
                              Q8_0 matrices with the config-1 distributions

    python tests/golden/make_golden.py --q8_0     # only reference_q8_0.npz
    python tests/golden/make_golden.py --wc       # only the parity-model files
    python tests/golden/make_golden.py --restatement   # only the two restatement fixtures
"""
import json
import os
import re
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "minicpm5.cpp_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

N_PROMPT, N_GEN, PROMPT_SEED = 16, 16, 1234
# Parity model (synth.write_model dscale): the config-0 shape, 128 prompt ids + 64 greedy tokens.
PARITY_DSCALE, WC_PROMPT, WC_GEN = 0.04, 128, 64
N_SPREAD_RUNS = 8   # 4-thread reference runs that measure its own spread
KERNEL_CASES = [("q4k", 12, 64, 2048, 101), ("q4k", 12, 48, 6144, 102), ("q6k", 14, 64, 2048, 103),
                ("q6k", 14, 40, 6144, 104)]


def metadata_digest(ref_tree):
    from mcpm import spec
    text = open(os.path.join(ref_tree, "include", "minicpm_metadata.h")).read()
    rows = re.findall(r'\{ "([^"]+)", (\d+), (\d+), (\d+), \{ (\d+), (\d+), (\d+), (\d+) \}, "([^"]+)" \}', text)
    import hashlib
    h = hashlib.sha256()
    for r in rows:
        h.update(f"{r[0]},{r[1]},{r[2]},{r[3]},{r[4]},{r[5]},{r[6]},{r[7]},{r[8]}\n".encode())
    return {"rows": len(rows), "sha256": h.hexdigest(), "data_start": int(rows[0][1]),
            "file_end": int(rows[-1][1]) + int(rows[-1][2]), "note": "computed by make_golden.py"}


def kernel_inputs(ggml_type, rows, cols, seed):
    from mcpm import spec, synth
    w = synth.tensor_bytes(spec.TensorInfo("w", ggml_type, (cols, rows)), np.random.Generator(np.random.PCG64([seed, 1])))
    x = np.random.Generator(np.random.PCG64([seed, 2])).normal(0, 2, cols).astype(np.float32)
    return w, x


def kernels():
    import oracle as O
    ref = O.Ref()
    out = {}
    for name, t, rows, cols, seed in KERNEL_CASES:
        w, x = kernel_inputs(t, rows, cols, seed)
        xq = ref.quantize_q8k(x)
        out[f"{name}_{rows}x{cols}_xq"] = xq.view(np.uint8)
        out[f"{name}_{rows}x{cols}_y"] = ref.gemv_q8k(t, w, xq, rows, cols)
    rng = np.random.Generator(np.random.PCG64([7, 7]))
    xi = rng.integers(-60, 61, 2048).astype(np.float32)
    wn = (1 + rng.normal(0, 0.02, 2048)).astype(np.float32)
    out["rmsnorm_int_x"], out["rmsnorm_int_w"] = xi, wn
    out["rmsnorm_int_q8k"] = ref.rmsnorm_q8k(xi, wn).view(np.uint8)
    return out


Q8_0_CASES = [(64, 2048, 301), (40, 6144, 302), (16, 256, 303)]


def q8_0_inputs(rows, cols, seed):
    rng = np.random.Generator(np.random.PCG64([seed, 3]))
    nb = rows * cols // 32
    blk = np.zeros(nb, dtype=[("d", "<f2"), ("qs", "i1", 32)])
    blk["d"] = np.abs(rng.normal(0, 2e-3, nb)).astype(np.float16)
    blk["qs"] = rng.integers(-127, 128, (nb, 32))
    x = rng.normal(0, 1, cols).astype(np.float32)
    return blk.view(np.uint8), x


def q8_0_kernels():
    import oracle as O
    ref = O.Ref()
    out = {}
    for rows, cols, seed in Q8_0_CASES:
        w, x = q8_0_inputs(rows, cols, seed)
        out[f"q8_0_{rows}x{cols}_y"] = ref.gemv_f32(8, w, x, rows, cols)
    return out


DECODE_CHILD = r"""
import sys, json, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
import oracle as O
from mcpm import synth
n_prompt, n_gen, seed = int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
dscale = float(sys.argv[7]) if len(sys.argv) > 7 else 1.0
path = synth.ensure_model("q4_k_m", 0, dscale=dscale)
e = O.RefEngine(O.Ref(), path, n_prompt + n_gen + 1)
prompt = synth.prompt_ids(n_prompt, seed=seed)
lg = np.zeros(130560, np.float32)
toks, top_i, top_v, strided = [], [], [], []
tok = None
full = None
for pos in range(n_prompt + n_gen):
    t = int(prompt[pos]) if pos < n_prompt else tok
    tok = e.forward(t, pos, lg)
    toks.append(tok)
    idx = np.argsort(-lg, kind="stable")[:32]
    top_i.append(idx.astype(np.int32)); top_v.append(lg[idx].copy()); strided.append(lg[::256].copy())
    if pos == n_prompt - 1:
        full = lg.copy()
extra = {"full_last_prompt": full, "dscale": np.float64(dscale)} if dscale != 1.0 else {}
np.savez_compressed(sys.argv[6], prompt=prompt, tokens=np.array(toks, np.int32), top_idx=np.array(top_i),
                    top_val=np.array(top_v), strided=np.array(strided), **extra)
"""


def decode(threads, out_path, n_prompt=N_PROMPT, n_gen=N_GEN, dscale=1.0):
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    subprocess.run([sys.executable, "-c", DECODE_CHILD, os.path.join(REPO, "oracle"),
                    os.path.join(REPO, "minicpm5.cpp_b200"), str(n_prompt), str(n_gen), str(PROMPT_SEED), out_path,
                    str(dscale)], env=env, check=True)


TF_CHILD = r"""
import sys, json, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
import oracle as O
from mcpm import synth
golden, which, out, dscale = sys.argv[3], sys.argv[4], sys.argv[5], float(sys.argv[6])
g = np.load(golden)
toks, prompt = g["tokens"], g["prompt"]
n = len(toks)
inputs = list(prompt) + list(toks[len(prompt) - 1:n - 1])   # teacher forcing: the 1-thread run's tokens
path = synth.ensure_model("q4_k_m", 0, dscale=dscale)
eng = O.OracleModel(O.Oracle(), path, n + 1) if which.startswith("restatement") else O.RefEngine(O.Ref(), path, n + 1)
if which == "restatement_block":   # the engine's default GEMV order (ORC_ORDER_BATCH)
    eng.set_order(O.Oracle.ORDER_BATCH)
lg = np.zeros(130560, np.float32)
am, top = [], []
for pos in range(n):
    am.append(eng.forward(int(inputs[pos]), pos, lg))
    top.append(lg[g["top_idx"][pos]].copy())
np.savez_compressed(out, argmax=np.array(am, np.int32), top_val=np.array(top))
"""


def teacher_forced(which, threads, out_path):
    """`which` ("reference", "restatement" or "restatement_block") over the parity run's inputs, fed the 1-thread
    reference's own tokens: argmax and the logits at the 1-thread run's top-32 indices."""
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    subprocess.run([sys.executable, "-c", TF_CHILD, os.path.join(REPO, "oracle"), os.path.join(REPO, "minicpm5.cpp_b200"),
                    os.path.join(HERE, "reference_decode_wc.npz"), which, out_path, str(PARITY_DSCALE)],
                   env=env, check=True)


def restatement_fixtures():
    teacher_forced("restatement", 8, os.path.join(HERE, "restatement_decode_wc.npz"))
    teacher_forced("restatement_block", 8, os.path.join(HERE, "restatement_decode_wc_block.npz"))


def parity_model_goldens():
    """The config-0 shape on the parity model.

    reference_decode_wc.npz: the reference at 1 OpenMP thread (deterministic), free-running.
    reference_variability_wc.json: N_SPREAD_RUNS teacher-forced runs of the reference at 4 threads.  At
    more than one thread the reference does not repeat itself (its OpenMP reduction of the
    RMSNorm sum combines per-thread partials in arrival order), and the int8 re-quantisation
    in front of every GEMV turns those last-bit differences into logit differences of several
    units on this model; per position, `spread` is the largest |difference| over the top-32
    logits of either run against the 1-thread run.  A position is `decidable` when the
    1-thread run's top-2 margin exceeds that spread.
    restatement_decode_wc.npz: this project's C restatement, teacher-forced the same way, in the
    reference's eight-lane GEMV order (the CUDA engine with MCPM_GEMM_MMA must reproduce it bit for
    bit); restatement_decode_wc_block.npz: the same in the block order (ORC_ORDER_BATCH, the
    engine's default).
    """
    from mcpm import synth
    man = json.load(open(synth.ensure_model("q4_k_m", 0, dscale=PARITY_DSCALE) + ".json"))
    out = os.path.join(HERE, "reference_decode_wc.npz")
    decode(1, out, WC_PROMPT, WC_GEN, PARITY_DSCALE)
    a = np.load(out)
    runs = []
    for r in range(N_SPREAD_RUNS):
        tmp = os.path.join(HERE, f"_tmp_tf4_{r}.npz")
        teacher_forced("reference", 4, tmp)
        runs.append(dict(np.load(tmp)))
        os.unlink(tmp)
    restatement_fixtures()
    d = [np.abs(r["top_val"] - a["top_val"]) for r in runs]
    spread = np.max([x.max(1) for x in d], axis=0)
    margin = a["top_val"][:, 0] - a["top_val"][:, 1]
    gen = a["tokens"][WC_PROMPT - 1:]
    var = {"threads": [1, 4], "teacher_forced": True,
           "distinct_generated_tokens": int(len(set(gen.tolist()))), "generated": int(len(gen)),
           "argmax_agree_4_vs_1": [int(np.sum(r["argmax"] == a["tokens"])) for r in runs], "positions": int(len(margin)),
           "mean_abs_top32_4_vs_1": [float(x.mean()) for x in d],
           "spread": [round(float(x), 4) for x in spread],
           "decidable": [bool(x) for x in margin > spread],
           "model_manifest": man}
    with open(os.path.join(HERE, "reference_variability_wc.json"), "w") as f:
        json.dump(var, f)
    print(json.dumps({k: v for k, v in var.items() if k not in ("spread", "decidable")}))


def main():
    import oracle as O
    from mcpm import synth
    O.build(reference=True)
    assert O.have_ref(), "needs the reference tree"
    if "--wc" in sys.argv:
        parity_model_goldens()
        return
    if "--restatement" in sys.argv:   # only the restatement's teacher-forced fixtures (no reference run)
        restatement_fixtures()
        return
    np.savez_compressed(os.path.join(HERE, "reference_q8_0.npz"), **q8_0_kernels())
    if "--q8_0" in sys.argv:
        return
    ref_tree = O.REFERENCE_TREE
    with open(os.path.join(HERE, "metadata_digest.json"), "w") as f:
        json.dump(metadata_digest(ref_tree), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "reference_kernels.npz"), **kernels())
    man = json.load(open(synth.ensure_model("q4_k_m", 0) + ".json"))
    decode(1, os.path.join(HERE, "reference_decode_q4km.npz"))
    tmp = os.path.join(HERE, "_tmp_ref4.npz")
    decode(4, tmp)
    a, b = np.load(os.path.join(HERE, "reference_decode_q4km.npz")), np.load(tmp)
    err = np.abs(a["top_val"] - b["top_val"])
    var = {"threads": [1, 4], "tokens_equal": bool(np.array_equal(a["tokens"], b["tokens"])),
           "max_abs_top32": float(err.max()),
           "max_rel_to_row_max": float((np.abs(a["strided"] - b["strided"]).max(1) / np.abs(a["strided"]).max(1)).max()),
           "model_manifest": man}
    os.unlink(tmp)
    with open(os.path.join(HERE, "reference_variability.json"), "w") as f:
        json.dump(var, f, indent=1)
    print(json.dumps(var))
    parity_model_goldens()


if __name__ == "__main__":
    main()
