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
  reference_q8_0.npz          gemv_q8_0 of the reference build (fp32 activations) on seeded
                              Q8_0 matrices with the config-1 distributions

    python tests/golden/make_golden.py --q8_0     # only reference_q8_0.npz
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
path = synth.ensure_model("q4_k_m", 0)
n_prompt, n_gen, seed = int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
e = O.RefEngine(O.Ref(), path, n_prompt + n_gen + 1)
prompt = synth.prompt_ids(n_prompt, seed=seed)
lg = np.zeros(130560, np.float32)
toks, top_i, top_v, strided = [], [], [], []
tok = None
for pos in range(n_prompt + n_gen):
    t = int(prompt[pos]) if pos < n_prompt else tok
    tok = e.forward(t, pos, lg)
    toks.append(tok)
    idx = np.argsort(-lg, kind="stable")[:32]
    top_i.append(idx.astype(np.int32)); top_v.append(lg[idx].copy()); strided.append(lg[::256].copy())
np.savez_compressed(sys.argv[6], prompt=prompt, tokens=np.array(toks, np.int32), top_idx=np.array(top_i),
                    top_val=np.array(top_v), strided=np.array(strided))
"""


def decode(threads, out_path):
    env = dict(os.environ, OMP_NUM_THREADS=str(threads))
    subprocess.run([sys.executable, "-c", DECODE_CHILD, os.path.join(REPO, "oracle"),
                    os.path.join(REPO, "minicpm5.cpp_b200"), str(N_PROMPT), str(N_GEN), str(PROMPT_SEED), out_path],
                   env=env, check=True)


def main():
    import oracle as O
    from mcpm import synth
    O.build(reference=True)
    assert O.have_ref(), "needs the reference tree"
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


if __name__ == "__main__":
    main()
