"""Pins the C restatement (oracle/mcpm_oracle.c) to the reference build (CPU only).

1. Committed golden vectors produced by the reference build (tests/golden/make_golden.py):
   the tensor table, GEMV and quantiser outputs (bit-exact), and a 32-step decode at one
   OpenMP thread (tokens identical; logits within the reference's own thread-count spread).
2. When the reference library is present (oracle/_ref), the same checks against the live
   build on fresh inputs.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

import oracle as O
from mcpm import spec, synth


def golden(name):
    return os.path.join(GOLDEN, name)


def test_tensor_table_matches_reference_header():
    g = json.load(open(golden("metadata_digest.json")))
    table = spec.q4km_table()
    assert len(table) == g["rows"] == 381
    assert spec.table_digest(table) == g["sha256"]
    assert table[0].offset == g["data_start"]
    assert table[-1].offset + table[-1].nbytes == g["file_end"]


def test_weight_bytes_per_token():
    w = spec.weight_bytes_per_token(spec.q4km_table())
    assert w["total"] == 1_405_768_832 and w["embedding_row"] == 1152
    assert spec.KV_BYTES_PER_POSITION == 86_016


@pytest.mark.parametrize("rows,cols,name,t,seed", [(64, 2048, "q4k", 12, 101), (48, 6144, "q4k", 12, 102),
                                                    (64, 2048, "q6k", 14, 103), (40, 6144, "q6k", 14, 104)])
def test_gemv_and_quantize_bitexact_vs_reference_golden(oracle, rows, cols, name, t, seed):
    import make_golden as mg
    g = np.load(golden("reference_kernels.npz"))
    w, x = mg.kernel_inputs(t, rows, cols, seed)
    xq = oracle.quantize_q8k(x, oracle.ROUND_EVEN, 1)
    assert np.array_equal(xq.view(np.uint8), g[f"{name}_{rows}x{cols}_xq"])
    y = oracle.gemv_q8k(t, w, xq, rows, cols, order=1, fused_min=1)
    assert np.array_equal(y.view(np.uint32), g[f"{name}_{rows}x{cols}_y"].view(np.uint32))


@pytest.mark.parametrize("rows,cols,seed", [(64, 2048, 301), (40, 6144, 302), (16, 256, 303)])
def test_gemv_q8_0_bitexact_vs_reference_golden(oracle, rows, cols, seed):
    """Q8_0 x fp32 GEMV (gemv_q8_0 as the reference build evaluates it)."""
    import make_golden as mg
    g = np.load(golden("reference_q8_0.npz"))
    w, x = mg.q8_0_inputs(rows, cols, seed)
    y = oracle.gemv_q8_0(w, x, rows, cols)
    assert np.array_equal(y.view(np.uint32), g[f"q8_0_{rows}x{cols}_y"].view(np.uint32))


def test_rmsnorm_quantize_vs_reference_golden(oracle):
    """Integer-valued input: the sum of squares is exact in any order, so only the
    reference's rsqrt estimate can differ; the int8 values and block sums must match."""
    g = np.load(golden("reference_kernels.npz"))
    got = oracle.rmsnorm_q8k(g["rmsnorm_int_x"], g["rmsnorm_int_w"])
    want = g["rmsnorm_int_q8k"].view(O.Q8K_DTYPE)
    assert np.array_equal(got["qs"], want["qs"]) and np.array_equal(got["bsums"], want["bsums"])
    np.testing.assert_allclose(got["d"], want["d"], rtol=3e-7)


def test_integer_block_sums_agree_with_scalar_reference_formula(oracle):
    """Q4_K/Q6_K block sums restate dot_row_q*_K_q8_K_scalar: check them against an
    independent numpy evaluation of the dequantised product."""
    import make_golden as mg
    for t, cols in ((12, 2048), (14, 2048)):
        w, x = mg.kernel_inputs(t, 4, cols, 55)
        xq = oracle.quantize_q8k(x, 1, 1)
        isum, aux = oracle.blocksums(t, w, xq, 4, cols)
        q8 = xq["qs"].astype(np.int64)
        blocks = w.reshape(4 * cols // 256, -1)
        for r in range(4):
            for b in range(cols // 256):
                blk = blocks[r * (cols // 256) + b]
                if t == 12:
                    sc = np.zeros(8, np.int64); mn = np.zeros(8, np.int64)
                    q = blk[4:16]
                    for j in range(4):
                        sc[j], mn[j] = q[j] & 63, q[j + 4] & 63
                        sc[j + 4] = (q[j + 8] & 15) | ((q[j] >> 6) << 4)
                        mn[j + 4] = (q[j + 8] >> 4) | ((q[j + 4] >> 6) << 4)
                    qs = blk[16:]
                    vals = np.zeros(256, np.int64)
                    for j in range(4):
                        vals[64 * j:64 * j + 32] = (qs[32 * j:32 * j + 32] & 15) * sc[2 * j]
                        vals[64 * j + 32:64 * j + 64] = (qs[32 * j:32 * j + 32] >> 4) * sc[2 * j + 1]
                    assert isum[r, b] == int(np.dot(vals, q8[b]))
                    bs = xq["bsums"][b].astype(np.int64)
                    assert aux[r, b] == int(sum(mn[g] * (bs[2 * g] + bs[2 * g + 1]) for g in range(8)))
                else:
                    ql, qh, s = blk[:128].astype(np.int64), blk[128:192].astype(np.int64), blk[192:208].view(np.int8)
                    vals = np.zeros(256, np.int64)
                    for h in range(2):
                        for l in range(32):
                            for k in range(4):
                                lo = ql[64 * h + l + (32 if k & 1 else 0)]
                                lo = (lo >> 4) if k & 2 else (lo & 15)
                                qv = lo | (((qh[32 * h + l] >> (2 * k)) & 3) << 4)
                                vals[128 * h + 32 * k + l] = qv * s[8 * h + 2 * k + (l >= 16)]
                    assert isum[r, b] == int(np.dot(vals, q8[b]))
                    assert aux[r, b] == 32 * int(np.dot(s.astype(np.int64), xq["bsums"][b].astype(np.int64)))


@pytest.fixture(scope="module")
def decode_golden():
    return np.load(golden("reference_decode_q4km.npz"))


def test_restatement_decode_matches_reference_golden(oracle, model_path, decode_golden):
    """Greedy tokens identical to the reference build; logits within 2e-3 + 1e-3*max|row|,
    the scale of the reference's own variation between OpenMP thread counts
    (tests/golden/reference_variability.json)."""
    g = decode_golden
    var = json.load(open(golden("reference_variability.json")))
    assert json.load(open(model_path + ".json"))["content_digest"] == var["model_manifest"]["content_digest"]
    prompt = g["prompt"]
    n = len(g["tokens"])
    om = O.OracleModel(oracle, model_path, n + 1)
    lg = np.zeros(spec.N_VOCAB, np.float32)
    tok = None
    for pos in range(n):
        t = int(prompt[pos]) if pos < len(prompt) else tok
        tok = om.forward(t, pos, lg)
        assert tok == g["tokens"][pos], f"pos {pos}"
        row_scale = np.abs(g["strided"][pos]).max()
        np.testing.assert_allclose(lg[::256], g["strided"][pos], rtol=0, atol=2e-3 + 1e-3 * row_scale)
        np.testing.assert_array_equal(np.sort(g["top_idx"][pos][:4]), np.sort(np.argsort(-lg, kind="stable")[:4]))


def test_reference_variability_bounds_the_tolerance():
    var = json.load(open(golden("reference_variability.json")))
    assert var["tokens_equal"]
    assert var["max_rel_to_row_max"] < 1e-3


# ---------------------------------------------------------------- live reference (optional)
@pytest.mark.parametrize("t,rows,cols", [(12, 300, 2048), (14, 300, 6144), (14, 1000, 2048)])
def test_live_reference_gemv_bitexact(oracle, ref, t, rows, cols):
    import make_golden as mg
    w, x = mg.kernel_inputs(t, rows, cols, 900 + rows)
    xq = ref.quantize_q8k(x)
    assert np.array_equal(xq.view(np.uint8), oracle.quantize_q8k(x, 0, 1).view(np.uint8))
    assert np.array_equal(ref.gemv_q8k(t, w, xq, rows, cols), oracle.gemv_q8k(t, w, xq, rows, cols, 1, 1))


def test_live_reference_gemv_q8_0_bitexact(oracle, ref):
    import make_golden as mg
    w, x = mg.q8_0_inputs(200, 2048, 777)
    assert np.array_equal(ref.gemv_f32(8, w, x, 200, 2048).view(np.uint32), oracle.gemv_q8_0(w, x, 200, 2048).view(np.uint32))


def test_live_reference_embedding_exact(oracle, ref, model_path):
    om = O.OracleModel(oracle, model_path, 2)
    w = om.tensor("token_embd.weight")
    for tok in (0, 1, 65535, 130559):
        assert np.array_equal(ref.embedding(w, "Q4_K", tok), oracle.embedding(w, spec.GGML_Q4_K, tok))


def test_live_reference_swiglu_nan_semantics(oracle, ref):
    """|g| large enough that exp(-g) overflows: the build's silu is NaN and whole blocks
    become zeros; the restatement reproduces the int8 output."""
    rng = np.random.default_rng(4)
    g = (rng.normal(0, 1, 6144) * 1500).astype(np.float32)
    u = (rng.normal(0, 1, 6144) * 1500).astype(np.float32)
    a, b = ref.swiglu_q8k(g, u), oracle.swiglu_q8k(g, u)
    assert np.array_equal(a["qs"], b["qs"]) and np.array_equal(a["bsums"], b["bsums"])


# ---- floating-point ops against the reference build, per element: |a - b| <= 2e-3 + 1e-3 |b|
def _close(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= 2e-3 + 1e-3 * np.abs(b)))


@pytest.mark.parametrize("pos", [0, 31, 300, 3000, 16383])
def test_attention_vs_reference(oracle, ref, pos):
    """execute_attention (ops.cpp:537-628): K/V append at pos, then softmax(q.K^T/sqrt(128)) V
    over positions 0..pos; the restatement's split-KV chunks and combine order against the
    reference's single pass, with the reference build's expf."""
    from oracle import _fptr
    rng = np.random.default_rng(pos + 11)
    max_seq = pos + 1
    q = rng.normal(0, 1, 2048).astype(np.float32)
    k = rng.normal(0, 1, 256).astype(np.float32)
    v = rng.normal(0, 1, 256).astype(np.float32)
    kc = rng.normal(0, 1, (max_seq, 256)).astype(np.float32)
    vc = rng.normal(0, 1, (max_seq, 256)).astype(np.float32)
    outs = []
    for lib, fn in ((ref.lib, "ref_attention"), (oracle.lib, "orc_attention")):
        o = np.zeros(2048, np.float32)
        kk, vv = kc.copy(), vc.copy()
        getattr(lib, fn)(_fptr(o), _fptr(q), _fptr(k), _fptr(v), _fptr(kk), _fptr(vv), pos, max_seq, 16, 2, 128)
        assert np.array_equal(kk[pos], k) and np.array_equal(vv[pos], v)
        outs.append(o)
    assert _close(outs[1], outs[0])


@pytest.mark.parametrize("pos", [1, 100, 5000, 16383])
def test_rope_vs_reference(oracle, ref, pos):
    """apply_rope (ops.cpp:502-516), interleaved pairs, theta = 5e6^(-i/128), on 16 query
    heads and 2 key heads."""
    rng = np.random.default_rng(pos)
    for n_heads in (16, 2):
        x = rng.normal(0, 3, n_heads * 128).astype(np.float32)
        want = ref.rope(x, pos, n_heads)
        got = oracle.rope(x, pos, n_heads)
        assert _close(got, want)


def test_rmsnorm_vs_reference(oracle, ref):
    """rmsnorm (ops.cpp:468-481) on real-valued input: the reference's reciprocal square-root
    estimate and summation order against the restatement's canonical order."""
    rng = np.random.default_rng(5)
    for scale in (0.01, 1.0, 300.0):
        x = (rng.normal(0, 1, 2048) * scale).astype(np.float32)
        w = (1 + rng.normal(0, 0.02, 2048)).astype(np.float32)
        assert _close(oracle.rmsnorm(x, w), ref.rmsnorm(x, w))
