"""Kernel-level parity on the GPU, through the C ABI.

Bit-exact checks: Q8_K quantisers (both rounding rules), the quantised GEMVs (Q4_K, Q6_K;
outputs identical to the reference's AVX2 kernels and to the C restatement), their
integer block sums, RMSNorm->Q8_K and SwiGLU->Q8_K against the restatement.
"""
import numpy as np
import pytest

from conftest import rand_tensor_bytes

pytestmark = pytest.mark.gpu


def _dev(cuda, arr):
    return cuda.from_numpy(np.ascontiguousarray(arr)).cuda()


def _q8k_from_dev(cuda, t):
    import oracle as O
    return t.cpu().numpy().view(O.Q8K_DTYPE)


def _q8k_eq(a, b):
    assert np.array_equal(a["qs"], b["qs"])
    assert np.array_equal(a["bsums"], b["bsums"])
    assert np.array_equal(a["d"].view(np.uint32), b["d"].view(np.uint32))


@pytest.mark.parametrize("rounding", [0, 1])
@pytest.mark.parametrize("kind", ["normal", "zeros", "tiny", "nan", "huge"])
def test_quantize_q8k_exact(cuda, oracle, rounding, kind):
    from mcpm import engine as E
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 256 * 24).astype(np.float32)
    if kind == "zeros":
        x[:512] = 0
    elif kind == "tiny":
        x *= 1e-38
    elif kind == "nan":
        x[5] = np.nan
        x[256 + 255] = np.nan          # last element of a block: block amax NaN -> zero block
        x[512 + 100] = np.nan
    elif kind == "huge":
        x[7] = 3e38
    xd = _dev(cuda, x)
    yd = cuda.zeros(24 * 292, dtype=cuda.uint8, device="cuda")
    E.quantize_q8k(xd.data_ptr(), yd.data_ptr(), x.size, rounding)
    cuda.cuda.synchronize()
    got = _q8k_from_dev(cuda, yd)
    _q8k_eq(got, oracle.quantize_q8k(x, rounding, 1))


SHAPES = [(2048, 2048), (256, 2048), (6144, 2048), (2048, 6144), (1, 2048), (37, 2048), (130560, 2048)]


@pytest.mark.parametrize("ggml_type", [12, 14])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_bitexact(cuda, oracle, ggml_type, rows, cols):
    from mcpm import engine as E
    if ggml_type == 12 and rows == 130560:
        pytest.skip("LM head is Q6_K")
    w = rand_tensor_bytes(ggml_type, rows, cols, seed=rows * 7 + cols + ggml_type)
    x = np.random.default_rng(rows + cols).normal(0, 1, cols).astype(np.float32)
    xq = oracle.quantize_q8k(x, 0, 1)
    wd, xqd = _dev(cuda, w), _dev(cuda, xq.view(np.uint8))
    yd = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    E.gemv_q8k(ggml_type, wd.data_ptr(), xqd.data_ptr(), yd.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    got = yd.cpu().numpy()
    want = oracle.gemv_q8k(ggml_type, w, xq, rows, cols, order=1, fused_min=1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{np.sum(got != want)} of {rows} rows differ, max {np.max(np.abs(got - want))}"


@pytest.mark.parametrize("ggml_type", [12, 14])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_block_order_bitexact(cuda, oracle, ggml_type, rows, cols):
    """The decode kernel's warp-per-row GEMV (block order) against the restatement's
    ORC_ORDER_BATCH, bit for bit, including the Q6_K LM head shape."""
    from mcpm import engine as E
    if ggml_type == 12 and rows == 130560:
        pytest.skip("LM head is Q6_K")
    w = rand_tensor_bytes(ggml_type, rows, cols, seed=rows * 5 + cols + ggml_type)
    x = np.random.default_rng(rows + cols + 1).normal(0, 1, cols).astype(np.float32)
    xq = oracle.quantize_q8k(x, 0, 1)
    wd, xqd = _dev(cuda, w), _dev(cuda, xq.view(np.uint8))
    yd = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    E.gemv_q8k_block(ggml_type, wd.data_ptr(), xqd.data_ptr(), yd.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    got = yd.cpu().numpy()
    want = oracle.gemv_q8k(ggml_type, w, xq, rows, cols, order=2, fused_min=1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{np.sum(got != want)} of {rows} rows differ, max {np.max(np.abs(got - want))}"


@pytest.mark.parametrize("ggml_type", [12, 14])
def test_gemv_matches_reference_build(cuda, oracle, ref, ggml_type):
    from mcpm import engine as E
    rows, cols = 512, 6144
    w = rand_tensor_bytes(ggml_type, rows, cols, seed=11)
    xq = ref.quantize_q8k(np.random.default_rng(5).normal(0, 3, cols).astype(np.float32))
    wd, xqd = _dev(cuda, w), _dev(cuda, xq.view(np.uint8))
    yd = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    E.gemv_q8k(ggml_type, wd.data_ptr(), xqd.data_ptr(), yd.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), ref.gemv_q8k(ggml_type, w, xq, rows, cols))


def q8_0_matrix(rows, cols, seed):
    """Q8_0 blocks with the config-1 distributions: fp16 d ~ |N(0, 2e-3)|, int8 uniform -127..127."""
    rng = np.random.default_rng(seed)
    nb = rows * cols // 32
    blk = np.zeros(nb, dtype=[("d", "<f2"), ("qs", "i1", 32)])
    blk["d"] = np.abs(rng.normal(0, 2e-3, nb)).astype(np.float16)
    blk["qs"] = rng.integers(-127, 128, (nb, 32))
    return blk.view(np.uint8)


@pytest.mark.parametrize("rows,cols", [(2048, 2048), (256, 2048), (12288, 2048), (2048, 6144), (1, 256), (37, 8192)])
def test_gemv_q8_0_bitexact(cuda, oracle, rows, cols):
    """Q8_0 x fp32 GEMV against the restatement of the reference build's evaluation order."""
    from mcpm import engine as E
    w = q8_0_matrix(rows, cols, rows + cols)
    x = np.random.default_rng(cols).normal(0, 1, cols).astype(np.float32)
    wd, xd = _dev(cuda, w), _dev(cuda, x)
    yd = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    E.gemv_q8_0(wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    want = oracle.gemv_q8_0(w, x, rows, cols)
    got = yd.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.max(np.abs(got - want))


def test_gemv_q8_0_matches_reference_build(cuda, ref):
    from mcpm import engine as E
    rows, cols = 300, 6144
    w = q8_0_matrix(rows, cols, 5)
    x = np.random.default_rng(6).normal(0, 1, cols).astype(np.float32)
    wd, xd = _dev(cuda, w), _dev(cuda, x)
    yd = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    E.gemv_q8_0(wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), ref.gemv_f32(8, w, x, rows, cols).view(np.uint32))


@pytest.mark.parametrize("ggml_type", [12, 14])
def test_blocksums_exact(cuda, oracle, ggml_type):
    from mcpm import engine as E
    rows, cols = 300, 6144 if ggml_type == 14 else 2048
    w = rand_tensor_bytes(ggml_type, rows, cols, seed=21)
    xq = oracle.quantize_q8k(np.random.default_rng(9).normal(0, 1, cols).astype(np.float32), 1, 1)
    nb = cols // 256
    wd, xqd = _dev(cuda, w), _dev(cuda, xq.view(np.uint8))
    isum = cuda.zeros(rows * nb, dtype=cuda.int32, device="cuda")
    aux = cuda.zeros(rows * nb, dtype=cuda.int32, device="cuda")
    E.gemv_blocksums(ggml_type, wd.data_ptr(), xqd.data_ptr(), isum.data_ptr(), aux.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    wi, wa = oracle.blocksums(ggml_type, w, xq, rows, cols)
    assert np.array_equal(isum.cpu().numpy().reshape(rows, nb), wi)
    assert np.array_equal(aux.cpu().numpy().reshape(rows, nb), wa)


def test_gate_up(cuda, oracle):
    from mcpm import engine as E
    rows, cols = 6144, 2048
    wg = rand_tensor_bytes(12, rows, cols, seed=31)
    wu = rand_tensor_bytes(12, rows, cols, seed=32)
    xq = oracle.quantize_q8k(np.random.default_rng(1).normal(0, 1, cols).astype(np.float32), 1, 1)
    g = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    u = cuda.zeros(rows, dtype=cuda.float32, device="cuda")
    xqd = _dev(cuda, xq.view(np.uint8))
    wgd, wud = _dev(cuda, wg), _dev(cuda, wu)   # keep the device copies alive across the launch
    E.gemv_gate_up_q8k(wgd.data_ptr(), wud.data_ptr(), xqd.data_ptr(), g.data_ptr(), u.data_ptr(), rows, cols)
    cuda.cuda.synchronize()
    assert np.array_equal(g.cpu().numpy(), oracle.gemv_q8k(12, wg, xq, rows, cols, 1, 1))
    assert np.array_equal(u.cpu().numpy(), oracle.gemv_q8k(12, wu, xq, rows, cols, 1, 1))


@pytest.mark.parametrize("scale", [1.0, 300.0, 1e-30])
def test_rmsnorm_q8k_exact(cuda, oracle, scale):
    from mcpm import engine as E
    rng = np.random.default_rng(int(scale * 7) % 1000)
    x = (rng.normal(0, 1, 2048) * scale).astype(np.float32)
    w = (1 + rng.normal(0, 0.02, 2048)).astype(np.float32)
    out = cuda.zeros(8 * 292, dtype=cuda.uint8, device="cuda")
    xd, wd = _dev(cuda, x), _dev(cuda, w)
    E.rmsnorm_q8k(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), 2048, 1e-6)
    cuda.cuda.synchronize()
    _q8k_eq(_q8k_from_dev(cuda, out), oracle.rmsnorm_q8k(x, w))


@pytest.mark.parametrize("scale", [1.0, 50.0, 2000.0])
def test_swiglu_q8k_exact(cuda, oracle, scale):
    """Large |g| makes exp(-g) overflow: the reference build's silu is NaN there."""
    from mcpm import engine as E
    rng = np.random.default_rng(int(scale))
    g = (rng.normal(0, 1, 6144) * scale).astype(np.float32)
    u = (rng.normal(0, 1, 6144) * scale).astype(np.float32)
    out = cuda.zeros(24 * 292, dtype=cuda.uint8, device="cuda")
    gd, ud = _dev(cuda, g), _dev(cuda, u)
    E.swiglu_q8k(gd.data_ptr(), ud.data_ptr(), out.data_ptr(), 6144)
    cuda.cuda.synchronize()
    _q8k_eq(_q8k_from_dev(cuda, out), oracle.swiglu_q8k(g, u))


def test_op_argument_errors(cuda):
    from mcpm import engine as E
    t = cuda.zeros(4096, dtype=cuda.float32, device="cuda")
    with pytest.raises(E.MCPMError) as ei:
        E.quantize_q8k(t.data_ptr(), t.data_ptr(), 100, 0)
    assert ei.value.status == E.BAD_ARG
    with pytest.raises(E.MCPMError) as ei:
        E.gemv_q8k(8, t.data_ptr(), t.data_ptr(), t.data_ptr(), 4, 2048)
    assert ei.value.status == E.UNSUPPORTED_TYPE
    with pytest.raises(E.MCPMError):
        E.gemv_q8k(14, t.data_ptr(), t.data_ptr(), t.data_ptr(), 4, 256)   # Q6_K rows must be 16-byte multiples


@pytest.mark.parametrize("pos", [0, 1, 31, 32, 100, 2047, 2048, 5000, 8200, 12000, 16383])
def test_attention_exact(cuda, oracle, pos):
    """Split-KV GQA attention (execute_attention) against the restatement, including the
    K/V append at pos and the ties-to-even Q8_K of the output (the o_proj input).  Chunk
    lengths 32 .. 256 (160-row staging: one round up to 10240 positions, two beyond), 1 .. 64
    chunks."""
    import ctypes as C
    import oracle as O
    from mcpm import engine as E
    max_seq = max(6000, pos + 1)
    rng = np.random.default_rng(pos + 1)
    q = (rng.normal(0, 3, 2048)).astype(np.float32)
    k = (rng.normal(0, 3, 256)).astype(np.float32)
    v = (rng.normal(0, 3, 256)).astype(np.float32)
    kc = (rng.normal(0, 3, (max_seq, 256))).astype(np.float32)
    vc = (rng.normal(0, 3, (max_seq, 256))).astype(np.float32)
    qd, kd, vd, kcd, vcd = (_dev(cuda, a) for a in (q, k, v, kc, vc))
    out = cuda.zeros(2048, dtype=cuda.float32, device="cuda")
    oq = cuda.zeros(8 * 292, dtype=cuda.uint8, device="cuda")
    E.attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kcd.data_ptr(), vcd.data_ptr(), pos, max_seq,
                out.data_ptr(), oq.data_ptr())
    cuda.cuda.synchronize()
    want = np.zeros(2048, np.float32)
    assert oracle.lib.orc_attention(O._fptr(want), O._fptr(q), O._fptr(k), O._fptr(v), O._fptr(kc), O._fptr(vc),
                                    pos, max_seq, 16, 2, 128) == 0
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.max(np.abs(got - want))
    assert np.array_equal(kcd.cpu().numpy()[pos], k) and np.array_equal(vcd.cpu().numpy()[pos], v)
    _q8k_eq(_q8k_from_dev(cuda, oq), oracle.quantize_q8k(want, 0, 1))


def test_attention_rejects_out_of_range(cuda):
    from mcpm import engine as E
    t = cuda.zeros(4096, dtype=cuda.float32, device="cuda")
    with pytest.raises(E.MCPMError) as ei:
        E.attention(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 8, 8, t.data_ptr())
    assert ei.value.status == E.CTX_OVERFLOW
    with pytest.raises(E.MCPMError) as ei:
        E.attention(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 20000, t.data_ptr())
    assert ei.value.status == E.BAD_ARG


def test_rope_kv_append_bitexact(cuda, oracle):
    """mcpm_rope_kv_append: q (16 heads) and k (2 heads) rotated in place exactly as the
    restatement's apply_rope, k and v written at row pos, every other cache row untouched."""
    from mcpm import engine as E
    rng = np.random.default_rng(21)
    max_seq = 40
    for pos in (0, 7, 39):
        q = rng.normal(0, 3, 2048).astype(np.float32)
        k = rng.normal(0, 3, 256).astype(np.float32)
        v = rng.normal(0, 3, 256).astype(np.float32)
        kc = rng.normal(0, 1, (max_seq, 256)).astype(np.float32)
        vc = rng.normal(0, 1, (max_seq, 256)).astype(np.float32)
        d = [cuda.from_numpy(a.copy()).cuda() for a in (q, k, v, kc, vc)]
        E.rope_kv_append(*[t.data_ptr() for t in d], pos, max_seq)
        cuda.cuda.synchronize()
        want_q, want_k = oracle.rope(q, pos, 16), oracle.rope(k, pos, 2)
        gq, gk, gkc, gvc = d[0].cpu().numpy(), d[1].cpu().numpy(), d[3].cpu().numpy(), d[4].cpu().numpy()
        assert np.array_equal(gq.view(np.uint32), want_q.view(np.uint32))
        assert np.array_equal(gk.view(np.uint32), want_k.view(np.uint32))
        assert np.array_equal(gkc[pos], want_k) and np.array_equal(gvc[pos], v)
        others = np.arange(max_seq) != pos
        assert np.array_equal(gkc[others], kc[others]) and np.array_equal(gvc[others], vc[others])
    lib = E.load_library()
    t = cuda.zeros(4096, dtype=cuda.float32, device="cuda")
    p = t.data_ptr()
    assert lib.mcpm_rope_kv_append(p, p, p, p, p, 8, 8, 5e6, None) == E.CTX_OVERFLOW
    assert lib.mcpm_rope_kv_append(None, p, p, p, p, 0, 8, 5e6, None) == E.BAD_ARG
