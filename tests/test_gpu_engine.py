"""Whole-forward parity on the GPU through the C ABI.

The CUDA decode path and the C restatement follow the same canonical numerics, so logits,
the residual stream, K/V cache rows and greedy tokens are compared for exact equality, in both
GEMV orders of the engine: the block order (mcpm_config::batch_gemm MCPM_GEMM_TCGEN05, the
default; the restatement's ORC_ORDER_BATCH) and the reference's eight-lane order (MCPM_GEMM_MMA;
ORC_ORDER_AVX2).  The restatement itself is checked against the reference build in
test_oracle_vs_reference and test_parity_model.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PROMPT, N_GEN = 12, 8
MAX_SEQ = 64
ORDERS = ("block", "avx2")


def gemm_of(order):
    from mcpm import engine as E
    return E.GEMM_TCGEN05 if order == "block" else E.GEMM_MMA


def oracle_order(order):
    import oracle as O
    return O.Oracle.ORDER_BATCH if order == "block" else O.Oracle.ORDER_AVX2


@pytest.fixture(scope="module", params=ORDERS)
def order(request):
    return request.param


@pytest.fixture(scope="module")
def engine(cuda, model_path, order):
    from mcpm import engine as E
    e = E.MiniCPM5Engine(device=0, max_seq=MAX_SEQ, batch_gemm=gemm_of(order))
    assert e.load_model(model_path)
    yield e
    e.close()


@pytest.fixture(scope="module")
def oracle_model(oracle, model_path, order):
    import oracle as O
    m = O.OracleModel(oracle, model_path, MAX_SEQ)
    m.set_order(oracle_order(order))
    return m


def test_forward_bitexact_vs_restatement(engine, oracle_model):
    from mcpm import synth
    prompt = synth.prompt_ids(N_PROMPT)
    ref_logits = np.zeros(engine.n_vocab, np.float32)
    tok = None
    for pos in range(N_PROMPT + N_GEN):
        t = int(prompt[pos]) if pos < N_PROMPT else tok
        got = engine.forward(t, pos).copy()
        want_tok = oracle_model.forward(t, pos, ref_logits)
        gx, ox = engine.read_x(), oracle_model.x()
        assert np.array_equal(gx.view(np.uint32), ox.view(np.uint32)), \
            f"pos {pos}: residual differs in {np.sum(gx != ox)} elements"
        diff = np.sum(got.view(np.uint32) != ref_logits.view(np.uint32))
        assert diff == 0, f"pos {pos}: {diff} logits differ, max {np.max(np.abs(got - ref_logits))}"
        assert engine.last_argmax == want_tok
        tok = want_tok


@pytest.mark.parametrize("pos,order", [(300, "block"), (1000, "block"), (3000, "block"), (8200, "block"),
                                       (10300, "block"), (300, "avx2"), (8200, "avx2")])
def test_late_steps_bitexact_vs_restatement(cuda, oracle, model_path, pos, order):
    """Two decode steps at a late position over a seeded cache (the same random K/V rows
    0..pos-1 in the engine and in the restatement), covering every attention path of the
    decode kernel: 300 positions (32-row chunks, 10 chunks combined in the o_proj prologue
    behind a grid barrier), 1000 (32-row chunks, 32 chunks: head-pair combiners polled
    without a barrier), 3000 / 8200 (64- / 160-row chunks), 10300 (192-row chunks, two
    staging rounds)."""
    import oracle as O
    from mcpm import engine as E, spec
    max_seq = pos + 2
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=gemm_of(order))
    assert e.load_model(model_path)
    om = O.OracleModel(oracle, model_path, max_seq)
    om.set_order(oracle_order(order))
    try:
        rng = np.random.default_rng(pos)
        k = rng.normal(0, 1, (pos, 256)).astype(np.float32)
        v = rng.normal(0, 1, (pos, 256)).astype(np.float32)
        for layer in range(spec.N_LAYER):
            kl, vl = np.roll(k, layer, axis=0), np.roll(v, 3 * layer, axis=0)
            e.write_kv(layer, 0, kl, vl)
            om.set_kv(layer, kl, vl)
        ref_logits = np.zeros(e.n_vocab, np.float32)
        tok = 7
        for p in (pos, pos + 1):
            got = e.forward(tok, p).copy()
            want_tok = om.forward(tok, p, ref_logits)
            gx, ox = e.read_x(), om.x()
            assert np.array_equal(gx.view(np.uint32), ox.view(np.uint32)), \
                f"pos {p}: residual differs in {np.sum(gx != ox)} elements"
            diff = np.sum(got.view(np.uint32) != ref_logits.view(np.uint32))
            assert diff == 0, f"pos {p}: {diff} logits differ, max {np.max(np.abs(got - ref_logits))}"
            assert e.last_argmax == want_tok
            tok = want_tok
    finally:
        e.close()
        om.close()


def test_kv_rows_written_at_pos(engine, oracle):
    k, v = engine.read_kv(3, 5)
    assert np.all(np.isfinite(k)) and np.any(k != 0) and np.any(v != 0)


def test_greedy_chain_on_device(cuda, model_path):
    """token < 0 feeds the previous step's device argmax back without a host round trip;
    the chained run must produce the same tokens as a host-driven run."""
    from mcpm import engine as E, synth
    prompt = synth.prompt_ids(4)
    host = E.MiniCPM5Engine(device=0, max_seq=MAX_SEQ)
    chain = E.MiniCPM5Engine(device=0, max_seq=MAX_SEQ)
    assert host.load_model(model_path) and chain.load_model(model_path)
    tok = None
    for pos in range(10):
        tok = host.forward_greedy(int(prompt[pos]) if pos < 4 else tok, pos)
    for pos in range(4):
        chain.forward_async(int(prompt[pos]), pos)
    for pos in range(4, 9):
        chain.forward_async(-1, pos)
    chain.sync()
    assert chain.forward_greedy(-1, 9) == tok
    host.close()
    chain.close()


def test_errors_are_reported(engine):
    from mcpm import engine as E
    with pytest.raises(E.MCPMError) as ei:
        engine.forward(0, MAX_SEQ)
    assert ei.value.status == E.CTX_OVERFLOW
    with pytest.raises(E.MCPMError) as ei:
        engine.forward(engine.n_vocab, 0)
    assert ei.value.status == E.BAD_TOKEN
    # the engine keeps working after rejected calls
    assert isinstance(engine.forward_greedy(1, 0), int)


def test_bad_file(cuda, tmp_path):
    from mcpm import engine as E
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\xff" * 64)
    e = E.MiniCPM5Engine(device=0, max_seq=8)
    assert not e.load_model(str(p))
    with pytest.raises(E.MCPMError) as ei:
        e.forward(1, 0)
    assert ei.value.status == E.NOT_LOADED
    e.close()


def test_cpp_facade_token_loop(cuda, model_path, tmp_path):
    """A token loop written against the reference's MiniCPM5Engine interface (C++ facade over
    the C ABI) produces the same greedy tokens as the Python binding."""
    import subprocess
    from mcpm import engine as E, synth
    from test_abi import facade_build
    exe = facade_build(tmp_path)
    prompt = [int(t) for t in synth.prompt_ids(5)]
    r = subprocess.run([exe, model_path, "4"] + [str(t) for t in prompt], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = [int(v) for v in r.stdout.split()]
    e = E.MiniCPM5Engine(device=0, max_seq=16)
    assert e.load_model(model_path)
    want, tok = [], None
    for pos in range(9):
        tok = e.forward_greedy(prompt[pos] if pos < 5 else tok, pos)
        want.append(tok)
    e.close()
    assert got == want


def test_cpp_sampler_loop_device_logits(cuda, oracle, model_path, tmp_path):
    """The reference's sampling loop (engine.forward, then Sampler::sample on the returned
    vector) through the C++ facades: with the logits copied to the host, left on the device
    (set_host_logits(false)), or copied into the caller's own vector, the same seeded draws
    give the same tokens, and each equals the C restatement's top-p draw on its logits."""
    import subprocess
    import oracle as O
    from mcpm import synth
    from test_abi import facade_build
    exe = facade_build(tmp_path, "sampler_driver")
    prompt = [int(t) for t in synth.prompt_ids(5, seed=31)]
    temp, top_p, seed, n_gen = 30.0, 0.95, 7, 4   # temperature 30 spreads this model's logits
    runs = {}
    for mode in ("host", "device", "copy"):
        r = subprocess.run([exe, model_path, mode, str(n_gen), str(temp), str(top_p), str(seed)] +
                           [str(t) for t in prompt], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        runs[mode] = [(int(a), float(b)) for a, b in (ln.split() for ln in r.stdout.split("\n") if ln.strip())]
    assert runs["host"] == runs["device"] == runs["copy"]
    toks = [t for t, _ in runs["host"]]
    assert len(set(toks)) > 1
    om = O.OracleModel(oracle, model_path, 16)
    om.set_order(O.Oracle.ORDER_BATCH)   # the facade's engine runs the default (block) order
    lg = np.zeros(130560, np.float32)
    inputs = prompt + toks[:-1]
    k = 0
    for pos, t in enumerate(inputs):
        om.forward(t, pos, lg)
        if pos >= len(prompt) - 1:
            tok, r = runs["host"][k]
            assert oracle.sample_top_p(lg, temp, top_p, r)[0] == tok
            k += 1
    om.close()


@pytest.mark.parametrize("n_prompt,pos0,order", [(5, 0, "block"), (64, 0, "block"), (150, 0, "block"),
                                                 (70, 9, "block"), (5, 0, "avx2"), (150, 0, "avx2"),
                                                 (70, 9, "avx2")])
def test_batched_prefill_equals_token_by_token(cuda, model_path, n_prompt, pos0, order):
    """mcpm_prefill (the prompt as batched steps of up to 64 positions sharing the engine's KV
    cache) against one mcpm_forward per position, in either GEMV order (block: tcgen05 GEMMs and
    the decode kernel's warp GEMVs; avx2: mma.sync GEMMs and the eight-lane GEMVs): the last
    position's logits, every K/V row written and the greedy continuation are bit-identical."""
    from mcpm import engine as E, synth
    prompt = [int(t) for t in synth.prompt_ids(pos0 + n_prompt, seed=77)]
    max_seq = pos0 + n_prompt + 8
    a = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=gemm_of(order))
    b = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=gemm_of(order))
    try:
        assert a.load_model(model_path) and b.load_model(model_path)
        for pos in range(pos0):   # both engines decode the first pos0 positions one by one
            a.forward_async(prompt[pos], pos)
            b.forward_async(prompt[pos], pos)
        a.sync()
        b.sync()
        tok_a, lg_a = a.prefill(prompt[pos0:], pos0)
        for pos in range(pos0, pos0 + n_prompt):
            lg_b = b.forward(prompt[pos], pos)
        assert np.array_equal(lg_a.view(np.uint32), lg_b.view(np.uint32))
        assert tok_a == b.last_argmax
        for layer in (0, 17, 41):
            for pos in (pos0, pos0 + n_prompt // 2, pos0 + n_prompt - 1):
                ka, va = a.read_kv(layer, pos)
                kb, vb = b.read_kv(layer, pos)
                assert np.array_equal(ka, kb) and np.array_equal(va, vb)
        pos = pos0 + n_prompt
        for _ in range(3):   # greedy continuation from the device-resident token
            assert a.forward_greedy(-1, pos) == b.forward_greedy(-1, pos)
            pos += 1
    finally:
        a.close()
        b.close()


def test_prefill_argument_errors(cuda, model_path):
    from mcpm import engine as E
    e = E.MiniCPM5Engine(device=0, max_seq=16)
    try:
        assert e.load_model(model_path)
        with pytest.raises(E.MCPMError) as ei:
            e.prefill([1] * 10, 8)
        assert ei.value.status == E.CTX_OVERFLOW
        with pytest.raises(E.MCPMError) as ei:
            e.prefill([1, 130560], 0)
        assert ei.value.status == E.BAD_TOKEN
    finally:
        e.close()


def test_kv_snapshot_restore_session(cuda, model_path):
    """A session snapshot restored into the same engine or into a second one continues the
    decode exactly: a second turn prefilled after the restore gives the same logits as the
    uninterrupted session."""
    from mcpm import engine as E, synth
    turn1 = [int(t) for t in synth.prompt_ids(40, seed=5)]
    turn2 = [int(t) for t in synth.prompt_ids(12, seed=6)]
    a = E.MiniCPM5Engine(device=0, max_seq=80)
    b = E.MiniCPM5Engine(device=0, max_seq=64)
    try:
        assert a.load_model(model_path) and b.load_model(model_path)
        a.prefill(turn1, 0, logits=False)
        n = len(turn1)
        snap = a.kv_snapshot(n)
        assert snap.size == 42 * 2 * n * 256
        _, want = a.prefill(turn2, n)            # the uninterrupted session
        a.prefill([7, 8, 9], n)                  # another branch overwrites positions n..n+2
        a.kv_restore(n, snap)
        _, again = a.prefill(turn2, n)
        assert np.array_equal(again.view(np.uint32), want.view(np.uint32))
        b.kv_restore(n, snap)                    # a second engine continues the same session
        _, other = b.prefill(turn2, n)
        assert np.array_equal(other.view(np.uint32), want.view(np.uint32))
        with pytest.raises(E.MCPMError) as ei:
            b.kv_restore(65, np.zeros(42 * 2 * 65 * 256, np.float32))
        assert ei.value.status == E.CTX_OVERFLOW
    finally:
        a.close()
        b.close()


# ------------------------------------------------------------------ fp16 KV cache option
def _f16_engine(model_path, max_seq, batch_gemm=None):
    from mcpm import engine as E
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq, kv_type=E.KV_F16,
                         batch_gemm=E.GEMM_MMA if batch_gemm is None else batch_gemm)
    assert e.load_model(model_path)
    return e


def test_f16_kv_forward_bitexact_vs_restatement(cuda, oracle, model_path):
    """kv_type MCPM_KV_F16: K and V rounded to half precision (nearest even) when a step writes
    them, read back exactly, attention in fp32.  The restatement with the same option gives
    bit-identical residuals, logits, cache rows and greedy tokens."""
    import oracle as O
    from mcpm import synth
    e = _f16_engine(model_path, MAX_SEQ)
    om = O.OracleModel(oracle, model_path, MAX_SEQ, kv_f16=True)
    try:
        prompt = synth.prompt_ids(N_PROMPT)
        ref_logits = np.zeros(e.n_vocab, np.float32)
        tok = None
        for pos in range(N_PROMPT + N_GEN):
            t = int(prompt[pos]) if pos < N_PROMPT else tok
            got = e.forward(t, pos).copy()
            want_tok = om.forward(t, pos, ref_logits)
            assert np.array_equal(e.read_x().view(np.uint32), om.x().view(np.uint32)), f"pos {pos}"
            diff = np.sum(got.view(np.uint32) != ref_logits.view(np.uint32))
            assert diff == 0, f"pos {pos}: {diff} logits differ"
            assert e.last_argmax == want_tok
            tok = want_tok
        k, v = e.read_kv(5, 3)   # stored rows are half-representable
        assert np.array_equal(k.astype(np.float16).astype(np.float32), k)
        assert np.array_equal(v.astype(np.float16).astype(np.float32), v)
        assert np.any(k != 0)
    finally:
        e.close()
        om.close()


@pytest.mark.parametrize("pos", [300, 1000, 10300])
def test_f16_kv_late_steps_bitexact_vs_restatement(cuda, oracle, model_path, pos):
    """Late positions over a seeded fp16 cache: every attention chunking of the decode kernel
    reading half rows (mcpm_write_kv rounds the seeded rows the way a step rounds its own)."""
    import oracle as O
    from mcpm import spec
    max_seq = pos + 2
    e = _f16_engine(model_path, max_seq)
    om = O.OracleModel(oracle, model_path, max_seq, kv_f16=True)
    try:
        rng = np.random.default_rng(pos + 1)
        k = rng.normal(0, 1, (pos, 256)).astype(np.float32)
        v = rng.normal(0, 1, (pos, 256)).astype(np.float32)
        kh, vh = k.astype(np.float16).astype(np.float32), v.astype(np.float16).astype(np.float32)
        for layer in range(spec.N_LAYER):
            e.write_kv(layer, 0, np.roll(k, layer, axis=0), np.roll(v, 3 * layer, axis=0))
            om.set_kv(layer, np.roll(kh, layer, axis=0), np.roll(vh, 3 * layer, axis=0))
        gk, gv = e.read_kv(7, pos - 1)
        assert np.array_equal(gk, np.roll(kh, 7, axis=0)[pos - 1]) and np.array_equal(gv, np.roll(vh, 21, axis=0)[pos - 1])
        ref_logits = np.zeros(e.n_vocab, np.float32)
        tok = 7
        for p in (pos, pos + 1):
            got = e.forward(tok, p).copy()
            want_tok = om.forward(tok, p, ref_logits)
            assert np.array_equal(e.read_x().view(np.uint32), om.x().view(np.uint32)), f"pos {p}"
            diff = np.sum(got.view(np.uint32) != ref_logits.view(np.uint32))
            assert diff == 0, f"pos {p}: {diff} logits differ"
            assert e.last_argmax == want_tok
            tok = want_tok
    finally:
        e.close()
        om.close()


def test_f16_kv_prefill_snapshot_and_accuracy(cuda, model_path):
    """fp16 cache: batched prefill equals one forward per position bit for bit, a snapshot is half
    the fp32 size and restores exactly, and the logits stay close to the fp32 cache's (the only
    change is the rounding of K and V to 11 significant bits)."""
    from mcpm import engine as E, synth
    prompt = [int(t) for t in synth.prompt_ids(90, seed=31)]
    a = _f16_engine(model_path, 128)
    b = _f16_engine(model_path, 128)
    c = E.MiniCPM5Engine(device=0, max_seq=128)
    try:
        assert c.load_model(model_path)
        tok_a, lg_a = a.prefill(prompt, 0)
        for pos, t in enumerate(prompt):
            lg_b = b.forward(t, pos).copy()
            lg_c = c.forward(t, pos).copy()
        assert np.array_equal(lg_a.view(np.uint32), lg_b.view(np.uint32)) and tok_a == b.last_argmax
        snap = a.kv_snapshot(len(prompt))
        assert snap.dtype == np.float16 and snap.nbytes == 42 * 2 * len(prompt) * 256 * 2
        b.kv_restore(len(prompt), snap)
        assert a.forward_greedy(-1, len(prompt)) == b.forward_greedy(-1, len(prompt))
        # fp16 rounding of K and V against the fp32 cache: relative logit error well under 1%
        rel = np.max(np.abs(lg_a - lg_c)) / np.max(np.abs(lg_c))
        assert rel < 1e-2, rel
    finally:
        a.close()
        b.close()
        c.close()


def test_kv_type_validated(cuda):
    from mcpm import engine as E
    with pytest.raises(E.MCPMError) as ei:
        E.MiniCPM5Engine(device=0, max_seq=16, kv_type=2)
    assert ei.value.status == E.BAD_ARG


@pytest.mark.parametrize("pos0", [0, 290])
def test_schedule_options_bitexact(cuda, model_path, pos0):
    """Decode schedule options (mcpm_config::sched: L2 prefetch, head-pair attention combiners at
    every context length) change when copies are issued and who combines the attention chunks,
    never the arithmetic: logits are bit-identical to the default schedule.  pos0 = 290 runs 10
    attention chunks, combined by every CTA by default and by the combiners with option 2."""
    from mcpm import engine as E, spec, synth
    scheds = (0, 1, 2, 3, 4, 6)
    max_seq = pos0 + 40
    engs = [E.MiniCPM5Engine(device=0, max_seq=max_seq, sched=s) for s in scheds]
    try:
        for e in engs:
            assert e.load_model(model_path)
        if pos0:
            rng = np.random.default_rng(11)
            k = rng.normal(0, 1, (pos0, 256)).astype(np.float32)
            v = rng.normal(0, 1, (pos0, 256)).astype(np.float32)
            for layer in range(spec.N_LAYER):
                for e in engs:
                    e.write_kv(layer, 0, np.roll(k, layer, axis=0), np.roll(v, layer, axis=0))
        prompt = synth.prompt_ids(24, seed=99)
        for i in range(24):
            outs = [e.forward(int(prompt[i]), pos0 + i).copy() for e in engs]
            for s, o in zip(scheds[1:], outs[1:]):
                assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32)), f"sched {s} pos {pos0 + i}"
    finally:
        for e in engs:
            e.close()


@pytest.mark.parametrize("n_prompt", [6, 70])
def test_prefill_tcgen05_vs_restatement(cuda, oracle, model_path, n_prompt):
    """Prefill on the tcgen05 batched GEMM (block-order fp32 over exact block sums) against the
    restatement stepping the same positions in its BATCH order: last logits, greedy token and
    K/V rows bit for bit; the decode that follows (batch-1 kernel) continues in the same order."""
    import oracle as O
    from mcpm import engine as E, synth
    prompt = [int(t) for t in synth.prompt_ids(n_prompt, seed=41)]
    max_seq = n_prompt + 8
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=E.GEMM_TCGEN05)
    om = O.OracleModel(oracle, model_path, max_seq)
    try:
        assert e.load_model(model_path)
        tok, lg = e.prefill(prompt, 0)
        om.set_order(O.Oracle.ORDER_BATCH)
        ref = np.zeros(e.n_vocab, np.float32)
        for pos, t in enumerate(prompt):
            want = om.forward(t, pos, ref)
        diff = np.sum(lg.view(np.uint32) != ref.view(np.uint32))
        assert diff == 0, f"{diff} logits differ, max {np.max(np.abs(lg - ref))}"
        assert tok == want
        pos = n_prompt
        for _ in range(3):
            got = e.forward_greedy(tok, pos)
            want = om.forward(tok, pos, ref)
            assert got == want
            assert np.array_equal(e.read_x().view(np.uint32), om.x().view(np.uint32))
            tok, pos = got, pos + 1
    finally:
        e.close()
        om.close()
