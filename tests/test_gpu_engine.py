"""Whole-forward parity on the GPU through the C ABI.

The CUDA decode path and the C restatement follow the same canonical numerics, so logits,
the residual stream, K/V cache rows and greedy tokens are compared for exact equality.
The restatement itself is checked against the reference build in test_oracle_vs_reference.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_PROMPT, N_GEN = 12, 8
MAX_SEQ = 64


@pytest.fixture(scope="module")
def engine(cuda, model_path):
    from mcpm import engine as E
    e = E.MiniCPM5Engine(device=0, max_seq=MAX_SEQ)
    assert e.load_model(model_path)
    yield e
    e.close()


@pytest.fixture(scope="module")
def oracle_model(oracle, model_path):
    import oracle as O
    return O.OracleModel(oracle, model_path, MAX_SEQ)


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


@pytest.mark.parametrize("pos", [300, 1000, 3000, 8200, 10300])
def test_late_steps_bitexact_vs_restatement(cuda, oracle, model_path, pos):
    """Two decode steps at a late position over a seeded cache (the same random K/V rows
    0..pos-1 in the engine and in the restatement), covering every attention path of the
    decode kernel: 300 positions (32-row chunks, 10 chunks combined in the o_proj prologue
    behind a grid barrier), 1000 (32-row chunks, 32 chunks: head-pair combiners polled
    without a barrier), 3000 / 8200 (64- / 160-row chunks), 10300 (192-row chunks, two
    staging rounds)."""
    import oracle as O
    from mcpm import engine as E, spec
    max_seq = pos + 2
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq)
    assert e.load_model(model_path)
    om = O.OracleModel(oracle, model_path, max_seq)
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
