"""Top-p sampler (Sampler::sample, src/sampler.cpp:8-72).

CPU: the C restatement's canonical draw against a direct port of the reference's sequential
algorithm (float32 sums in index / sorted order, libm exp).  The two differ only in fp32
summation order and exp, so for the same uniform r they pick the same token unless r lies
within rounding distance of a cumulative boundary.

GPU: the device sampler against the restatement, token and kept count bit for bit."""
import numpy as np
import pytest


def reference_sample(logits, temperature, top_p, r):
    """Sampler::sample with the draw r given (the reference's sequential fp32 order)."""
    f32 = np.float32
    inv = f32(1.0) / f32(temperature) if temperature > 0 else f32(1.0)
    apply = temperature != 1.0 and temperature > 0
    v = (logits.astype(np.float32) * inv).astype(np.float32) if apply else logits.astype(np.float32)
    m = f32(-1e9)
    for x in v:
        if x > m:
            m = x
    p = np.exp((v - m).astype(np.float32)).astype(np.float32)
    s = f32(0.0)
    for x in p:
        s = f32(s + x)
    p = (p / s).astype(np.float32)
    order = np.arange(p.size)
    if 0.0 < top_p < 1.0:
        order = np.lexsort((order, -p))   # descending p; ties by index (the reference's sort is unstable)
        ps = p[order]
        c = f32(0.0)
        last = ps.size - 1
        for k, x in enumerate(ps):
            c = f32(c + x)
            if c >= f32(top_p):
                last = k
                break
        order, ps = order[:last + 1], (ps[:last + 1] / c).astype(np.float32)
    else:
        ps = p
    cur = f32(0.0)
    cums = np.empty(ps.size, np.float32)
    for k, x in enumerate(ps):
        cur = f32(cur + x)
        cums[k] = cur
    hit = np.nonzero(f32(r) <= cums)[0]
    k = hit[0] if hit.size else ps.size - 1
    return int(order[k]), cums


def test_restatement_matches_reference_algorithm(oracle):
    rng = np.random.default_rng(11)
    checked = 0
    for case in range(40):
        n = int(rng.integers(50, 3000))
        logits = rng.normal(0, [0.5, 2.0, 5.0][case % 3], n).astype(np.float32)
        t = [1.0, 0.7, 1.3, 0.0][case % 4]
        tp = [0.95, 0.5, 0.9, 1.0][(case // 4) % 4]
        for r in (0.0, 0.2, 0.5, 0.77, 0.999):
            want, cums = reference_sample(logits, t, tp, r)
            got, _ = oracle.sample_top_p(logits, t, tp, r)
            if got != want:   # only allowed where r sits on a boundary within fp32 rounding
                assert np.min(np.abs(cums - np.float32(r))) < 1e-5, (case, r, got, want)
            checked += 1
    assert checked == 200


def test_restatement_edge_cases(oracle):
    lg = np.zeros(10, np.float32)   # uniform: cumulative 0.1, 0.2, ...
    assert oracle.sample_top_p(lg, 1.0, 1.0, 0.0) == (0, 10)
    assert oracle.sample_top_p(lg, 1.0, 1.0, 0.35)[0] == 3
    assert oracle.sample_top_p(lg, 1.0, 1.0, 1.0)[0] in (9,)
    one_hot = np.full(10, -1e4, np.float32)
    one_hot[7] = 5.0
    for r in (0.0, 0.5, 0.999):
        assert oracle.sample_top_p(one_hot, 1.0, 0.95, r) == (7, 1)


CASES = [(n, sd, t, tp) for n in (130560, 4097, 33) for sd in (0.3, 4.0) for t in (1.0, 0.7, 0.0)
         for tp in (0.95, 0.5, 1.0)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,sd,t,tp", CASES)
def test_device_sampler_matches_restatement(cuda, oracle, n, sd, t, tp):
    from mcpm import engine as E
    rng = np.random.default_rng(n + int(sd * 10) + int(t * 100) + int(tp * 1000))
    logits = rng.normal(0, sd, n).astype(np.float32)
    ld = cuda.from_numpy(logits).cuda()
    out = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    for r in (0.0, 0.31, 0.9, 0.99999):
        E.sample_top_p(ld.data_ptr(), n, t, tp, r, out.data_ptr())
        cuda.cuda.synchronize()
        got = tuple(int(v) for v in out.cpu().numpy())
        want = oracle.sample_top_p(logits, t, tp, r)
        assert got == want, (r, got, want)


@pytest.mark.gpu
def test_engine_sample_feeds_next_step(cuda, model_path):
    from mcpm import engine as E, synth
    e = E.MiniCPM5Engine(device=0, max_seq=16)
    assert e.load_model(model_path)
    try:
        prompt = synth.prompt_ids(3)
        for pos in range(3):
            lg = e.forward(int(prompt[pos]), pos).copy()
        tok = e.sample(1.0, 0.95, 0.42)
        import oracle as O
        assert tok == O.Oracle().sample_top_p(lg, 1.0, 0.95, 0.42)[0]
        e.forward(-1, 3)   # consumes the sampled token on the device
        assert e.read_kv(0, 3)[0].any()
    finally:
        e.close()
