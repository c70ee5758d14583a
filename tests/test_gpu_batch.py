"""Batched decode (n_seq independent sequences in lockstep) on the GPU against the C
restatement, one restatement model per sequence, bit for bit.  The mma.sync GEMMs keep the
batch-1 decode's eight AVX2 lane partials per block (restatement order AVX2: every sequence
equals a batch-1 decode of it); the tcgen05 GEMM scales exact block sums with one fma per
block (restatement order BATCH)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gemm", [1, 0], ids=["mma", "tcgen05"])
@pytest.mark.parametrize("n_seq,n_prompt,n_gen,check", [(5, 6, 4, None), (64, 2, 1, (0, 9, 31, 40, 63)),
                                                        (37, 2, 1, (0, 31, 32, 36)), (20, 2, 1, (0, 7, 8, 19)),
                                                        (12, 2, 1, (0, 8, 11))])
def test_batch_decode_bitexact(cuda, oracle, model_path, n_seq, n_prompt, n_gen, check, gemm):
    import oracle as O
    from mcpm import engine as E
    max_seq = 32
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=gemm)
    assert e.load_model(model_path)
    e.batch_init(n_seq, max_seq)
    seqs = list(range(n_seq)) if check is None else list(check)
    oms = {s: O.OracleModel(oracle, model_path, max_seq) for s in seqs}
    for om in oms.values():   # tcgen05: the batched path's own fp32 order over exact block sums
        om.set_order(O.Oracle.ORDER_BATCH if gemm == E.GEMM_TCGEN05 else O.Oracle.ORDER_AVX2)
    rng = np.random.default_rng(n_seq)
    prompts = rng.integers(0, e.n_vocab, (n_seq, n_prompt)).astype(np.int32)
    ref = np.zeros(e.n_vocab, np.float32)
    toks = None
    try:
        for step in range(n_prompt + n_gen):
            if step < n_prompt:
                tin = prompts[:, step]
                am, lg = e.batch_step(tin, np.full(n_seq, step, np.int32), logits=True)
            else:   # greedy continuation fed back on the device
                tin = toks
                am, lg = e.batch_step(None, None, logits=True)
            for s in seqs:
                want = oms[s].forward(int(tin[s]), step, ref)
                diff = np.sum(lg[s].view(np.uint32) != ref.view(np.uint32))
                assert diff == 0, f"seq {s} step {step}: {diff} logits differ, max {np.max(np.abs(lg[s] - ref))}"
                assert am[s] == want, f"seq {s} step {step}: token {am[s]} vs {want}"
            toks = am.copy()
    finally:
        e.close()
        for om in oms.values():
            om.close()


@pytest.mark.parametrize("gemm", [1, 0], ids=["mma", "tcgen05"])
def test_batch_decode_f16_kv_bitexact(cuda, oracle, model_path, gemm):
    """Batched decode over fp16 cache rows (kv_type MCPM_KV_F16) against the restatement with
    the same option."""
    import oracle as O
    from mcpm import engine as E
    n_seq, max_seq, n_steps = 9, 24, 6
    e = E.MiniCPM5Engine(device=0, max_seq=max_seq, batch_gemm=gemm, kv_type=E.KV_F16)
    assert e.load_model(model_path)
    e.batch_init(n_seq, max_seq)
    seqs = (0, 4, 8)
    oms = {s: O.OracleModel(oracle, model_path, max_seq, kv_f16=True) for s in seqs}
    for om in oms.values():
        om.set_order(O.Oracle.ORDER_BATCH if gemm == E.GEMM_TCGEN05 else O.Oracle.ORDER_AVX2)
    prompts = np.random.default_rng(3).integers(0, e.n_vocab, (n_seq, 3)).astype(np.int32)
    ref = np.zeros(e.n_vocab, np.float32)
    toks = None
    try:
        for step in range(n_steps):
            if step < 3:
                tin = prompts[:, step]
                am, lg = e.batch_step(tin, np.full(n_seq, step, np.int32), logits=True)
            else:
                tin = toks
                am, lg = e.batch_step(None, None, logits=True)
            for s in seqs:
                want = oms[s].forward(int(tin[s]), step, ref)
                assert np.array_equal(lg[s].view(np.uint32), ref.view(np.uint32)), f"seq {s} step {step}"
                assert am[s] == want
            toks = am.copy()
    finally:
        e.close()
        for om in oms.values():
            om.close()


def test_batch_rejects_bad_arguments(cuda, model_path):
    from mcpm import engine as E
    e = E.MiniCPM5Engine(device=0, max_seq=16)
    assert e.load_model(model_path)
    try:
        with pytest.raises(E.MCPMError):
            e.batch_init(65, 16)   # more than 64 sequences
        e.batch_init(2, 4)
        with pytest.raises(E.MCPMError) as ei:
            e.batch_step_async([1, 2], [0, 4])   # position beyond the batch cache
        assert ei.value.status == E.CTX_OVERFLOW
        with pytest.raises(E.MCPMError) as ei:
            e.batch_step_async([1, e.n_vocab], [0, 0])
        assert ei.value.status == E.BAD_TOKEN
    finally:
        e.close()
