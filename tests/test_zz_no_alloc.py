"""mcpm_attention_noalloc: the attention op for callers that cannot allocate device memory
(code inside another component's graph capture, hosts that own every allocation, loops that
must not call the allocator).  Its workspace is a fixed array in the library's static device
memory; this test calls it through the C ABI twice in a row and requires exactly the
results of mcpm_attention (the tolerance every attention test here uses: bit equality).
Collected last so that a stop-at-first-failure run has already run every other test."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(lib_fn, cuda, tensors, pos, max_seq):
    q, k, v, kc, vc = tensors
    out = cuda.zeros(2048, dtype=cuda.float32, device="cuda")
    oq = cuda.zeros(8 * 292, dtype=cuda.uint8, device="cuda")
    st = lib_fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, max_seq, out.data_ptr(),
                oq.data_ptr(), None)
    cuda.cuda.synchronize()
    return st, out.cpu().numpy(), oq.cpu().numpy()


def test_noalloc_attention_matches_allocating_op_twice(cuda):
    from mcpm import engine as E
    lib = E.load_library()
    max_seq = 3000
    rng = np.random.default_rng(77)
    host = [rng.normal(0, 3, n).astype(np.float32) for n in (2048, 256, 256)]
    caches = [rng.normal(0, 3, (max_seq, 256)).astype(np.float32) for _ in range(2)]

    def dev_inputs():
        return [cuda.from_numpy(a.copy()).cuda() for a in host + caches]

    ref_in, new_in = dev_inputs(), dev_inputs()
    for pos in (2500, 2501):   # two calls in a row; the second sees the first call's workspace contents
        st_ref, out_ref, q8_ref = _call(lib.mcpm_attention, cuda, ref_in, pos, max_seq)
        st_new, out_new, q8_new = _call(lib.mcpm_attention_noalloc, cuda, new_in, pos, max_seq)
        assert st_ref == E.OK and st_new == E.OK
        assert np.array_equal(out_new.view(np.uint32), out_ref.view(np.uint32))
        assert np.array_equal(q8_new, q8_ref)
    assert np.array_equal(new_in[3].cpu().numpy(), ref_in[3].cpu().numpy())   # K rows appended alike


def test_noalloc_attention_rejects_context_beyond_workspace(cuda):
    from mcpm import engine as E
    lib = E.load_library()
    t = cuda.zeros(4096, dtype=cuda.float32, device="cuda")
    p = t.data_ptr()
    assert lib.mcpm_attention_noalloc(p, p, p, p, p, 16384, 20000, p, None, None) == E.BAD_ARG
    # pos beyond a cache that is itself too large: both ops report the cache size first
    assert lib.mcpm_attention(p, p, p, p, p, 20000, 20000, p, None, None) == E.BAD_ARG
    assert lib.mcpm_attention_noalloc(p, p, p, p, p, 20000, 20000, p, None, None) == E.BAD_ARG
    assert lib.mcpm_attention(p, p, p, p, p, 9, 9, p, None, None) == E.CTX_OVERFLOW
    assert lib.mcpm_attention_noalloc(p, p, p, p, p, 9, 9, p, None, None) == E.CTX_OVERFLOW
