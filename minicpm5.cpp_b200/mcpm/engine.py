"""Python binding of the C ABI (include/mcpm.h) through ctypes.

`MiniCPM5Engine` mirrors the reference class (include/model.h:37-70): `init_kv_cache`,
`load_model`, `forward(token_id, pos, max_seq_len)` returning the logits.  Errors raise
`MCPMError` carrying the C status.  There is no CPU fallback: without a built library
or without a CUDA device every call fails loudly.

The op functions take device pointers (ints), e.g. `torch.Tensor.data_ptr()`.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import build as _build

_lib = None

STATUS = {0: "ok", 1: "bad argument", 2: "bad file", 3: "unsupported type", 4: "context overflow",
          5: "CUDA error", 6: "NCCL error", 7: "timeout", 8: "out of memory", 9: "bad token", 10: "not loaded"}
OK, BAD_ARG, BAD_FILE, UNSUPPORTED_TYPE, CTX_OVERFLOW, CUDA_ERROR, NCCL_ERROR, TIMEOUT, OOM, BAD_TOKEN, NOT_LOADED = range(11)
ROUND_EVEN, ROUND_AWAY = 0, 1
Q4_K, Q6_K, Q8_0 = 12, 14, 8


class MCPMError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        super().__init__(f"{what}: {STATUS.get(status, status)} ({status})")
        self.status = status


class mcpm_config(C.Structure):
    _fields_ = [("device", C.c_int), ("max_seq", C.c_int), ("n_ctas", C.c_int), ("batch_gemm", C.c_int),
                ("sched", C.c_int), ("kv_type", C.c_int), ("reserved", C.c_int * 2)]


KV_F32, KV_F16 = 0, 1
GEMM_TCGEN05, GEMM_MMA = 0, 1


P, I, F = C.c_void_p, C.c_int, C.c_float

# exported symbol -> (restype, argtypes); tests check that every declared symbol exists
SIGNATURES = {
    "mcpm_status_string": (C.c_char_p, [I]),
    "mcpm_engine_create": (I, [C.POINTER(mcpm_config), C.POINTER(P)]),
    "mcpm_load_gguf": (I, [P, C.c_char_p]),
    "mcpm_init_kv": (I, [P, I]),
    "mcpm_forward": (I, [P, I, I, C.POINTER(F), C.POINTER(I)]),
    "mcpm_forward_async": (I, [P, I, I, I]),
    "mcpm_sync": (I, [P]),
    "mcpm_logits_device": (P, [P]),
    "mcpm_argmax_device": (P, [P]),
    "mcpm_read_x": (I, [P, C.POINTER(F)]),
    "mcpm_read_kv": (I, [P, I, I, C.POINTER(F), C.POINTER(F)]),
    "mcpm_write_kv": (I, [P, I, I, I, C.POINTER(F), C.POINTER(F)]),
    "mcpm_batch_init": (I, [P, I, I]),
    "mcpm_prefill": (I, [P, C.POINTER(I), I, I, C.POINTER(F), C.POINTER(I)]),
    "mcpm_kv_snapshot_bytes": (C.c_size_t, [P, I]),
    "mcpm_kv_snapshot": (I, [P, I, P, C.c_size_t]),
    "mcpm_kv_restore": (I, [P, I, P, C.c_size_t]),
    "mcpm_sample_top_p": (I, [P, I, F, F, F, P, P]),
    "mcpm_sample": (I, [P, F, F, F, C.POINTER(I)]),
    "mcpm_sample_top_p_host": (I, [C.POINTER(F), I, F, F, F, C.POINTER(I)]),
    "mcpm_rope_kv_append": (I, [P, P, P, P, P, I, I, F, P]),
    "mcpm_batch_step_async": (I, [P, C.POINTER(I), C.POINTER(I)]),
    "mcpm_batch_read": (I, [P, C.POINTER(F), C.POINTER(I)]),
    "mcpm_model_dims": (I, [P, C.POINTER(I)]),
    "mcpm_engine_stream": (P, [P]),
    "mcpm_engine_n_ctas": (I, [P]),
    "mcpm_engine_destroy": (None, [P]),
    "mcpm_quantize_q8k": (I, [P, P, I, I, P]),
    "mcpm_gemv_q8k": (I, [I, P, P, P, I, I, P]),
    "mcpm_gemv_q8k_block": (I, [I, P, P, P, I, I, P]),
    "mcpm_gemv_q8_0_f32": (I, [P, P, P, I, I, P]),
    "mcpm_gemv_blocksums": (I, [I, P, P, P, P, I, I, P]),
    "mcpm_gemv_gate_up_q8k": (I, [P, P, P, P, P, I, I, P]),
    "mcpm_rmsnorm_q8k": (I, [P, P, P, I, F, P]),
    "mcpm_swiglu_q8k": (I, [P, P, P, I, P]),
    "mcpm_gemv_q8k_timed": (I, [I, P, I, P, P, I, I, I, I, C.POINTER(F), P]),
    "mcpm_attention": (I, [P, P, P, P, P, I, I, P, P, P]),
    "mcpm_attention_noalloc": (I, [P, P, P, P, P, I, I, P, P, P]),
    "mcpm_trace_enable": (I, [P, I]),
    "mcpm_trace_read": (I, [P, C.POINTER(C.c_uint64), I]),
    "mcpm_tp_nccl_id": (I, [P]),
    "mcpm_tp_create": (I, [P, C.POINTER(P)]),
    "mcpm_tp_load_gguf": (I, [P, C.c_char_p]),
    "mcpm_tp_ipc_handle": (I, [P, P]),
    "mcpm_tp_connect": (I, [P, P, P]),
    "mcpm_tp_forward": (I, [P, I, I, C.POINTER(F), C.POINTER(I)]),
    "mcpm_tp_generate_async": (I, [P, I]),
    "mcpm_tp_sync": (I, [P]),
    "mcpm_tp_read_tokens": (I, [P, I, I, C.POINTER(I)]),
    "mcpm_tp_info": (I, [P, C.POINTER(I)]),
    "mcpm_tp_reset": (I, [P]),
    "mcpm_tp_profile": (I, [P, I, C.POINTER(F), C.POINTER(F)]),
    "mcpm_tp_stream": (P, [P]),
    "mcpm_tp_destroy": (None, [P]),
}


def lib_path() -> str:
    return _build.LIB


def load_library(build_if_needed: bool = True) -> C.CDLL:
    """Loads libmcpm.so (building it first when sources changed)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.build() if build_if_needed else _build.LIB
    if not os.path.exists(path):
        raise MCPMError(CUDA_ERROR, f"native library missing: {path}")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def sample_top_p(logits_ptr: int, n: int, temperature: float, top_p: float, r: float, out_ptr: int,
                 stream: int = 0) -> None:
    """Device top-p sampler (logits and out are device pointers; out receives token, kept)."""
    check(load_library().mcpm_sample_top_p(logits_ptr, n, temperature, top_p, r, out_ptr, stream),
          "mcpm_sample_top_p")


def check(status: int, what: str) -> None:
    if status != OK:
        raise MCPMError(status, what)


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


class MiniCPM5Engine:
    """Device engine behind the reference's MiniCPM5Engine interface."""

    def __init__(self, device: int = 0, max_seq: int = 0, n_ctas: int = 0, batch_gemm: int = 0, sched: int = 0,
                 kv_type: int = KV_F32):
        """batch_gemm (batched decode and prefill): GEMM_TCGEN05 (default; block-order fp32 over exact block
        sums) or GEMM_MMA (int8 mma.sync in the batch-1 decode's order: bit-identical to forward()).
        sched: decode schedule option bits (include/mcpm.h MCPM_SCHED_*; results are the same).
        kv_type: KV_F32 (the reference's fp32 cache) or KV_F16 (rows rounded to fp16 when written)."""
        self.lib = load_library()
        cfg = mcpm_config(device, max_seq, n_ctas, batch_gemm, sched, kv_type)
        self.kv_type = kv_type
        h = P()
        check(self.lib.mcpm_engine_create(C.byref(cfg), C.byref(h)), "mcpm_engine_create")
        self.h = h
        self.n_vocab = 0
        self._logits = None

    # reference: void init_kv_cache(int max_seq_len)
    def init_kv_cache(self, max_seq_len: int) -> None:
        check(self.lib.mcpm_init_kv(self.h, max_seq_len), "mcpm_init_kv")

    # reference: bool load_model(const std::string&, bool verbose)
    def load_model(self, path: str, verbose: bool = False) -> bool:
        st = self.lib.mcpm_load_gguf(self.h, path.encode())
        if st != OK:
            if verbose:
                print(f"[mcpm] load_model failed: {STATUS.get(st, st)}")
            return False
        dims = (C.c_int * 6)()
        check(self.lib.mcpm_model_dims(self.h, dims), "mcpm_model_dims")
        self.n_vocab = dims[5]
        self._logits = np.zeros(self.n_vocab, np.float32)
        return True

    # reference: const std::vector<float>& forward(int token_id, int pos, int max_seq_len)
    def forward(self, token_id: int, pos: int, max_seq_len: Optional[int] = None) -> np.ndarray:
        am = C.c_int()
        lg = _fptr(self._logits) if self._logits is not None else None
        check(self.lib.mcpm_forward(self.h, token_id, pos, lg, C.byref(am)), "mcpm_forward")
        self.last_argmax = am.value
        return self._logits

    def forward_greedy(self, token_id: int, pos: int) -> int:
        """One step returning only the device argmax (no logits copy)."""
        am = C.c_int()
        check(self.lib.mcpm_forward(self.h, token_id, pos, None, C.byref(am)), "mcpm_forward")
        return am.value

    def prefill(self, tokens, pos0: int = 0, logits: bool = True):
        """Batched prefill of positions pos0 .. pos0+len(tokens)-1: (greedy token after the last
        position, its logits or None).  Equal to len(tokens) forward() calls bit for bit."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        am = C.c_int()
        lg = _fptr(self._logits) if (logits and self._logits is not None) else None
        check(self.lib.mcpm_prefill(self.h, t.ctypes.data_as(C.POINTER(C.c_int)), t.size, pos0, lg, C.byref(am)),
              "mcpm_prefill")
        return am.value, (self._logits.copy() if lg is not None else None)

    def kv_snapshot(self, n_pos: int) -> np.ndarray:
        """KV rows of positions [0, n_pos) of every layer ([layer][K, V][pos][256], fp32 or fp16 as the
        cache holds them)."""
        nbytes = self.lib.mcpm_kv_snapshot_bytes(self.h, n_pos)
        dt = np.float16 if self.kv_type == KV_F16 else np.float32
        buf = np.zeros(nbytes // np.dtype(dt).itemsize, dt)
        check(self.lib.mcpm_kv_snapshot(self.h, n_pos, buf.ctypes.data_as(P), buf.nbytes), "mcpm_kv_snapshot")
        return buf

    def kv_restore(self, n_pos: int, snap: np.ndarray) -> None:
        snap = np.ascontiguousarray(snap, dtype=np.float16 if self.kv_type == KV_F16 else np.float32)
        check(self.lib.mcpm_kv_restore(self.h, n_pos, snap.ctypes.data_as(P), snap.nbytes), "mcpm_kv_restore")

    def forward_async(self, token_id: int, pos: int, write_logits: bool = False) -> None:
        check(self.lib.mcpm_forward_async(self.h, token_id, pos, int(write_logits)), "mcpm_forward_async")

    def sync(self) -> None:
        check(self.lib.mcpm_sync(self.h), "mcpm_sync")

    def read_x(self) -> np.ndarray:
        x = np.zeros(2048, np.float32)
        check(self.lib.mcpm_read_x(self.h, _fptr(x)), "mcpm_read_x")
        return x

    def read_kv(self, layer: int, pos: int):
        k = np.zeros(256, np.float32)
        v = np.zeros(256, np.float32)
        check(self.lib.mcpm_read_kv(self.h, layer, pos, _fptr(k), _fptr(v)), "mcpm_read_kv")
        return k, v

    # reference: Sampler::sample on the last step's logits (forward with write_logits); the
    # token also becomes the next step's input (forward with token < 0)
    def sample(self, temperature: float = 1.0, top_p: float = 0.95, r: float = 0.5) -> int:
        tok = C.c_int(-1)
        check(self.lib.mcpm_sample(self.h, temperature, top_p, r, C.byref(tok)), "mcpm_sample")
        return tok.value

    # batched decode: n_seq independent sequences in lockstep
    def batch_init(self, n_seq: int, max_seq: int) -> None:
        check(self.lib.mcpm_batch_init(self.h, n_seq, max_seq), "mcpm_batch_init")
        self.batch_n = n_seq

    def batch_step_async(self, tokens=None, pos=None) -> None:
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        p = None if pos is None else np.ascontiguousarray(pos, dtype=np.int32)
        ip = C.POINTER(C.c_int)
        check(self.lib.mcpm_batch_step_async(self.h, None if t is None else t.ctypes.data_as(ip),
                                             None if p is None else p.ctypes.data_as(ip)), "mcpm_batch_step_async")

    def batch_read(self, logits: bool = False):
        am = np.zeros(self.batch_n, np.int32)
        lg = np.zeros((self.batch_n, self.n_vocab), np.float32) if logits else None
        check(self.lib.mcpm_batch_read(self.h, None if lg is None else _fptr(lg),
                                       am.ctypes.data_as(C.POINTER(C.c_int))), "mcpm_batch_read")
        return am, lg

    def batch_step(self, tokens=None, pos=None, logits: bool = False):
        self.batch_step_async(tokens, pos)
        return self.batch_read(logits)

    def write_kv(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        assert k.shape == v.shape and k.ndim == 2 and k.shape[1] == 256
        check(self.lib.mcpm_write_kv(self.h, layer, pos0, k.shape[0], _fptr(k), _fptr(v)), "mcpm_write_kv")

    def trace_enable(self, on: bool = True) -> None:
        check(self.lib.mcpm_trace_enable(self.h, int(on)), "mcpm_trace_enable")

    def trace_read(self, n_layer: int = 42) -> np.ndarray:
        n = 3 + 2 * 5 * n_layer
        buf = (C.c_uint64 * n)()
        check(self.lib.mcpm_trace_read(self.h, buf, n), "mcpm_trace_read")
        return np.array(buf, dtype=np.uint64)

    @property
    def stream(self) -> int:
        return self.lib.mcpm_engine_stream(self.h) or 0

    @property
    def n_ctas(self) -> int:
        return self.lib.mcpm_engine_n_ctas(self.h)

    @property
    def logits_device_ptr(self) -> int:
        return self.lib.mcpm_logits_device(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.mcpm_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ ops on device pointers
def quantize_q8k(x_ptr: int, y_ptr: int, n: int, rounding: int, stream: int = 0) -> None:
    check(load_library().mcpm_quantize_q8k(x_ptr, y_ptr, n, rounding, stream), "mcpm_quantize_q8k")


def gemv_q8k(ggml_type: int, w_ptr: int, xq_ptr: int, y_ptr: int, rows: int, cols: int, stream: int = 0) -> None:
    check(load_library().mcpm_gemv_q8k(ggml_type, w_ptr, xq_ptr, y_ptr, rows, cols, stream), "mcpm_gemv_q8k")


def gemv_q8k_block(ggml_type: int, w_ptr: int, xq_ptr: int, y_ptr: int, rows: int, cols: int, stream: int = 0) -> None:
    """The same product in the engine's default block order (exact block sums, one fma per block in groups of
    four blocks): the order of the decode kernel and of the batched GEMM with GEMM_TCGEN05."""
    check(load_library().mcpm_gemv_q8k_block(ggml_type, w_ptr, xq_ptr, y_ptr, rows, cols, stream),
          "mcpm_gemv_q8k_block")


def gemv_q8_0(w_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, stream: int = 0) -> None:
    check(load_library().mcpm_gemv_q8_0_f32(w_ptr, x_ptr, y_ptr, rows, cols, stream), "mcpm_gemv_q8_0_f32")


def gemv_blocksums(ggml_type: int, w_ptr: int, xq_ptr: int, isum_ptr: int, aux_ptr: int, rows: int, cols: int,
                   stream: int = 0) -> None:
    check(load_library().mcpm_gemv_blocksums(ggml_type, w_ptr, xq_ptr, isum_ptr, aux_ptr, rows, cols, stream),
          "mcpm_gemv_blocksums")


def gemv_gate_up_q8k(wg_ptr, wu_ptr, xq_ptr, g_ptr, u_ptr, rows, cols, stream=0) -> None:
    check(load_library().mcpm_gemv_gate_up_q8k(wg_ptr, wu_ptr, xq_ptr, g_ptr, u_ptr, rows, cols, stream),
          "mcpm_gemv_gate_up_q8k")


def rmsnorm_q8k(x_ptr: int, w_ptr: int, out_ptr: int, n: int, eps: float = 1e-6, stream: int = 0) -> None:
    check(load_library().mcpm_rmsnorm_q8k(x_ptr, w_ptr, out_ptr, n, eps, stream), "mcpm_rmsnorm_q8k")


def swiglu_q8k(g_ptr: int, u_ptr: int, out_ptr: int, n: int, stream: int = 0) -> None:
    check(load_library().mcpm_swiglu_q8k(g_ptr, u_ptr, out_ptr, n, stream), "mcpm_swiglu_q8k")


ORDER_AVX2, ORDER_BLOCK = 0, 1


def gemv_q8k_timed(ggml_type, w_ptr, n_copies, xq_ptr, y_ptr, rows, cols, reps, stream=0, order=ORDER_BLOCK) -> float:
    ms = C.c_float()
    check(load_library().mcpm_gemv_q8k_timed(ggml_type, w_ptr, n_copies, xq_ptr, y_ptr, rows, cols, order, reps,
                                             C.byref(ms), stream), "mcpm_gemv_q8k_timed")
    return ms.value


def rope_kv_append(q_ptr, k_ptr, v_ptr, kc_ptr, vc_ptr, pos, max_seq, rope_base=5000000.0, stream=0) -> None:
    """apply_rope on q (16 heads) and k (2 heads) in place, then k, v written at row pos."""
    check(load_library().mcpm_rope_kv_append(q_ptr, k_ptr, v_ptr, kc_ptr, vc_ptr, pos, max_seq, rope_base, stream),
          "mcpm_rope_kv_append")


def sample_top_p_host(logits: np.ndarray, temperature: float, top_p: float, r: float) -> int:
    """Sampler::sample on host logits, run on the device (same token as the device sampler)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    tok = C.c_int()
    check(load_library().mcpm_sample_top_p_host(_fptr(lg), lg.size, temperature, top_p, r, C.byref(tok)),
          "mcpm_sample_top_p_host")
    return tok.value


def attention(q_ptr, k_ptr, v_ptr, kc_ptr, vc_ptr, pos, max_seq, out_ptr, out_q8k_ptr=None, stream=0) -> None:
    check(load_library().mcpm_attention(q_ptr, k_ptr, v_ptr, kc_ptr, vc_ptr, pos, max_seq, out_ptr, out_q8k_ptr,
                                        stream), "mcpm_attention")
