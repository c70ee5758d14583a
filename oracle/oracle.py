"""TEST INFRASTRUCTURE ONLY -- the parity checker, never shipped or measured as the product.

ctypes access to the two CPU checkers built by ``oracle/Makefile``:

* ``Ref``    -- the reference engine compiled from its own sources (``_ref/libref_minicpm5.so``),
* ``Oracle`` -- this project's plain-C restatement (``_build/liboracle.so``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libref_minicpm5.so")
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
# The reference source tree: $MCPM_REFERENCE_TREE, else a directory `reference` beside this
# repository's root.  Only the build of the checker library reads it.
REFERENCE_TREE = os.environ.get("MCPM_REFERENCE_TREE") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                         "reference")

_pkg = os.path.join(os.path.dirname(HERE), "minicpm5.cpp_b200")
if _pkg not in sys.path:
    sys.path.insert(0, _pkg)
from mcpm import gguf, spec  # noqa: E402

Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292

P = C.c_void_p
F = C.POINTER(C.c_float)
I32 = C.POINTER(C.c_int32)


def build(reference: bool = True) -> None:
    """Compile the C restatement and, where the reference tree exists, the reference library."""
    targets = ["oracle"]
    if reference and os.path.isdir(os.path.join(REFERENCE_TREE, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REFERENCE_TREE}"] + targets, check=True)


def have_ref() -> bool:
    return os.path.exists(REF_SO)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(P)


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(F)


class Ref:
    """The reference CPU build (AVX2 + OpenMP) behind its own functions."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        L.ref_engine_create.restype = P
        L.ref_engine_create.argtypes = [C.c_char_p, C.c_int]
        L.ref_engine_destroy.argtypes = [P]
        L.ref_forward.restype = C.c_int
        L.ref_forward.argtypes = [P, C.c_int, C.c_int, F]
        L.ref_omp_threads.restype = C.c_int
        for n in ("ref_quantize_row_q8k_avx2", "ref_quantize_row_q8k_scalar"):
            getattr(L, n).argtypes = [F, P, C.c_int]
        for n in ("ref_gemv_q4k_q8k", "ref_gemv_q6k_q8k"):
            getattr(L, n).argtypes = [P, P, F, C.c_int, C.c_int]
        for n in ("ref_gemv_q4k_f32", "ref_gemv_q6k_f32", "ref_gemv_q8_0"):
            getattr(L, n).argtypes = [P, F, F, C.c_int, C.c_int]
        L.ref_gemv_qkv.argtypes = [P, P, P, C.c_int, P, F, F, F, C.c_int, C.c_int, C.c_int]
        L.ref_gemv_gate_up.argtypes = [P, P, P, F, F, C.c_int, C.c_int]
        L.ref_rmsnorm.argtypes = [F, F, F, C.c_int]
        L.ref_rmsnorm_quantize_q8k.argtypes = [P, F, F, C.c_int]
        L.ref_swiglu_quantize_q8k.argtypes = [P, F, F, C.c_int]
        L.ref_apply_rope.argtypes = [F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.ref_attention.argtypes = [F, F, F, F, F, F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_get_embedding.argtypes = [F, P, C.c_char_p, C.c_int, C.c_int, C.c_int]
        L.ref_dot_row_q4k_scalar.restype = C.c_float
        L.ref_dot_row_q4k_scalar.argtypes = [P, P, C.c_int]
        L.ref_dot_row_q6k_scalar.restype = C.c_float
        L.ref_dot_row_q6k_scalar.argtypes = [P, P, C.c_int]
        L.ref_silu.restype = C.c_float
        L.ref_silu.argtypes = [C.c_float]

    def threads(self) -> int:
        return self.lib.ref_omp_threads()

    def quantize_q8k(self, x: np.ndarray, scalar: bool = False) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(x.size // 256, Q8K_DTYPE)
        fn = self.lib.ref_quantize_row_q8k_scalar if scalar else self.lib.ref_quantize_row_q8k_avx2
        fn(_fptr(x), _ptr(y), x.size)
        return y

    def gemv_q8k(self, ggml_type: int, w: np.ndarray, xq: np.ndarray, rows: int, cols: int) -> np.ndarray:
        y = np.zeros(rows, np.float32)
        fn = self.lib.ref_gemv_q4k_q8k if ggml_type == spec.GGML_Q4_K else self.lib.ref_gemv_q6k_q8k
        fn(_ptr(w), _ptr(xq), _fptr(y), rows, cols)
        return y

    def gemv_f32(self, ggml_type: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(rows, np.float32)
        fn = {spec.GGML_Q4_K: self.lib.ref_gemv_q4k_f32, spec.GGML_Q6_K: self.lib.ref_gemv_q6k_f32,
              spec.GGML_Q8_0: self.lib.ref_gemv_q8_0}[ggml_type]
        fn(_ptr(w), _fptr(x), _fptr(y), rows, cols)
        return y

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.zeros_like(x)
        self.lib.ref_rmsnorm(_fptr(out), _fptr(x), _fptr(w), x.size)
        return out

    def rmsnorm_q8k(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.zeros(x.size // 256, Q8K_DTYPE)
        self.lib.ref_rmsnorm_quantize_q8k(_ptr(y), _fptr(x), _fptr(w), x.size)
        return y

    def swiglu_q8k(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        y = np.zeros(g.size // 256, Q8K_DTYPE)
        self.lib.ref_swiglu_quantize_q8k(_ptr(y), _fptr(g), _fptr(u), g.size)
        return y

    def rope(self, v, pos, n_heads, head_dim=spec.HEAD_DIM, base=spec.ROPE_BASE):
        v = np.array(v, np.float32).copy()
        for h in range(n_heads):
            self.lib.ref_apply_rope(_fptr(v), v.size, pos, h, head_dim, base)
        return v

    def embedding(self, w, type_str: str, token: int, dim=spec.N_EMBD, vocab=spec.N_VOCAB):
        out = np.zeros(dim, np.float32)
        self.lib.ref_get_embedding(_fptr(out), _ptr(w), type_str.encode(), token, dim, vocab)
        return out


class RefEngine:
    """MiniCPM5Engine from the reference build, loaded on a GGUF file."""

    def __init__(self, ref: Ref, path: str, max_seq: int):
        self.ref = ref
        self.h = ref.lib.ref_engine_create(path.encode(), max_seq)
        if not self.h:
            raise RuntimeError("reference load_model failed")

    def forward(self, token: int, pos: int, logits: Optional[np.ndarray] = None) -> int:
        return self.ref.lib.ref_forward(self.h, token, pos, _fptr(logits) if logits is not None else None)

    def close(self):
        if self.h:
            self.ref.lib.ref_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class orc_model_desc(C.Structure):
    _fields_ = [("base", P), ("tok_embd", C.c_uint64), ("out_norm", C.c_uint64), ("output", C.c_uint64),
                ("tok_embd_type", C.c_int), ("output_type", C.c_int),
                ("layer", (C.c_uint64 * 9) * 64), ("layer_type", (C.c_int * 9) * 64),
                ("n_layer", C.c_int), ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_head", C.c_int),
                ("n_head_kv", C.c_int), ("n_vocab", C.c_int), ("rope_base", C.c_float), ("eps", C.c_float),
                ("kv_f16", C.c_int)]


class Oracle:
    """This project's plain-C restatement."""

    ROUND_EVEN, ROUND_AWAY = 0, 1
    ORDER_SCALAR, ORDER_AVX2, ORDER_BATCH = 0, 1, 2

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(reference=False)
        L = self.lib = C.CDLL(path)
        L.orc_fp16_to_fp32.restype = C.c_float
        L.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        L.orc_quantize_q8k.argtypes = [F, C.c_int, P, C.c_int, C.c_int]
        L.orc_blocksums.argtypes = [C.c_int, P, P, C.c_int, C.c_int, I32, I32]
        L.orc_gemv_q4k_q8k.argtypes = [P, P, F, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_gemv_q6k_q8k.argtypes = [P, P, F, C.c_int, C.c_int, C.c_int]
        L.orc_gemv_q8_0.argtypes = [P, F, F, C.c_int, C.c_int]
        L.orc_rmsnorm_q8k.argtypes = [F, F, C.c_int, C.c_float, P]
        L.orc_rmsnorm.argtypes = [F, F, C.c_int, C.c_float, F]
        L.orc_swiglu_q8k.argtypes = [F, F, C.c_int, P]
        L.orc_rope.argtypes = [F, C.c_int, C.c_int, C.c_int, C.c_float]
        L.orc_attention.restype = C.c_int
        L.orc_attention.argtypes = [F, F, F, F, F, F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.orc_embedding.argtypes = [P, C.c_int, C.c_int, C.c_int, F]
        L.orc_create.restype = P
        L.orc_create.argtypes = [C.POINTER(orc_model_desc), C.c_int]
        L.orc_destroy.argtypes = [P]
        L.orc_forward.restype = C.c_int
        L.orc_forward.argtypes = [P, C.c_int, C.c_int, F]
        L.orc_get_x.argtypes = [P, F]
        L.orc_get_kv.argtypes = [P, C.c_int, F, F, C.c_int]
        L.orc_set_kv.argtypes = [P, C.c_int, F, F, C.c_int]
        L.orc_set_order.restype = None
        L.orc_set_order.argtypes = [P, C.c_int]
        L.orc_sample_top_p.restype = C.c_int
        L.orc_sample_top_p.argtypes = [F, C.c_int, C.c_float, C.c_float, C.c_float, C.POINTER(C.c_int)]

    def fp16(self, h: int) -> float:
        return self.lib.orc_fp16_to_fp32(h)

    def sample_top_p(self, logits, temperature: float, top_p: float, r: float):
        """Canonical top-p draw (token, number of tokens kept)."""
        lg = np.ascontiguousarray(logits, np.float32)
        kept = C.c_int(0)
        tok = self.lib.orc_sample_top_p(_fptr(lg), lg.size, temperature, top_p, r, C.byref(kept))
        return tok, kept.value

    def quantize_q8k(self, x, rounding=0, recip_d=0):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(x.size // 256, Q8K_DTYPE)
        self.lib.orc_quantize_q8k(_fptr(x), x.size, _ptr(y), rounding, recip_d)
        return y

    def blocksums(self, ggml_type, w, xq, rows, cols):
        nb = cols // 256
        isum = np.zeros((rows, nb), np.int32)
        aux = np.zeros((rows, nb), np.int32)
        self.lib.orc_blocksums(ggml_type, _ptr(w), _ptr(xq), rows, cols,
                               isum.ctypes.data_as(I32), aux.ctypes.data_as(I32))
        return isum, aux

    def gemv_q8k(self, ggml_type, w, xq, rows, cols, order=1, fused_min=0):
        y = np.zeros(rows, np.float32)
        if ggml_type == spec.GGML_Q4_K:
            self.lib.orc_gemv_q4k_q8k(_ptr(w), _ptr(xq), _fptr(y), rows, cols, order, fused_min)
        else:
            self.lib.orc_gemv_q6k_q8k(_ptr(w), _ptr(xq), _fptr(y), rows, cols, order)
        return y

    def gemv_q8_0(self, w, x, rows, cols):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(rows, np.float32)
        self.lib.orc_gemv_q8_0(_ptr(w), _fptr(x), _fptr(y), rows, cols)
        return y

    def rmsnorm_q8k(self, x, w, eps=spec.RMS_EPS):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.zeros(x.size // 256, Q8K_DTYPE)
        self.lib.orc_rmsnorm_q8k(_fptr(x), _fptr(w), x.size, eps, _ptr(y))
        return y

    def rmsnorm(self, x, w, eps=spec.RMS_EPS):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.zeros_like(x)
        self.lib.orc_rmsnorm(_fptr(x), _fptr(w), x.size, eps, _fptr(out))
        return out

    def swiglu_q8k(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        y = np.zeros(g.size // 256, Q8K_DTYPE)
        self.lib.orc_swiglu_q8k(_fptr(g), _fptr(u), g.size, _ptr(y))
        return y

    def rope(self, v, pos, n_heads, head_dim=spec.HEAD_DIM, base=spec.ROPE_BASE):
        v = np.array(v, np.float32).copy()
        self.lib.orc_rope(_fptr(v), n_heads, head_dim, pos, base)
        return v

    def embedding(self, w, ggml_type, token, dim=spec.N_EMBD):
        out = np.zeros(dim, np.float32)
        self.lib.orc_embedding(_ptr(w), ggml_type, token, dim, _fptr(out))
        return out


_LAYER_INDEX = {n: i for i, n in enumerate(spec.LAYER_TENSORS)}


class OracleModel:
    """Whole-model forward of the C restatement over a mapped GGUF file."""

    def __init__(self, oracle: Oracle, path: str, max_seq: int, kv_f16: bool = False):
        """kv_f16: the K/V cache holds half-precision rows (the engine's fp16 KV option)."""
        self.o = oracle
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        kv, tensors, _ = gguf.read_header(path)
        d = orc_model_desc()
        d.base = self.mm.ctypes.data
        for t in tensors:
            if t.name == "token_embd.weight":
                d.tok_embd, d.tok_embd_type = t.offset, t.ggml_type
            elif t.name == "output_norm.weight":
                d.out_norm = t.offset
            elif t.name == "output.weight":
                d.output, d.output_type = t.offset, t.ggml_type
            else:
                _, layer, base, _ = t.name.split(".")
                d.layer[int(layer)][_LAYER_INDEX[base]] = t.offset
                d.layer_type[int(layer)][_LAYER_INDEX[base]] = t.ggml_type
        d.n_layer, d.n_embd, d.n_ff = spec.N_LAYER, spec.N_EMBD, spec.N_FF
        d.n_head, d.n_head_kv, d.n_vocab = spec.N_HEAD, spec.N_HEAD_KV, spec.N_VOCAB
        d.rope_base, d.eps = spec.ROPE_BASE, spec.RMS_EPS
        d.kv_f16 = int(kv_f16)
        self.desc = d
        self.tensors = {t.name: t for t in tensors}
        self.h = oracle.lib.orc_create(C.byref(d), max_seq)

    def forward(self, token: int, pos: int, logits: Optional[np.ndarray] = None) -> int:
        return self.o.lib.orc_forward(self.h, token, pos, _fptr(logits) if logits is not None else None)

    def x(self) -> np.ndarray:
        out = np.zeros(spec.N_EMBD, np.float32)
        self.o.lib.orc_get_x(self.h, _fptr(out))
        return out

    def set_order(self, order: int) -> None:
        """GEMV order of later forward calls: Oracle.ORDER_AVX2 (batch-1 decode, the default) or
        Oracle.ORDER_BATCH (the tcgen05 batched GEMM: batched decode and prefill)."""
        self.o.lib.orc_set_order(self.h, order)

    def set_kv(self, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        self.o.lib.orc_set_kv(self.h, layer, _fptr(k), _fptr(v), k.shape[0])

    def tensor(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self.mm[t.offset:t.offset + t.nbytes]

    def close(self):
        if self.h:
            self.o.lib.orc_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
