"""MiniCPM5-2B architecture constants and the GGUF tensor table.

The reference engine indexes its weights by a generated table of absolute file
offsets (reference ``include/minicpm_metadata.h:10-17`` for the constants,
``:19-411`` for the 381 tensor rows).  This module rebuilds that table from
first principles instead of copying it:

* the architecture constants (``MODEL_DIM`` ... ``GGUF_ALIGNMENT``),
* the GGUF tensor order of the released file (``output``, ``output_norm``,
  ``token_embd``, then each block's tensors in name order, blocks in numeric
  order),
* the Q4_K_M type rule of llama.cpp's quantiser: ``attn_v`` and ``ffn_down``
  use Q6_K in the first ``n/8`` blocks, the last ``n/8`` blocks and every third
  block in between; ``output`` is Q6_K, all other matrices are Q4_K, norms F32,
* the data-section start of the released file (5,145,568), which is where its
  5 MB header (vocabulary included) ends,
* 32-byte alignment between tensors.

``tests/test_spec.py`` checks the rebuilt table against a digest of the
reference header (``tests/golden/metadata_digest.json``).
"""
from __future__ import annotations

import dataclasses
import hashlib
from typing import Dict, List, Tuple

# Architecture (reference include/minicpm_metadata.h:10-17).
N_EMBD = 2048
N_FF = 6144
N_LAYER = 42
N_HEAD = 16
N_HEAD_KV = 2
HEAD_DIM = N_EMBD // N_HEAD          # 128, derived in reference src/model.cpp:186
KV_DIM = N_HEAD_KV * HEAD_DIM        # 256
N_VOCAB = 130560
ROPE_BASE = 5_000_000.0
RMS_EPS = 1e-6                       # default argument, reference include/ops.h:114,117
GGUF_ALIGNMENT = 32
Q4KM_DATA_START = 5_145_568          # first tensor byte of the released Q4_K_M file

# ggml type ids (GGUF tensor-info type field) and block geometry.
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 8, 12, 14
TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q8_0: "Q8_0",
              GGML_Q4_K: "Q4_K", GGML_Q6_K: "Q6_K"}
NAME_TYPES = {v: k for k, v in TYPE_NAMES.items()}
# (elements per block, bytes per block); reference include/ops.h:33-65
BLOCK_GEOM = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q8_0: (32, 34),
              GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}

LAYER_TENSORS = ("attn_k", "attn_norm", "attn_output", "attn_q", "attn_v",
                 "ffn_down", "ffn_gate", "ffn_norm", "ffn_up")


@dataclasses.dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    dims: Tuple[int, ...]        # GGUF order: dims[0] = columns (input), dims[1] = rows
    offset: int = 0              # absolute file offset (filled in by layout())

    @property
    def type_str(self) -> str:
        return TYPE_NAMES[self.ggml_type]

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        per, nbytes = BLOCK_GEOM[self.ggml_type]
        assert self.n_elements % per == 0, self.name
        return self.n_elements // per * nbytes


def q4km_uses_q6k(layer: int, n_layer: int = N_LAYER) -> bool:
    """llama.cpp Q4_K_M ``use_more_bits`` rule for attn_v / ffn_down."""
    eighth = n_layer // 8
    return layer < eighth or layer >= 7 * n_layer // 8 or (layer - eighth) % 3 == 2


def _dims(base: str) -> Tuple[int, ...]:
    return {
        "attn_q": (N_EMBD, N_EMBD), "attn_k": (N_EMBD, KV_DIM), "attn_v": (N_EMBD, KV_DIM),
        "attn_output": (N_EMBD, N_EMBD), "ffn_gate": (N_EMBD, N_FF), "ffn_up": (N_EMBD, N_FF),
        "ffn_down": (N_FF, N_EMBD), "attn_norm": (N_EMBD,), "ffn_norm": (N_EMBD,),
    }[base]


def tensor_list(variant: str = "q4_k_m") -> List[TensorInfo]:
    """Tensors in file order, offsets not yet assigned.

    ``variant``: ``"q4_k_m"`` (the released mix) or
    ``"q8_0"`` (every matrix Q8_0).
    """
    if variant not in ("q4_k_m", "q8_0"):
        raise ValueError(variant)
    q8 = variant == "q8_0"
    out = [
        TensorInfo("output.weight", GGML_Q8_0 if q8 else GGML_Q6_K, (N_EMBD, N_VOCAB)),
        TensorInfo("output_norm.weight", GGML_F32, (N_EMBD,)),
        TensorInfo("token_embd.weight", GGML_Q8_0 if q8 else GGML_Q4_K, (N_EMBD, N_VOCAB)),
    ]
    for layer in range(N_LAYER):
        for base in LAYER_TENSORS:
            if base.endswith("norm"):
                t = GGML_F32
            elif q8:
                t = GGML_Q8_0
            elif base in ("attn_v", "ffn_down") and q4km_uses_q6k(layer):
                t = GGML_Q6_K
            else:
                t = GGML_Q4_K
            out.append(TensorInfo(f"blk.{layer}.{base}.weight", t, _dims(base)))
    return out


def align(n: int, a: int = GGUF_ALIGNMENT) -> int:
    return (n + a - 1) // a * a


def layout(tensors: List[TensorInfo], data_start: int) -> List[TensorInfo]:
    """Assign absolute offsets: consecutive, each aligned to GGUF_ALIGNMENT."""
    assert data_start % GGUF_ALIGNMENT == 0
    off = data_start
    res = []
    for t in tensors:
        res.append(dataclasses.replace(t, offset=off))
        off = align(off + t.nbytes)
    return res


def q4km_table() -> List[TensorInfo]:
    return layout(tensor_list("q4_k_m"), Q4KM_DATA_START)


def table_digest(tensors: List[TensorInfo]) -> str:
    """sha256 over 'name,offset,size,dims,type' lines (same fields as the reference header rows)."""
    h = hashlib.sha256()
    for t in tensors:
        dims = list(t.dims) + [0] * (4 - len(t.dims))
        h.update(f"{t.name},{t.offset},{t.nbytes},{len(t.dims)},{dims[0]},{dims[1]},{dims[2]},{dims[3]},{t.type_str}\n".encode())
    return h.hexdigest()


def weight_bytes_per_token(tensors: List[TensorInfo]) -> Dict[str, int]:
    """Algorithmic weight bytes one decode step reads: every tensor except the
    embedding matrix, plus one embedding row."""
    total = 0
    emb_row = 0
    for t in tensors:
        if t.name == "token_embd.weight":
            emb_row = t.nbytes // t.dims[1]
        else:
            total += t.nbytes
    return {"weights": total, "embedding_row": emb_row, "total": total + emb_row}


KV_BYTES_PER_POSITION = N_LAYER * 2 * KV_DIM * 4   # 86,016 B of fp32 K+V per position
