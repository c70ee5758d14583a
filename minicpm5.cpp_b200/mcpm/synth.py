"""Seeded synthetic MiniCPM5-2B GGUF files (random-init weights, real layout).

There is no network and no checkpoint, so every benchmark and parity run uses
a random-init model with the released file's layout.  Value distributions
follow the benchmark definition of the workloads:

* Q4_K super-block (144 B, reference ``include/ops.h:43-48``): fp16 ``d`` and
  ``dmin`` = |N(0, 2e-3)|; the 12 packed scale bytes and the 128 nibble bytes
  uniform, which makes every 6-bit scale/min uniform on 0..63 and every nibble
  uniform on 0..15.
* Q6_K super-block (210 B, ``include/ops.h:51-56``): ``ql``/``qh`` uniform
  bytes, int8 ``scales`` uniform on -32..31, fp16 ``d`` = |N(0, 2e-3)|.
* Q8_0 block (34 B, ``include/ops.h:35-38``): fp16 ``d`` = |N(0, 2e-3)|, int8
  quants uniform on -127..127.
* F32 norm weights: 1 + N(0, 0.02).

The file is a valid GGUF v3 file: a key/value section, tensor infos, and for
the Q4_K_M variant a padding string sized so that the data section starts at
the released file's offset 5,145,568; the reference engine (which maps tensors
by hard-coded absolute offsets, ``src/model.cpp:78-133``) therefore loads the
same file as this project's header-parsing loader.

Each tensor is drawn from its own ``numpy.random.PCG64`` stream seeded by
``(seed, tensor index)``, so files are bit-reproducible.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from typing import List, Optional

import numpy as np

from . import spec

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
# GGUF metadata value types
_U32, _F32, _STR, _U64 = 4, 6, 8, 10

DEFAULT_DIR = os.environ.get("MCPM_MODEL_DIR", "/tmp/mcpm_models")


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _gguf_str(key) + struct.pack("<I", vtype)
    if vtype == _U32:
        out += struct.pack("<I", value)
    elif vtype == _F32:
        out += struct.pack("<f", value)
    elif vtype == _U64:
        out += struct.pack("<Q", value)
    elif vtype == _STR:
        out += _gguf_str(value)
    else:
        raise ValueError(vtype)
    return out


def _fp16_absnormal(rng: np.random.Generator, n: int, sigma: float = 2e-3) -> np.ndarray:
    return np.abs(rng.normal(0.0, sigma, n)).astype(np.float16).view(np.uint16)


def tensor_bytes(t: spec.TensorInfo, rng: np.random.Generator, sigma: float = 2e-3, balanced: bool = False) -> np.ndarray:
    """Random contents of one tensor as a flat uint8 array (fp16 block scales |N(0, sigma)|).

    ``balanced``: a Q4_K block's ``dmin`` is 7.5 * ``d`` instead of an independent draw, so
    the expected value of every dequantised weight, d*sc*q - dmin*m with sc, m uniform on
    0..63 and q on 0..15, is zero."""
    if t.ggml_type == spec.GGML_F32:
        return (1.0 + rng.normal(0.0, 0.02, t.n_elements)).astype(np.float32).view(np.uint8)
    per, nb = spec.BLOCK_GEOM[t.ggml_type]
    nblk = t.n_elements // per
    raw = np.frombuffer(rng.bytes(nblk * nb), dtype=np.uint8).reshape(nblk, nb).copy()
    if t.ggml_type == spec.GGML_Q4_K:
        d = _fp16_absnormal(rng, nblk, sigma)
        dmin = _fp16_absnormal(rng, nblk, sigma)
        if balanced:
            dmin = (d.view(np.float16).astype(np.float32) * 7.5).astype(np.float16).view(np.uint16)
        raw[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
        raw[:, 2:4] = dmin.view(np.uint8).reshape(nblk, 2)
    elif t.ggml_type == spec.GGML_Q6_K:
        raw[:, 192:208] = rng.integers(-32, 32, (nblk, 16), dtype=np.int8).view(np.uint8)
        raw[:, 208:210] = _fp16_absnormal(rng, nblk, sigma).view(np.uint8).reshape(nblk, 2)
    elif t.ggml_type == spec.GGML_Q8_0:
        raw[:, 0:2] = _fp16_absnormal(rng, nblk, sigma).view(np.uint8).reshape(nblk, 2)
        raw[:, 2:34] = rng.integers(-127, 128, (nblk, 32), dtype=np.int8).view(np.uint8)
    else:
        raise ValueError(t.ggml_type)
    return raw.reshape(-1)


def _header(tensors: List[spec.TensorInfo], data_start: Optional[int], variant: str) -> bytes:
    kvs = [
        _kv("general.architecture", _STR, "minicpm5"),
        _kv("general.name", _STR, f"MiniCPM5-2B synthetic {variant}"),
        _kv("general.alignment", _U32, spec.GGUF_ALIGNMENT),
        _kv("minicpm5.block_count", _U32, spec.N_LAYER),
        _kv("minicpm5.embedding_length", _U32, spec.N_EMBD),
        _kv("minicpm5.feed_forward_length", _U32, spec.N_FF),
        _kv("minicpm5.attention.head_count", _U32, spec.N_HEAD),
        _kv("minicpm5.attention.head_count_kv", _U32, spec.N_HEAD_KV),
        _kv("minicpm5.rope.freq_base", _F32, spec.ROPE_BASE),
        _kv("minicpm5.attention.layer_norm_rms_epsilon", _F32, spec.RMS_EPS),
        _kv("minicpm5.vocab_size", _U32, spec.N_VOCAB),
    ]
    infos = b""
    for t in tensors:
        infos += _gguf_str(t.name) + struct.pack("<I", len(t.dims))
        infos += b"".join(struct.pack("<Q", d) for d in t.dims)
        infos += struct.pack("<IQ", t.ggml_type, t.offset - tensors[0].offset)

    def assemble(pad_kv: bytes) -> bytes:
        n_kv = len(kvs) + (1 if pad_kv else 0)
        return (GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(tensors), n_kv)
                + b"".join(kvs) + pad_kv + infos)

    hdr = assemble(b"")
    if data_start is None:
        return hdr
    # A padding string KV moves the end of the header to just below data_start.
    empty_pad = _kv("general.padding", _STR, "")
    room = data_start - len(hdr) - len(empty_pad)
    if room < 0:
        raise ValueError("header does not fit before the data section")
    hdr = assemble(_kv("general.padding", _STR, "#" * room))
    assert spec.align(len(hdr)) == data_start
    return hdr


def write_model(path: str, variant: str = "q4_k_m", seed: int = 0, dscale: float = 1.0) -> dict:
    """Write a synthetic model; returns its manifest (also stored as path + '.json').

    ``dscale`` = 1.0: the benchmark distribution.  Its Q4_K weights have a positive mean
    (nibbles 0..15 against small mins), so every layer amplifies the all-ones direction of
    the residual stream, SwiGLU's exp overflows in many blocks, and the greedy stream
    hardly depends on the prompt.  ``dscale`` != 1.0: a parity model with the same layout
    and types whose Q4_K blocks are balanced (zero-mean weights, see ``tensor_bytes``) and
    whose per-layer block scales (``blk.*``) are multiplied by ``dscale``, so activations
    stay near unit size and the logits depend on the input."""
    base = spec.tensor_list(variant)
    if variant == "q4_k_m":
        data_start = spec.Q4KM_DATA_START
    else:
        data_start = spec.align(len(_header(spec.layout(base, 0), None, variant)) + 64)
    tensors = spec.layout(base, data_start)
    hdr = _header(tensors, data_start, variant)
    tmp = path + ".tmp"
    digest = hashlib.sha256()
    with open(tmp, "wb") as f:
        f.write(hdr)
        f.write(b"\0" * (data_start - len(hdr)))
        pos = data_start
        for i, t in enumerate(tensors):
            assert pos <= t.offset
            if pos < t.offset:
                f.write(b"\0" * (t.offset - pos))
                pos = t.offset
            rng = np.random.Generator(np.random.PCG64([seed, i]))
            b = tensor_bytes(t, rng, 2e-3 * (dscale if t.name.startswith("blk.") else 1.0), balanced=dscale != 1.0)
            assert b.size == t.nbytes
            digest.update(b[:4096].tobytes())
            f.write(b.tobytes())
            pos += b.size
    os.replace(tmp, path)
    manifest = {"variant": variant, "seed": seed, "dscale": dscale, "size": os.path.getsize(path),
                "data_start": data_start, "table": spec.table_digest(tensors),
                "content_digest": digest.hexdigest()}
    with open(path + ".json", "w") as f:
        json.dump(manifest, f)
    return manifest


def model_path(variant: str = "q4_k_m", seed: int = 0, directory: Optional[str] = None, dscale: float = 1.0) -> str:
    directory = directory or DEFAULT_DIR
    tag = "" if dscale == 1.0 else f"-d{dscale:g}"
    return os.path.join(directory, f"minicpm5-2b-synth-{variant}-s{seed}{tag}.gguf")


def ensure_model(variant: str = "q4_k_m", seed: int = 0, directory: Optional[str] = None, dscale: float = 1.0) -> str:
    """Path of the synthetic model, writing it first if it is absent or stale."""
    path = model_path(variant, seed, directory, dscale)
    meta = path + ".json"
    if os.path.exists(path) and os.path.exists(meta):
        try:
            with open(meta) as f:
                m = json.load(f)
            if m.get("size") == os.path.getsize(path) and m.get("seed") == seed and m.get("dscale", 1.0) == dscale:
                return path
        except (OSError, ValueError):
            pass
    os.makedirs(os.path.dirname(path), exist_ok=True)
    write_model(path, variant, seed, dscale)
    return path


def prompt_ids(n: int, seed: int = 1234, vocab: int = spec.N_VOCAB) -> np.ndarray:
    """Seeded prompt of ``n`` token ids uniform on [0, vocab)."""
    return np.random.Generator(np.random.PCG64([seed, 7])).integers(0, vocab, n).astype(np.int32)
