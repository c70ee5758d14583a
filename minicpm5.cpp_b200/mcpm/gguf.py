"""Minimal GGUF v2/v3 reader: key/values and tensor infos (absolute offsets).

Used by tests and the benchmark to locate tensors in a model file; the engine
itself parses the header in C++ (csrc/gguf.cpp).
"""
from __future__ import annotations

import struct
from typing import Dict, List, Tuple

from . import spec

_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class GGUFError(ValueError):
    pass


def _read(f, fmt):
    n = struct.calcsize(fmt)
    b = f.read(n)
    if len(b) != n:
        raise GGUFError("truncated GGUF header")
    return struct.unpack(fmt, b)[0]


def _read_str(f) -> str:
    n = _read(f, "<Q")
    if n > 1 << 30:
        raise GGUFError("string length out of range")
    b = f.read(n)
    if len(b) != n:
        raise GGUFError("truncated GGUF string")
    return b.decode("utf-8", "replace")


def _read_value(f, vtype):
    if vtype in _SCALARS:
        return _read(f, _SCALARS[vtype])
    if vtype == 8:
        return _read_str(f)
    if vtype == 9:
        etype = _read(f, "<I")
        n = _read(f, "<Q")
        if etype in _SCALARS and n > 4096:     # large arrays: skip the bytes
            f.seek(n * struct.calcsize(_SCALARS[etype]), 1)
            return None
        return [_read_value(f, etype) for _ in range(n)]
    raise GGUFError(f"unknown GGUF value type {vtype}")


def read_header(path: str) -> Tuple[Dict[str, object], List[spec.TensorInfo], int]:
    """Returns (kv, tensors with absolute offsets, data_start)."""
    with open(path, "rb") as f:
        if f.read(4) != b"GGUF":
            raise GGUFError("not a GGUF file")
        version = _read(f, "<I")
        if version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {version}")
        n_tensors = _read(f, "<Q")
        n_kv = _read(f, "<Q")
        kv = {}
        for _ in range(n_kv):
            key = _read_str(f)
            kv[key] = _read_value(f, _read(f, "<I"))
        infos = []
        for _ in range(n_tensors):
            name = _read_str(f)
            nd = _read(f, "<I")
            dims = tuple(_read(f, "<Q") for _ in range(nd))
            t = _read(f, "<I")
            off = _read(f, "<Q")
            infos.append((name, t, dims, off))
        align = int(kv.get("general.alignment", spec.GGUF_ALIGNMENT))
        data_start = spec.align(f.tell(), align)
    tensors = [spec.TensorInfo(n, t, d, data_start + off) for n, t, d, off in infos]
    return kv, tensors, data_start
