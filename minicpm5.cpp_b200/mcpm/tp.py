"""Tensor-parallel batch-1 decode of an all-Q8_0 model (C ABI `mcpm_tp_*` of include/mcpm.h).

One `TPEngine` per GPU and process.  Setup exchanges either rank 0's NCCL id (comm="nccl") or
every rank's CUDA-IPC receive-buffer handle (comm="p2p") through any host channel; `connect`
does it with `torch.distributed` collectives on an existing process group.  Every rank then
calls `forward` / `generate` with the same arguments and gets the same greedy tokens; each
rank's logits are its vocabulary slice [vocab_lo, vocab_hi).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from .engine import MCPMError, check, load_library  # noqa: F401  (MCPMError re-exported)

P2P, NCCL = 0, 1


class mcpm_tp_config(C.Structure):
    _fields_ = [("device", C.c_int), ("rank", C.c_int), ("world", C.c_int), ("max_seq", C.c_int),
                ("comm", C.c_int), ("eager", C.c_int), ("peer_wait_us", C.c_int), ("reserved", C.c_int * 1)]


def nccl_id() -> bytes:
    """Rank 0's NCCL unique id (128 bytes)."""
    buf = C.create_string_buffer(128)
    check(load_library().mcpm_tp_nccl_id(buf), "mcpm_tp_nccl_id")
    return buf.raw


class TPEngine:
    def __init__(self, device: int, rank: int, world: int, max_seq: int, comm: str = "p2p", eager: bool = False,
                 peer_wait_us: int = 0):
        """peer_wait_us: bound of every device-side wait for another rank (0 = 5 s)."""
        self.lib = load_library()
        self.rank, self.world, self.comm = rank, world, comm
        cfg = mcpm_tp_config(device, rank, world, max_seq, P2P if comm == "p2p" else NCCL, int(eager), int(peer_wait_us))
        h = C.c_void_p()
        check(self.lib.mcpm_tp_create(C.byref(cfg), C.byref(h)), "mcpm_tp_create")
        self.h = h

    def load(self, path: str) -> None:
        check(self.lib.mcpm_tp_load_gguf(self.h, path.encode()), "mcpm_tp_load_gguf")
        info = (C.c_int * 8)()
        check(self.lib.mcpm_tp_info(self.h, info), "mcpm_tp_info")
        self.n_layer, self.n_vocab, self.vocab_lo, self.vocab_hi = info[0], info[1], info[2], info[3]
        self.head0, self.n_heads, self.ffn0, self.n_ffn = info[4], info[5], info[6], info[7]
        self._logits = np.zeros(self.vocab_hi - self.vocab_lo, np.float32)

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        check(self.lib.mcpm_tp_ipc_handle(self.h, buf), "mcpm_tp_ipc_handle")
        return buf.raw

    def connect_with(self, nccl_id128: Optional[bytes] = None, handles: Optional[Sequence[bytes]] = None) -> None:
        hb = None if handles is None else C.create_string_buffer(b"".join(handles), 64 * len(handles))
        ib = None if nccl_id128 is None else C.create_string_buffer(nccl_id128, 128)
        check(self.lib.mcpm_tp_connect(self.h, ib, hb), "mcpm_tp_connect")

    def connect(self, dist=None) -> None:
        """Exchanges the setup data over torch.distributed (any backend) and connects."""
        if self.world == 1:
            self.connect_with()
            return
        assert dist is not None
        if self.comm == "nccl":
            obj = [nccl_id() if self.rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            self.connect_with(nccl_id128=obj[0])
        else:
            hs = [None] * self.world
            dist.all_gather_object(hs, self.ipc_handle())
            self.connect_with(handles=hs)

    def forward(self, token: int, pos: int, logits: bool = True):
        """(greedy token, this rank's logits slice or None)."""
        tok = C.c_int(-1)
        lg = self._logits.ctypes.data_as(C.POINTER(C.c_float)) if logits else None
        check(self.lib.mcpm_tp_forward(self.h, token, pos, lg, C.byref(tok)), "mcpm_tp_forward")
        return tok.value, (self._logits.copy() if logits else None)

    def generate_async(self, n: int) -> None:
        check(self.lib.mcpm_tp_generate_async(self.h, n), "mcpm_tp_generate_async")

    def sync(self) -> None:
        check(self.lib.mcpm_tp_sync(self.h), "mcpm_tp_sync")

    def read_tokens(self, pos0: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.int32)
        check(self.lib.mcpm_tp_read_tokens(self.h, pos0, n, out.ctypes.data_as(C.POINTER(C.c_int))),
              "mcpm_tp_read_tokens")
        return out

    def reset(self) -> None:
        check(self.lib.mcpm_tp_reset(self.h), "mcpm_tp_reset")

    def profile(self, n: int):
        """(ms per step, ms of exchange per step) over n eagerly launched greedy steps."""
        t, c = C.c_float(), C.c_float()
        check(self.lib.mcpm_tp_profile(self.h, n, C.byref(t), C.byref(c)), "mcpm_tp_profile")
        return t.value, c.value

    @property
    def stream(self) -> int:
        return self.lib.mcpm_tp_stream(self.h) or 0

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.mcpm_tp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
