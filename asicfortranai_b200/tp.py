"""Tensor-parallel group over libq35's NCCL communicator, bootstrapped with
torch.distributed (one process per GPU; any backend, gloo is enough: only the 128-byte
NCCL id and barriers travel through it)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


def exchange_unique_id(dist) -> bytes:
    """Rank 0 makes the NCCL id; every rank returns the same 128 bytes.  The id travels
    in a host tensor, or a device tensor when the process group's backend is NCCL."""
    import torch
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    buf = torch.zeros(128, dtype=torch.uint8)
    if dist.get_rank() == 0:
        raw = (C.c_uint8 * 128)()
        _lib.check(_lib.load().q35_tp_unique_id(raw, 128), "tp_unique_id")
        buf = torch.from_numpy(np.frombuffer(bytes(raw), dtype=np.uint8).copy())
    buf = buf.to(device)
    dist.broadcast(buf, src=0)
    return bytes(buf.cpu().numpy().tobytes())


class TPGroup:
    _close_last = True   # closed after the models built on it

    def __init__(self, ctx, rank: int, world: int, uid: bytes, timeout_s: float = 120.0):
        L = _lib.load()
        raw = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = C.c_void_p()
        _lib.check(L.q35_tp_create(ctx.h, rank, world, raw, 128, timeout_s, C.byref(h)), "tp_create")
        self.h, self.ctx, self.rank, self.world = h, ctx, rank, world
        ctx.adopt(self)

    @classmethod
    def from_torch(cls, ctx, dist, timeout_s: float = 120.0):
        return cls(ctx, dist.get_rank(), dist.get_world_size(), exchange_unique_id(dist), timeout_s)

    def allreduce_i32(self, ptr: int, count: int):
        _lib.check(_lib.load().q35_tp_allreduce_i32(self.h, self.ctx.h, ptr, count), "tp_allreduce_i32")

    def abort(self):
        """Abandon the communicator after a peer failed (callable from any thread): this
        rank's collectives still waiting for the peer return, later ones fail."""
        if self.h:
            _lib.load().q35_tp_abort(self.h)

    def close(self):
        if self.h:
            _lib.check(_lib.load().q35_tp_destroy(self.h), "tp_destroy")
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
