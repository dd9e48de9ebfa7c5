"""The library's own NCCL communicator (p2p_comm in include/p2p_attn.h), one per rank.

The reference engine has no multi-GPU code; this serves the ATTN dispatch (engine.js:222)
split over the GPUs of one node.  Rank 0 makes the 128-byte unique id and hands it to the other
ranks over any side channel (here: the torch.distributed group already used to launch the
ranks, or any host transport); every NCCL call inside the library is non-blocking with a host
timeout, so a peer that never joins or leaves between steps turns into P2P_ERR_TIMEOUT or
P2P_ERR_NCCL instead of a hang.
"""
from __future__ import annotations

import ctypes as C

from ._lib import P2P_COMM_ID_BYTES, P2PError, check, lib


def unique_id() -> bytes:
    buf = C.create_string_buffer(P2P_COMM_ID_BYTES)
    check(lib.p2p_comm_unique_id(buf))
    return buf.raw


class Comm:
    """p2p_comm over `nranks` processes; `ctx` is this rank's p2p Context."""

    def __init__(self, ctx, nranks: int, rank: int, uid: bytes, timeout_ms: int = 60000):
        if len(uid) != P2P_COMM_ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        h = C.c_void_p()
        st = lib.p2p_comm_create(ctx.h, nranks, rank, uid, timeout_ms, C.byref(h))
        check(st, ctx.h)
        self.h = h
        self.ctx = ctx
        self.nranks = nranks
        self.rank = rank

    @classmethod
    def from_process_group(cls, ctx, world: int, rank: int, group=None,
                           timeout_ms: int = 60000) -> "Comm":
        """Rank 0's unique id reaches the other ranks through a torch.distributed broadcast."""
        import torch.distributed as dist
        box = [unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(box, src=0, group=group)
        return cls(ctx, world, rank, box[0], timeout_ms)

    def _stream(self, stream):
        from .attention import _stream
        return _stream(stream)

    def wait(self, stream=None):
        """Bounded wait for the stream (collectives included), then the context's sync."""
        check(lib.p2p_comm_wait(self.h, self._stream(stream)), self.ctx.h)

    def barrier(self, stream=None):
        """One-element all-reduce on the stream: orders every rank's earlier work before any
        rank's later work."""
        check(lib.p2p_comm_barrier(self.h, self._stream(stream)), self.ctx.h)

    def close(self):
        if self.h:
            st = lib.p2p_comm_destroy(self.h)
            self.h = None
            if st:
                raise P2PError(st, lib.p2p_status_string(st).decode())

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib.p2p_comm_destroy(self.h)
        except Exception:
            pass
