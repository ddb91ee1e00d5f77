"""Data-parallel training across the GPUs of one node (one process per GPU).

The gradient all-reduce itself runs inside the library (NCCL in per-layer
buckets on a side stream of the step, include/toy_b200.h tb2_dp_init). This module is the host side: it uses
torch.distributed (gloo, over the torchrun rendezvous) only to hand rank 0's
NCCL unique id to every rank, and for host barriers / max-over-ranks timing.
"""
from __future__ import annotations

import ctypes as C
import datetime
import os
from typing import Optional

from ._lib import check, lib

UID_BYTES = 128


class RankFailure(RuntimeError):
    """A peer rank is gone or a collective did not complete in time."""


def _pg():
    import torch.distributed as dist
    return dist


class DataParallel:
    def __init__(self, rank: int, world: int, local_rank: int, timeout_s: float = 120.0):
        dist = _pg()
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if not dist.is_initialized():
            dist.init_process_group("gloo", rank=rank, world_size=world,
                                    timeout=datetime.timedelta(seconds=timeout_s))
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.sess = None

    def exchange_uid(self, uid: bytes | None) -> bytes:
        """Broadcast rank 0's id bytes to every rank (gloo)."""
        import torch
        dist = _pg()
        t = torch.zeros(UID_BYTES, dtype=torch.uint8)
        if self.rank == 0:
            t[:len(uid)] = torch.frombuffer(bytearray(uid), dtype=torch.uint8)
        dist.broadcast(t, src=0)
        return bytes(t.numpy().tobytes())

    def attach(self, eng, bucket_floats: Optional[int] = None, timeout_ms: Optional[int] = None) -> None:
        """Join the engine's session to the NCCL communicator of all ranks;
        gradients are reduced in buckets of at least bucket_floats floats.
        timeout_ms bounds every host wait on a peer (communicator creation,
        each step's collectives): past it the communicator is aborted and the
        step returns an error instead of hanging."""
        L = lib()
        uid = None
        if self.rank == 0:
            buf = (C.c_ubyte * UID_BYTES)()
            n = L.tb2_nccl_unique_id(C.cast(buf, C.c_void_p), UID_BYTES)
            if n <= 0:
                raise RuntimeError(f"tb2_nccl_unique_id failed: {n}")
            uid = bytes(buf)
        uid = self.exchange_uid(uid)
        ubuf = (C.c_ubyte * UID_BYTES).from_buffer_copy(uid)
        check(L.tb2_dp_init(eng.sess, C.cast(ubuf, C.c_void_p), self.rank, self.world), "tb2_dp_init")
        if bucket_floats is not None:
            check(L.tb2_dp_set_bucket_floats(eng.sess, int(bucket_floats)), "tb2_dp_set_bucket_floats")
        if timeout_ms is not None:   # after creation, which keeps the default limit
            check(L.tb2_dp_set_timeout_ms(int(timeout_ms)), "tb2_dp_set_timeout_ms")
        self.sess = eng.sess

    def check_peers(self) -> None:
        """Host-side liveness check before a step: a tiny gloo all-reduce every
        rank makes. A rank that left (or stopped answering) turns it into a
        RankFailure here, before this rank launches a collective that would
        wait for the missing peer on the GPU."""
        import torch
        dist = _pg()
        try:
            dist.all_reduce(torch.ones(1), op=dist.ReduceOp.SUM)
        except Exception as e:  # gloo: connection closed or timed out
            raise RankFailure(f"rank {self.rank}: a peer rank is gone ({type(e).__name__}: {e})") from e

    def status(self) -> int:
        """0 while the NCCL communicator is healthy, else the code that ended it."""
        return lib().tb2_dp_status(self.sess) if self.sess else 0

    def abort(self) -> None:
        """Abort the NCCL communicator from the host (collectives in flight end)."""
        if self.sess:
            lib().tb2_dp_abort(self.sess)

    def bucket_plan(self):
        """The attached session's gradient buckets as [(lo, hi), ...] in issue order."""
        L = lib()
        n = L.tb2_dp_session_bucket_plan(self.sess, None, 0)
        if n < 0:
            raise RuntimeError(f"tb2_dp_session_bucket_plan failed: {n}")
        out = (C.c_longlong * (2 * n + 2))()
        L.tb2_dp_session_bucket_plan(self.sess, out, 2 * n + 2)
        return [(out[2 * i], out[2 * i + 1]) for i in range(n)]

    def detach(self) -> None:
        """Free the attached session's communicator; the process group stays up
        for another attach."""
        if self.sess:
            check(lib().tb2_dp_free(self.sess), "tb2_dp_free")
            self.sess = None

    def barrier(self) -> None:
        _pg().barrier()

    def max_scalar(self, x: float) -> float:
        import torch
        dist = _pg()
        t = torch.tensor([float(x)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def mean_scalar(self, x: float) -> float:
        import torch
        dist = _pg()
        t = torch.tensor([float(x)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item()) / self.world

    def close(self, barrier: bool = True) -> None:
        """Free the communicator and leave the process group (after a barrier
        unless barrier=False). Releasing a healthy communicator is collective
        across the node's ranks (NCCL finalize and destroy); a rank that leaves
        alone calls abort() first."""
        if self.sess:
            lib().tb2_dp_free(self.sess)
            self.sess = None
        dist = _pg()
        if dist.is_initialized():
            if barrier:
                dist.barrier()
            dist.destroy_process_group()
