"""Host-side all-gather of the per-rank expert counts for one node.

Every rank of an expert-parallel group needs every rank's ``batch_sizes``
(host int64 tensors) before it can size its transfers.  A gloo all-gather
over TCP costs ~0.2 ms at 2 ranks and ~2 ms at 8; ranks on one host can
instead meet in a POSIX shared-memory block:

* the block holds two slots per rank (step parity), each ``[seq, counts[E]]``;
* a rank writes its counts into slot ``seq & 1`` and then the sequence number;
* it then spins until every rank's slot ``seq & 1`` carries ``seq`` and reads
  the counts.  A rank can only run one step ahead of the slowest reader (it
  cannot pass step ``seq + 1`` before every rank posted it, which each does
  after reading step ``seq``), so two slots never clobber unread data.

The spin is bounded (``timeout_s``); a rank that never posts makes the others
raise instead of hanging.  x86 keeps stores (and loads) in program order, so
writing counts before the sequence number publishes them safely.
"""

from __future__ import annotations

import os
import socket
import time
import uuid

import numpy as np
import torch
import torch.distributed as dist


class ShmCountExchange:
    """All-gather of a fixed-length int64 vector among the ranks of a one-host group."""

    def __init__(self, length: int, group=None, timeout_s: float = 60.0):
        from multiprocessing import shared_memory
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.length = length
        self.timeout_s = timeout_s
        self.slot = length + 1  # [seq, counts...]
        nbytes = 2 * self.world * self.slot * 8
        name = [f"gmm_ep_{uuid.uuid4().hex[:16]}" if self.rank == 0 else None]
        dist.broadcast_object_list(name, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        if self.rank == 0:
            self._shm = shared_memory.SharedMemory(name=name[0], create=True, size=nbytes)
            np.ndarray((nbytes // 8,), dtype=np.int64, buffer=self._shm.buf)[:] = -1
        dist.barrier(group=group)
        if self.rank != 0:
            self._shm = shared_memory.SharedMemory(name=name[0], create=False)
            try:  # the creator owns the segment's lifetime
                from multiprocessing import resource_tracker
                resource_tracker.unregister(self._shm._name, "shared_memory")
            except Exception:  # noqa: BLE001
                pass
        self._mem = np.ndarray((2, self.world, self.slot), dtype=np.int64, buffer=self._shm.buf)
        self._seq = 0
        dist.barrier(group=group)

    def __call__(self, counts: torch.Tensor) -> torch.Tensor:
        v = counts.numpy() if counts.dtype == torch.int64 else counts.to(torch.int64).numpy()
        if v.shape != (self.length,):
            raise ValueError(f"expected {self.length} counts, got {tuple(v.shape)}")
        self._seq += 1
        seq, par = self._seq, self._seq & 1
        mine = self._mem[par, self.rank]
        mine[1:] = v
        mine[0] = seq  # published after the counts
        t_end = time.monotonic() + self.timeout_s
        seqs = self._mem[par, :, 0]
        while not (seqs == seq).all():
            if time.monotonic() > t_end:
                missing = [int(r) for r in np.nonzero(seqs != seq)[0]]
                raise RuntimeError(f"count exchange step {seq}: ranks {missing} did not post "
                                   f"within {self.timeout_s:.0f} s")
            time.sleep(0)
        return torch.from_numpy(self._mem[par, :, 1:].copy())

    def close(self):
        if getattr(self, "_shm", None) is not None:
            self._shm.close()
            if self.rank == 0:
                try:
                    self._shm.unlink()
                except FileNotFoundError:
                    pass
            self._shm = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


def same_host(group=None) -> bool:
    """True if every rank of ``group`` runs on this host (collective)."""
    names = [None] * dist.get_world_size(group)
    dist.all_gather_object(names, socket.gethostname() + ":" + str(os.getuid()), group=group)
    return len(set(names)) == 1
