"""Grouped GEMM on host-resident operands, with the PCIe transfers pipelined.

``hopper_gmm_fwd_host(a, b, batch_sizes, trans_b)`` takes A, B (and returns D)
in pinned host memory.  The experts are cut into contiguous chunks; for each
chunk the H2D copy of its A rows and B slices (copy stream 1), its grouped GEMM
(compute stream) and the D2H copy of its output rows (copy stream 2) are
chained with events, so while chunk i is being multiplied chunk i+1 is
uploading and chunk i-1 is downloading.  PCIe is full duplex, so a step costs
about max(H2D bytes, D2H bytes) / PCIe bandwidth instead of their sum plus
the GEMM.  Device buffers are double-buffered and reused across calls.  Each
chunk carries at least ``min_chunk_bytes`` of operands and output: a chunk
costs a few microseconds of copy and launch latency (and tens of host
microseconds), so a small problem moves in one piece.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch


def _chunks(bs: List[int], n_chunks: int) -> List[Tuple[int, int]]:
    """Split experts [0, E) into at most n_chunks contiguous ranges of similar bytes."""
    E = len(bs)
    n_chunks = max(1, min(n_chunks, E))
    bounds = [round(i * E / n_chunks) for i in range(n_chunks + 1)]
    return [(bounds[i], bounds[i + 1]) for i in range(n_chunks) if bounds[i + 1] > bounds[i]]


def chunk_count(total_bytes: int, n_chunks: int, min_chunk_bytes: int) -> int:
    """Chunks for a problem of ``total_bytes`` (operands + output): at most
    ``n_chunks``, each carrying at least ``min_chunk_bytes``, at least one."""
    return max(1, min(n_chunks, total_bytes // max(1, min_chunk_bytes)))


class HostStreamedGmm:
    """Reusable pipeline state (streams, events, device buffers) for one device."""

    def __init__(self, device=None, n_chunks: int = 8, min_chunk_bytes: int = 32 << 20):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.n_chunks = n_chunks
        self.min_chunk_bytes = min_chunk_bytes
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._bufs = {}

    def _buf(self, key, numel, dtype):
        t = self._bufs.get(key)
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(max(numel, 1), dtype=dtype, device=self.device)
            self._bufs[key] = t
        return t[:numel]

    def __call__(self, a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor,
                 trans_b: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if a.is_cuda or b.is_cuda:
            raise ValueError("hopper_gmm_fwd_host takes host tensors; use hopper_gmm_fwd for device ones")
        bs = [int(v) for v in batch_sizes.tolist()]
        T, dim = a.shape
        E = b.shape[0]
        dim_out = b.shape[1] if trans_b else b.shape[2]
        if sum(bs) != T:
            raise RuntimeError(f"Sum of batch_sizes ({sum(bs)}) must equal A.size(0) ({T})")
        if out is None:
            out = torch.empty(T, dim_out, dtype=a.dtype, pin_memory=True)
        offs = [0]
        for m in bs:
            offs.append(offs[-1] + m)
        compute = torch.cuda.current_stream(self.device)
        total_bytes = (a.numel() + b.numel() + T * dim_out) * a.element_size()
        chunks = _chunks(bs, chunk_count(total_bytes, self.n_chunks, self.min_chunk_bytes))
        per_b = b[0].numel()
        max_rows = max(offs[e1] - offs[e0] for e0, e1 in chunks)
        max_e = max(e1 - e0 for e0, e1 in chunks)
        a_buf = [self._buf(("a", i), max_rows * dim, a.dtype) for i in range(2)]
        b_buf = [self._buf(("b", i), max_e * per_b, b.dtype) for i in range(2)]
        d_buf = [self._buf(("d", i), max_rows * dim_out, a.dtype) for i in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]    # GEMM done with a_buf/b_buf[i]
        drained = [torch.cuda.Event() for _ in range(2)]  # D2H done with d_buf[i]
        for ev in freed + drained:
            ev.record(compute)
        for i, (e0, e1) in enumerate(chunks):
            k = i & 1
            r0, r1 = offs[e0], offs[e1]
            rows, ne = r1 - r0, e1 - e0
            loaded = torch.cuda.Event()
            with torch.cuda.stream(self.h2d):
                self.h2d.wait_event(freed[k])
                a_d = a_buf[k][:rows * dim].view(rows, dim)
                b_d = b_buf[k][:ne * per_b].view(ne, *b.shape[1:])
                a_d.copy_(a[r0:r1], non_blocking=True)
                b_d.copy_(b[e0:e1], non_blocking=True)
                loaded.record(self.h2d)
            compute.wait_event(loaded)
            compute.wait_event(drained[k])
            d_d = d_buf[k][:rows * dim_out].view(rows, dim_out)
            if rows:
                _gmm_into(a_d, b_d, bs[e0:e1], trans_b, d_d)
            freed[k].record(compute)
            done = torch.cuda.Event()
            done.record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done)
                out[r0:r1].copy_(d_d, non_blocking=True)
                drained[k].record(self.d2h)
        compute.wait_stream(self.d2h)
        return out


def _gmm_into(a_d, b_d, bs, trans_b, d_d):
    """The grouped GEMM of one chunk, written into a reused device buffer (C ABI)."""
    from gmm_b200 import capi
    capi.forward(a_d, b_d, bs, d_d, trans_b=trans_b)


_PIPES = {}


def hopper_gmm_fwd_host(a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor,
                        trans_b: bool = False, out: Optional[torch.Tensor] = None,
                        device=None) -> torch.Tensor:
    """``hopper_gmm_fwd`` for operands in (pinned) host memory; returns D in host memory.

    The work is enqueued on the current CUDA stream of ``device``; synchronise
    that stream before reading the result."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    pipe = _PIPES.get(dev)
    if pipe is None:
        pipe = _PIPES[dev] = HostStreamedGmm(dev)
    return pipe(a, b, batch_sizes, trans_b, out)
