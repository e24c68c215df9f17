"""Expert parallelism around the grouped-GEMM forward.

The reference runs the grouped GEMM on one GPU only (it has no distributed
code); this layer shards the E experts of one MoE projection across the
ranks of a process group -- one process per GPU, NCCL over NVLink -- and
moves token rows with one exchange step each way:

1. counts: every rank's host ``batch_sizes`` (rows per global expert) are
   all-gathered over a CPU (gloo) group, so every split size is known on the
   host without a device synchronisation;
2. dispatch: rank r's rows for expert g go to g's owner as NCCL
   point-to-point messages that land directly in the owner's expert-major
   receive buffer (all sources of local expert 0, then of local expert 1, ...);
3. local grouped GEMM over the E/W local experts;
4. combine: each (expert, source) block of the result goes back to its
   source, into the rows the source's A occupied.

Pipelining: the owner's expert-major rows are cut into ``chunks`` pieces
(whole (expert, source-group) blocks, balanced by rows).  All dispatch
messages are posted first, chunk by chunk; chunk c's GEMM waits only for
chunk c's rows, and chunk c's combine runs on NCCL's stream while chunk
c+1's GEMM runs on the compute stream.  Every rank derives every owner's
chunking from the gathered counts, so both ends of each message agree on
which batch carries it.

Two transports carry steps 2 and 4:

* ``"direct"`` (default on GPUs, up to 8 ranks): every rank's token rows and
  output rows live in symmetric memory (``torch.distributed._symmetric_memory``),
  so each rank can address its peers' buffers over NVLink.  Dispatch is one
  gather kernel pulling each (expert, source) chunk into the expert-major
  receive buffer with peer loads; the combine is fused into the grouped-GEMM
  epilogue, which stores each result row straight into the output buffer of
  the rank it came from, tile by tile, while the next tiles are computed.
  Two cross-rank barriers order the step: inputs written everywhere before
  the gather, all peer stores landed before the output is read.  By default
  they are one small kernel each over symmetric-memory flags
  (``gmm_sm100_ep_barrier``: release/acquire at system scope, bounded wait);
  ``barrier="nccl"`` uses 1-element NCCL all-reduces instead.  The result is
  copied out of the symmetric output buffer into ``out`` (a new tensor by
  default); passing ``out=layer.output_buffer(...)`` skips that copy, and the
  result is then overwritten by the next call.
* ``"nccl"``: NCCL point-to-point messages (below); also what the CPU tests
  run on gloo ranks.

Rank r owns experts ``[r*E/W, (r+1)*E/W)``; any other placement is a
relabelling of the experts (label l = the expert placed in slot l, the rows
grouped by label), e.g. ``balanced_placement`` of measured loads.  Output rows are bit-identical
to the single-GPU operator on the same rows.  There is no CPU fallback: the
local GEMM is the CUDA kernel (through the C ABI, writing in place into a
reused buffer) unless a test substitutes the CPU oracle to check the
exchange logic on gloo ranks.
"""

from __future__ import annotations

from typing import Callable, List, Optional

import torch
import torch.distributed as dist


def balanced_placement(loads, world: int) -> List[int]:
    """Expert placement for expert parallelism: ``perm[l]`` is the expert that
    takes label ``l``, and rank r owns labels ``[r*E/W, (r+1)*E/W)``.  Experts
    go, heaviest first, to the rank with the fewest rows so far among those with
    a free slot (greedy longest-processing-time), so every rank computes about
    the same number of rows."""
    loads = [int(v) for v in loads]
    E = len(loads)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    rows = [0] * world
    owned: List[List[int]] = [[] for _ in range(world)]
    for e in sorted(range(E), key=lambda i: (-loads[i], i)):
        r = min((r for r in range(world) if len(owned[r]) < per), key=lambda r: (rows[r], r))
        owned[r].append(e)
        rows[r] += loads[e]
    return [e for r in range(world) for e in sorted(owned[r])]


class _Chunking:
    """Every owner's blocks and chunks for one exchange (identical on all ranks)."""

    def __init__(self, all_bs: List[List[int]], world: int, e_local: int, chunks: int):
        self.W, self.El = world, e_local
        n_src_groups = max(1, -(-chunks // e_local))  # ceil(chunks / El)
        n_src_groups = min(n_src_groups, world)
        bounds = [round(j * world / n_src_groups) for j in range(n_src_groups + 1)]
        self.src_groups = [(bounds[j], bounds[j + 1]) for j in range(n_src_groups)]
        self.chunks = chunks
        # per owner p: list of chunks, each a list of blocks (e, s0, s1, rows)
        self.owner_chunks = []
        for p in range(world):
            blocks = []
            for e in range(e_local):
                g = p * e_local + e
                for (s0, s1) in self.src_groups:
                    rows = sum(all_bs[s][g] for s in range(s0, s1))
                    blocks.append((e, s0, s1, rows))
            total = sum(b[3] for b in blocks)
            out = [[] for _ in range(chunks)]
            acc = 0
            for b in blocks:  # contiguous blocks -> chunk by row-count quantile
                c = min(chunks - 1, (acc * chunks) // max(total, 1))
                out[c].append(b)
                acc += b[3]
            self.owner_chunks.append(out)

    def chunk_of(self, p: int, e: int, s: int) -> int:
        for c, blocks in enumerate(self.owner_chunks[p]):
            for (be, s0, s1, _) in blocks:
                if be == e and s0 <= s < s1:
                    return c
        raise KeyError((p, e, s))


class ExpertParallelGmm:
    """Expert-parallel grouped GEMM forward over a process group.

    Args:
        num_experts: global number of experts E (divisible by the world size).
        group: process group carrying the token rows (NCCL for GPUs).
        count_group: CPU (gloo) group for the host-side count exchange; created
            from the world if not given.
        local_gemm: ``f(a, b_local, batch_sizes, trans_b) -> d`` replacing the CUDA
            kernel (tests only: checks the exchange logic on CPU ranks).
        chunks: pipeline depth of the ``"nccl"`` transport (GEMM / combine overlap);
            default 1 (measured fastest with NCCL point-to-point on 2 B200s).
        transport: ``"direct"``, ``"nccl"`` or ``"auto"`` (direct for CUDA tensors on
            up to 8 ranks without a substituted ``local_gemm``).
        count_exchange: ``"shm"`` (shared memory, ranks on one host), ``"gloo"``, or
            ``"auto"`` (shm when every rank is on this host).  Construction is
            collective over the count group.
        barrier: cross-rank barrier of the direct transport: ``"flags"`` (one small
            kernel over symmetric-memory flags) or ``"nccl"`` (1-element all-reduce).
    """

    def __init__(self, num_experts: int, group=None, count_group=None,
                 local_gemm: Optional[Callable] = None, chunks: int = 1, transport: str = "auto",
                 count_exchange: str = "auto", barrier: str = "flags"):
        if transport not in ("auto", "direct", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        if barrier not in ("flags", "nccl"):
            raise ValueError(f"unknown barrier {barrier!r}")
        self.transport = transport
        self.barrier = barrier
        self._epoch = 0
        self._flags = None  # (symmetric int32 flag slots, their per-rank addresses, handle)
        self.record_phases = False  # when set, CUDA events around each phase of a direct step
        self.phase_events = {}
        # direct transport: the own-rows GEMM overlaps the barrier + gather when this
        # rank's own rows average at least overlap_min_rows per local expert
        self.overlap = True
        self.overlap_min_rows = 256
        self._side = None
        self._sym = None  # (capacity rows, dim, dim_out, dtype, device, a_sym, out_sym, a_ptrs, out_ptrs)
        self._flag = None
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world != 0:
            raise ValueError(f"num_experts ({num_experts}) must be divisible by the world size "
                             f"({self.world})")
        self.num_experts = num_experts
        self.e_local = num_experts // self.world
        if count_group is None:
            count_group = group if dist.get_backend(group) == "gloo" else dist.new_group(backend="gloo")
        self.count_group = count_group
        self.local_gemm = local_gemm
        self.chunks = max(1, int(chunks))
        self._peer = [dist.get_global_rank(group, i) if group is not None else i
                      for i in range(self.world)]
        self._x = None
        self._y = None
        self._shm_counts = None
        if count_exchange not in ("auto", "shm", "gloo"):
            raise ValueError(f"unknown count_exchange {count_exchange!r}")
        if count_exchange != "gloo" and self.world > 1:
            from gmm_b200.host_exchange import ShmCountExchange, same_host
            if count_exchange == "shm" or same_host(self.count_group):
                self._shm_counts = ShmCountExchange(num_experts, self.count_group)

    # ------------------------------------------------------------------ plan
    def exchange_counts(self, batch_sizes: torch.Tensor) -> torch.Tensor:
        """All ranks' ``batch_sizes`` as a ``[W, E]`` int64 CPU tensor."""
        if batch_sizes.device.type != "cpu" or batch_sizes.dtype != torch.int64 \
                or batch_sizes.dim() != 1 or batch_sizes.numel() != self.num_experts:
            raise ValueError("batch_sizes must be a 1D CPU int64 tensor with num_experts entries")
        if (batch_sizes < 0).any():
            raise ValueError("batch_sizes must be non-negative")
        if self._shm_counts is not None:
            return self._shm_counts(batch_sizes.contiguous())
        out = [torch.empty_like(batch_sizes) for _ in range(self.world)]
        dist.all_gather(out, batch_sizes.contiguous(), group=self.count_group)
        return torch.stack(out)

    def _buffer(self, name, rows, cols, like):
        buf = getattr(self, name)
        need = rows * cols
        if buf is None or buf.numel() < need or buf.dtype != like.dtype or buf.device != like.device:
            buf = torch.empty(max(need, 1), dtype=like.dtype, device=like.device)
            setattr(self, name, buf)
        return buf[:need].view(rows, cols)

    def _gemm_into(self, x, b, bs_list, trans_b, y):
        if x.shape[0] == 0:
            return
        bs = torch.tensor(bs_list, dtype=torch.int64)
        if self.local_gemm is not None:
            y.copy_(self.local_gemm(x, b, bs, trans_b))
            return
        from gmm_b200 import capi
        capi.forward(x, b, bs_list, y, trans_b=trans_b)

    # ------------------------------------------------------- direct transport
    def _use_direct(self, a: torch.Tensor) -> bool:
        if self.transport == "nccl" or self.local_gemm is not None:
            return False
        ok = a.is_cuda and self.world <= 8
        if self.transport == "direct" and not ok:
            raise ValueError("the direct transport needs CUDA tensors and at most 8 ranks")
        return ok

    def _barrier(self, device):
        if self.barrier == "nccl":
            if self._flag is None or self._flag.device != device:
                self._flag = torch.zeros(1, dtype=torch.float32, device=device)
            dist.all_reduce(self._flag, group=self.group)
            return
        from gmm_b200 import capi
        if self._flags is None or self._flags[0].device != device:
            import torch.distributed._symmetric_memory as symm_mem
            group = self.group if self.group is not None else dist.group.WORLD
            f = symm_mem.empty(8, dtype=torch.int32, device=device)
            f.zero_()
            h = symm_mem.rendezvous(f, group)
            torch.cuda.synchronize(device)
            dist.barrier(group=self.count_group)  # every rank's slots are zero before any post
            self._flags = (f, list(h.buffer_ptrs), h)
            self._epoch = 0
        self._epoch += 1
        capi.ep_barrier(self._flags[1], self.rank, self._epoch, device)

    def _symmetric(self, rows: int, dim: int, dim_out: int, dtype, device):
        """(Re)allocate the symmetric token / output buffers; collective when it allocates.

        Every rank derives ``rows`` from the same gathered counts, so all ranks
        (re)allocate together."""
        import torch.distributed._symmetric_memory as symm_mem
        cur = self._sym
        if cur is not None and cur[0] >= rows and cur[1:5] == (dim, dim_out, dtype, device):
            return cur
        cap = max(rows, 1)
        cap = (cap + 1023) // 1024 * 1024
        group = self.group if self.group is not None else dist.group.WORLD
        a_sym = symm_mem.empty(cap * dim, dtype=dtype, device=device)
        h_a = symm_mem.rendezvous(a_sym, group)
        o_sym = symm_mem.empty(cap * dim_out, dtype=dtype, device=device)
        h_o = symm_mem.rendezvous(o_sym, group)
        self._sym = (cap, dim, dim_out, dtype, device, a_sym, o_sym,
                     list(h_a.buffer_ptrs), list(h_o.buffer_ptrs), h_a, h_o)
        return self._sym

    def input_buffer(self, rows: int, dim: int, dim_out: int, dtype, device) -> torch.Tensor:
        """A ``[rows, dim]`` view of this rank's symmetric token buffer.

        Writing the layer's input rows here (instead of passing any tensor)
        saves the copy into symmetric memory in ``forward``.  Collective: every
        rank must call it with the same capacity."""
        sym = self._symmetric(rows, dim, dim_out, dtype, device)
        return sym[5][:rows * dim].view(rows, dim)

    def output_buffer(self, rows: int, dim: int, dim_out: int, dtype, device) -> torch.Tensor:
        """A ``[rows, dim_out]`` view of this rank's symmetric output buffer.

        Passed as ``out=``, the result is left where the peers' epilogues
        stored it (no copy); it is then valid only until the next call.
        Collective like ``input_buffer``."""
        sym = self._symmetric(rows, dim, dim_out, dtype, device)
        return sym[6][:rows * dim_out].view(rows, dim_out)

    def _mark(self, device, name):
        if self.record_phases:
            e = torch.cuda.Event(enable_timing=True)
            e.record(torch.cuda.current_stream(device))
            self.phase_events[name] = e

    def _forward_direct(self, a, b_local, all_bs, trans_b, out=None):
        from gmm_b200 import capi
        W, El, r = self.world, self.e_local, self.rank
        dim = a.shape[1]
        dim_out = b_local.shape[1] if trans_b else b_local.shape[2]
        rows_max = int(all_bs.sum(1).max())
        sym = self._symmetric(rows_max, dim, dim_out, a.dtype, a.device)
        a_sym = sym[5][:a.shape[0] * dim].view(a.shape[0], dim)
        res = sym[6][:a.shape[0] * dim_out].view(a.shape[0], dim_out)
        if a.data_ptr() != a_sym.data_ptr():
            a_sym.copy_(a)
        # offsets of every global expert's rows in every rank's layout: [W, E]
        offs = torch.cumsum(all_bs, dim=1) - all_bs
        mine = slice(r * El, (r + 1) * El)
        # segment j of every local expert comes from rank (r + j) % W: each rank
        # starts with itself and walks the others in a rotated order, so no two
        # ranks read from or write to the same peer at the same time
        order = [(r + j) % W for j in range(W)]
        counts = all_bs[order][:, mine].t().contiguous().numpy()  # [El, W]
        rows_at = offs[order][:, mine].t().contiguous().numpy()   # where they sit on their rank
        if self.record_phases:
            self.phase_events = {}
        # Overlap only pays when the own-rows GEMM is compute-bound: it reads all
        # local experts' weights a second time, which for a few rows per
        # expert (HBM-bound) costs more than the gather it hides.
        overlap = (self.overlap and W > 1
                   and int(counts[:, 0].sum()) >= self.overlap_min_rows * El)
        if not overlap:
            n_recv = int(counts.sum())
            x = self._buffer("_x", n_recv, dim, a)
            self._mark(a.device, "start")
            self._barrier(a.device)  # every rank's token rows are in place
            self._mark(a.device, "barrier_in")
            if n_recv:
                capi.ep_gather(x, sym[7], counts, rows_at, El, dim * a.element_size(), rank_base=r)
                self._mark(a.device, "gather")
                capi.forward_ep(x, b_local, counts, rows_at, El, sym[8], trans_b=trans_b, rank_base=r)
            self._mark(a.device, "peer_gemm")
            self._barrier(a.device)  # every peer's result rows have landed here
            self._mark(a.device, "barrier_out")
            return self._result(res, out)
        # Overlapped step.  This rank's own rows for its local experts are one
        # contiguous block of its token rows: their GEMM (plain, local output)
        # needs no exchange and runs on the compute stream while a side stream
        # waits for the peers (barrier) and gathers their rows.  The peers'
        # segments then go through the GEMM whose epilogue stores each row on
        # its source rank.
        own = counts[:, 0].copy()
        o0 = int(offs[r, r * El])
        n_own = int(own.sum())
        peer = counts.copy()
        peer[:, 0] = 0
        n_peer = int(peer.sum())
        x = self._buffer("_x", n_peer, dim, a)
        main = torch.cuda.current_stream(a.device)
        if self._side is None or self._side.device != a.device:
            self._side = torch.cuda.Stream(device=a.device)
        side = self._side
        side.wait_stream(main)  # token rows written, previous step's reads of x done
        self._mark(a.device, "start")
        with torch.cuda.stream(side):
            if W > 1:
                self._barrier(a.device)  # every rank's token rows are in place
            self._mark(a.device, "barrier_in")
            if n_peer:
                capi.ep_gather(x, sym[7], peer, rows_at, El, dim * a.element_size(), rank_base=r)
            self._mark(a.device, "gather")
        if n_own:
            capi.forward(a_sym[o0:o0 + n_own], b_local, own, res[o0:o0 + n_own], trans_b=trans_b)
        self._mark(a.device, "own_gemm")
        main.wait_stream(side)
        if n_peer:
            capi.forward_ep(x, b_local, peer, rows_at, El, sym[8], trans_b=trans_b, rank_base=r)
        self._mark(a.device, "peer_gemm")
        if W > 1:
            self._barrier(a.device)  # every peer's result rows have landed here
        self._mark(a.device, "barrier_out")
        return self._result(res, out)

    @staticmethod
    def _result(res, out):
        if out is None:
            return res.clone()
        if out.data_ptr() != res.data_ptr():
            out.copy_(res)
        return out

    def phase_ms(self):
        """Milliseconds of the last direct step's phases (``record_phases`` must
        have been set), each from the step's start: when the entry barrier, the
        gather, the own-rows GEMM, the peer-rows GEMM (+ combine) and the exit
        barrier had finished."""
        ev = self.phase_events
        if not ev or "start" not in ev:
            return None
        return {k: ev["start"].elapsed_time(e) for k, e in ev.items() if k != "start"}

    # --------------------------------------------------------------- forward
    def forward(self, a: torch.Tensor, b_local: torch.Tensor, batch_sizes: torch.Tensor,
                trans_b: bool = False, all_bs: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``out[rows_g] = a[rows_g] @ B[g]`` for this rank's rows, with B sharded by expert.

        Args:
            a: ``[T_r, dim]`` this rank's rows, grouped by global expert.
            b_local: ``[E/W, dim, dim_out]`` (``[E/W, dim_out, dim]`` if trans_b), the
                weights of the experts this rank owns.
            batch_sizes: ``[E]`` CPU int64, this rank's rows per global expert.
            all_bs: the gathered ``[W, E]`` counts, if the caller already has them.
            out: ``[T_r, dim_out]`` tensor for the result (default: a new tensor);
                ``output_buffer(...)`` avoids the copy out of symmetric memory.
        """
        W, El, r = self.world, self.e_local, self.rank
        if a.dim() != 2 or b_local.dim() != 3 or b_local.shape[0] != El:
            raise ValueError(f"expected a [T, dim] and b_local [{El}, ...], got "
                             f"{tuple(a.shape)} and {tuple(b_local.shape)}")
        if int(batch_sizes.sum()) != a.shape[0]:
            raise ValueError(f"Sum of batch_sizes ({int(batch_sizes.sum())}) must equal "
                             f"A.size(0) ({a.shape[0]})")
        if all_bs is None:
            all_bs = self.exchange_counts(batch_sizes)
        if out is not None and (tuple(out.shape) != (a.shape[0], b_local.shape[1] if trans_b else b_local.shape[2])
                                or out.dtype != a.dtype or out.device != a.device):
            raise ValueError("out must be a [T_r, dim_out] tensor of a's dtype and device")
        if self._use_direct(a):
            torch.cuda.nvtx.range_push("gmm_b200 ep forward (direct)")  # Nsight timeline marker
            try:
                return self._forward_direct(a, b_local, all_bs, trans_b, out)
            finally:
                torch.cuda.nvtx.range_pop()
        bs = all_bs.tolist()
        ch = _Chunking(bs, W, El, self.chunks)
        C = ch.chunks
        dim = a.shape[1]
        dim_out = b_local.shape[1] if trans_b else b_local.shape[2]

        # this rank's row offsets per global expert (its A / output layout)
        my_off, o = [], 0
        for g in range(self.num_experts):
            my_off.append(o)
            o += bs[r][g]
        # expert-major receive offsets on this rank: (e, s)
        recv_off, off = [], 0
        for e in range(El):
            row = []
            for s in range(W):
                row.append(off)
                off += bs[s][r * El + e]
            recv_off.append(row)
        n_recv = off
        x = self._buffer("_x", n_recv, dim, a)
        y = self._buffer("_y", n_recv, dim_out, a)
        if out is None:
            out = torch.empty(a.shape[0], dim_out, dtype=a.dtype, device=a.device)

        # ---- dispatch: all batches posted up front, one per chunk
        pending = []
        for c in range(C):
            ops: List[dist.P2POp] = []
            for p in range(W):  # sends: my rows for p's chunk-c experts
                if p == r:
                    continue
                for (e, s0, s1, _) in ch.owner_chunks[p][c]:
                    g = p * El + e
                    m = bs[r][g]
                    if m and s0 <= r < s1:
                        ops.append(dist.P2POp(dist.isend, a[my_off[g]:my_off[g] + m],
                                              self._peer[p], self.group))
            for s in range(W):  # receives: rows from s for my chunk-c blocks
                if s == r:
                    continue
                for (e, s0, s1, _) in ch.owner_chunks[r][c]:
                    m = bs[s][r * El + e]
                    if m and s0 <= s < s1:
                        ops.append(dist.P2POp(dist.irecv, x[recv_off[e][s]:recv_off[e][s] + m],
                                              self._peer[s], self.group))
            pending.append(dist.batch_isend_irecv(ops) if ops else [])
        for e in range(El):  # own rows
            g = r * El + e
            m = bs[r][g]
            if m:
                x[recv_off[e][r]:recv_off[e][r] + m].copy_(a[my_off[g]:my_off[g] + m])

        # ---- per chunk: GEMM, then combine (overlaps the next chunk's GEMM)
        combine_works = []
        for c in range(C):
            for w in pending[c]:
                w.wait()
            blocks = ch.owner_chunks[r][c]
            if blocks:
                e_first, e_last = blocks[0][0], blocks[-1][0]
                row0 = recv_off[e_first][blocks[0][1]]
                per_e = [0] * (e_last - e_first + 1)
                for (e, s0, s1, rows) in blocks:
                    per_e[e - e_first] += rows
                n = sum(per_e)
                self._gemm_into(x[row0:row0 + n], b_local[e_first:e_last + 1], per_e, trans_b,
                                y[row0:row0 + n])
            ops = []
            for s in range(W):  # sends back: my chunk-c results owned by source s
                if s == r:
                    continue
                for (e, s0, s1, _) in blocks:
                    m = bs[s][r * El + e]
                    if m and s0 <= s < s1:
                        ops.append(dist.P2POp(dist.isend, y[recv_off[e][s]:recv_off[e][s] + m],
                                              self._peer[s], self.group))
            for p in range(W):  # receives: my rows computed in p's chunk c
                if p == r:
                    continue
                for (e, s0, s1, _) in ch.owner_chunks[p][c]:
                    g = p * El + e
                    m = bs[r][g]
                    if m and s0 <= r < s1:
                        ops.append(dist.P2POp(dist.irecv, out[my_off[g]:my_off[g] + m],
                                              self._peer[p], self.group))
            for (e, s0, s1, _) in blocks:  # own rows back
                g = r * El + e
                m = bs[r][g]
                if m and s0 <= r < s1:
                    out[my_off[g]:my_off[g] + m].copy_(y[recv_off[e][r]:recv_off[e][r] + m])
            if ops:
                combine_works.extend(dist.batch_isend_irecv(ops))
        for w in combine_works:
            w.wait()
        return out

    __call__ = forward
