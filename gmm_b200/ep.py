"""Expert parallelism around the grouped-GEMM forward.

The reference runs the grouped GEMM on one GPU only (it has no distributed
code); this layer shards the E experts of one MoE projection across the
ranks of a process group -- one process per GPU, NCCL over NVLink -- and
moves token rows with one exchange step each way:

1. counts: every rank's host ``batch_sizes`` (rows per global expert) are
   all-gathered over a CPU (gloo) group, so every split size is known on the
   host without a device synchronisation;
2. dispatch: rank r's rows for expert g go to g's owner, posted as one NCCL
   point-to-point message per (expert, peer) chunk that lands directly in
   the owner's expert-major receive buffer (all sources of local expert 0,
   then of local expert 1, ...);
3. local grouped GEMM over the E/W local experts (``hopper_gmm_fwd``), one
   contiguous segment per local expert;
4. combine: each (expert, source) block of the result goes back to its
   source, into the rows the source's A occupied.

Rank r owns experts ``[r*E/W, (r+1)*E/W)``.  The output rows are the input
rows' results, bit-identical to the single-GPU op on the same rows.  There
is no CPU fallback: ``local_gemm`` defaults to the CUDA operator; only the
tests substitute the CPU oracle to check the exchange logic on gloo ranks.
"""

from __future__ import annotations

from typing import Callable, List, Optional

import torch
import torch.distributed as dist


def _default_local_gemm(a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor,
                        trans_b: bool) -> torch.Tensor:
    from gmm_b200 import hopper_gmm_fwd
    return hopper_gmm_fwd(a, b, batch_sizes, trans_b=trans_b)


class ExpertParallelGmm:
    """Expert-parallel grouped GEMM forward over a process group.

    Args:
        num_experts: global number of experts E (divisible by the world size).
        group: process group carrying the token rows (NCCL for GPUs).
        count_group: CPU (gloo) group for the host-side count exchange; created
            from the world if not given.
        local_gemm: ``f(a, b_local, batch_sizes, trans_b) -> d`` for the local
            experts; the CUDA operator unless a test substitutes a checker.
    """

    def __init__(self, num_experts: int, group=None, count_group=None,
                 local_gemm: Optional[Callable] = None):
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
        self.local_gemm = local_gemm or _default_local_gemm
        self._peer_ranks = [dist.get_global_rank(group, i) if group is not None else i
                            for i in range(self.world)]

    # ------------------------------------------------------------------ plan
    def exchange_counts(self, batch_sizes: torch.Tensor) -> torch.Tensor:
        """All ranks' ``batch_sizes`` as a ``[W, E]`` int64 CPU tensor."""
        if batch_sizes.device.type != "cpu" or batch_sizes.dtype != torch.int64 \
                or batch_sizes.dim() != 1 or batch_sizes.numel() != self.num_experts:
            raise ValueError("batch_sizes must be a 1D CPU int64 tensor with num_experts entries")
        if (batch_sizes < 0).any():
            raise ValueError("batch_sizes must be non-negative")
        out = [torch.empty_like(batch_sizes) for _ in range(self.world)]
        dist.all_gather(out, batch_sizes.contiguous(), group=self.count_group)
        return torch.stack(out)

    def plan(self, all_bs: torch.Tensor):
        """Split sizes and offsets of one exchange, from the gathered counts."""
        W, El, r = self.world, self.e_local, self.rank
        bs = all_bs.tolist()
        mine = [[bs[s][r * El + e] for s in range(W)] for e in range(El)]  # [local e][src]
        local_bs = [sum(row) for row in mine]
        # expert-major receive offsets: (e, s)
        recv_off = []
        off = 0
        for e in range(El):
            row = []
            for s in range(W):
                row.append(off)
                off += mine[e][s]
            recv_off.append(row)
        # this rank's own row offsets per global expert (its A / output layout)
        my_off, o = [], 0
        for g in range(self.num_experts):
            my_off.append(o)
            o += bs[r][g]
        return mine, local_bs, recv_off, my_off, off

    # --------------------------------------------------------------- forward
    def forward(self, a: torch.Tensor, b_local: torch.Tensor, batch_sizes: torch.Tensor,
                trans_b: bool = False, all_bs: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``out[rows_g] = a[rows_g] @ B[g]`` for this rank's rows, with B sharded by expert.

        Args:
            a: ``[T_r, dim]`` this rank's rows, grouped by global expert.
            b_local: ``[E/W, dim, dim_out]`` (``[E/W, dim_out, dim]`` if trans_b), the
                weights of the experts this rank owns.
            batch_sizes: ``[E]`` CPU int64, this rank's rows per global expert.
            all_bs: the gathered ``[W, E]`` counts, if the caller already has them.
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
        mine, local_bs, recv_off, my_off, n_recv = self.plan(all_bs)
        my_bs = all_bs[r].tolist()
        dim = a.shape[1]
        dim_out = b_local.shape[1] if trans_b else b_local.shape[2]

        # ---- dispatch
        x = torch.empty(n_recv, dim, dtype=a.dtype, device=a.device)
        ops: List[dist.P2POp] = []
        for g in range(self.num_experts):  # sends, in global expert order per peer
            m = my_bs[g]
            p = g // El
            if m == 0 or p == r:
                continue
            ops.append(dist.P2POp(dist.isend, a[my_off[g]:my_off[g] + m], self._peer_ranks[p],
                                  self.group))
        for e in range(El):  # receives, in local expert order per peer
            for s in range(W):
                m = mine[e][s]
                if m == 0 or s == r:
                    continue
                ops.append(dist.P2POp(dist.irecv, x[recv_off[e][s]:recv_off[e][s] + m],
                                      self._peer_ranks[s], self.group))
        for e in range(El):  # own rows: local copy
            g = r * El + e
            m = my_bs[g]
            if m:
                x[recv_off[e][r]:recv_off[e][r] + m].copy_(a[my_off[g]:my_off[g] + m])
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

        # ---- local grouped GEMM
        y = self.local_gemm(x, b_local, torch.tensor(local_bs, dtype=torch.int64), trans_b)

        # ---- combine
        out = torch.empty(a.shape[0], dim_out, dtype=y.dtype, device=a.device)
        ops = []
        for e in range(El):  # sends back, in local expert order per source
            for s in range(W):
                m = mine[e][s]
                if m == 0 or s == r:
                    continue
                ops.append(dist.P2POp(dist.isend, y[recv_off[e][s]:recv_off[e][s] + m],
                                      self._peer_ranks[s], self.group))
        for g in range(self.num_experts):  # receives, in global expert order per owner
            m = my_bs[g]
            p = g // El
            if m == 0 or p == r:
                continue
            ops.append(dist.P2POp(dist.irecv, out[my_off[g]:my_off[g] + m], self._peer_ranks[p],
                                  self.group))
        for e in range(El):
            g = r * El + e
            m = my_bs[g]
            if m:
                out[my_off[g]:my_off[g] + m].copy_(y[recv_off[e][r]:recv_off[e][r] + m])
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        return out

    __call__ = forward
