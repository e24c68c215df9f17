"""Expert-parallel leg of ``bench.py`` (one process per GPU, launched by torchrun),
and the in-run parity check both legs use.

Headline workload (``--config``, default 2): cfg2 shapes, weak scaling -- every
rank routes 8192 tokens (top-2 over the 8 experts) and owns E/N experts; at
N = 1 this is exactly the single-GPU cfg2 workload.  ``--config 5`` / ``3``
make cfg5 / cfg3 the headline instead (strong scaling).

Every N also reports ``ep_configs``: the two expert-parallel configurations
of the north star, strong-scaled --

* cfg5 (Mixtral-8x22B shapes, bf16 NN): 32768 tokens in total, split evenly
  over the ranks; 8/N experts per rank;
* cfg3 (DeepSeek-V3 shapes, fp16 NT): 4096 tokens in total, 256/N experts
  per rank --

with the experts placed by load (``balanced_placement`` of another batch's
routed rows; ``GMM_EP_PLACEMENT=contiguous`` for E/N-expert blocks), each with
its step time, tokens/s, whole-job TFLOP/s, the load-imbalance ceiling of its
routing (mean / max rows computed per rank, also for contiguous blocks) and
``parity``:
sampled output rows of every rank, two or more per global expert (so every
rank's local experts are covered), against a plain PyTorch fp32 reference on
the GPU at the north-star tolerance.

A timed step is dispatch + local grouped GEMM + combine
(``gmm_b200.ep.ExpertParallelGmm``, direct transport: NVLink peer-load gather,
combine fused into the GEMM epilogue, flag barriers).  The routing is the same
every step, so the host count exchange runs once before the timed steps; its
own host cost (mean microseconds per ``exchange_counts`` call, max over ranks)
is reported beside the step time as ``count_exchange_us``.  Time is measured
with CUDA events on each rank's stream between barriers and reduced with MAX
over the ranks.
"""

from __future__ import annotations

import datetime
import json
import math
import os

import torch
import torch.distributed as dist


# ------------------------------------------------------------------ parity
def check_parity(out, a, bs, get_b, trans_b, rows_per_expert=2, seed=0, max_experts=None):
    """Sampled rows of ``out`` (grouped by expert per ``bs``) against a plain
    PyTorch fp32 matmul on the GPU, rounded to the output dtype.

    For every non-empty expert g (or the first ``max_experts`` of them) its first
    and last row and ``rows_per_expert`` random rows are checked against
    ``a[rows].float() @ B[g].float()`` with ``B[g] = get_b(g)``; tolerance
    rtol = atol from the north star (bf16 1.6e-2, fp16 2e-3, fp32 5e-3).
    Returns a JSON-ready summary."""
    from gmm_b200.configs import TOLERANCE
    tol = TOLERANCE[out.dtype]
    g = torch.Generator().manual_seed(seed)
    bsl = [int(v) for v in bs]
    off = 0
    n_rows = n_bad = n_exp = 0
    max_err = 0.0
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for e, m in enumerate(bsl):
            if m > 0 and (max_experts is None or n_exp < max_experts):
                rows = {off, off + m - 1}
                rows.update(int(v) for v in torch.randint(off, off + m, (rows_per_expert,), generator=g))
                idx = torch.tensor(sorted(rows), device=out.device)
                b = get_b(e).float()
                want = a[idx].float() @ (b.t() if trans_b else b)
                want = want.to(out.dtype).float()
                got = out[idx].float()
                err = (got - want).abs()
                n_bad += int((err > tol + tol * want.abs()).sum())
                if not torch.isfinite(got).all():
                    n_bad += 1
                max_err = max(max_err, float(err.max()))
                n_rows += len(rows)
                n_exp += 1
            off += m
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    return {"ok": n_bad == 0, "rows": n_rows, "experts": n_exp, "bad_elements": n_bad,
            "max_abs_err": max_err, "tol": tol,
            "reference": "torch fp32 matmul on the GPU (TF32 off), rounded to the output dtype"}


# ------------------------------------------------------------------ workloads
def routing(cfg, world, rank, weak, perm=None):
    """This rank's token shard of one global routing draw (same on every rank).

    ``perm`` (an expert placement, ``perm[label] = expert``): expert ids are
    relabelled so that rank r's experts are labels ``[r*E/W, (r+1)*E/W)``."""
    from gmm_b200.configs import route
    tokens_r = cfg.tokens if weak else cfg.tokens // world
    total = tokens_r * world
    gen = torch.Generator().manual_seed(cfg.seed)
    ids = route(cfg, gen, tokens=total)
    if perm is not None:
        inv = torch.empty(len(perm), dtype=torch.int64)
        inv[torch.as_tensor(perm)] = torch.arange(len(perm))
        ids = inv[ids]
    bs_all = [torch.bincount(ids[r * tokens_r:(r + 1) * tokens_r].flatten(),
                             minlength=cfg.num_experts).to(torch.int64) for r in range(world)]
    return bs_all[rank], tokens_r, total, torch.stack(bs_all)


def expert_weight(cfg, e, device):
    """B[e] of the expert-parallel workloads: its own seeded draw, so any rank can
    regenerate any expert's weights (the parity check does)."""
    from gmm_b200.configs import b_shape
    shape = b_shape(cfg, 1)[1:]
    gen = torch.Generator(device=device).manual_seed(cfg.seed * 100003 + e)
    w = torch.randn(*shape, generator=gen, device=device).mul_(1.0 / math.sqrt(cfg.dim))
    return w.to(cfg.dtype)


def local_weights(cfg, experts, device):
    from gmm_b200.configs import b_shape
    b = torch.empty(*b_shape(cfg, len(experts)), dtype=cfg.dtype, device=device)
    for i, e in enumerate(experts):
        b[i].copy_(expert_weight(cfg, e, device))
    return b


def _dtype_name(dtype):
    return {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[dtype]


def _max_over_ranks(v, dev):
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _sum_over_ranks(v, dev):
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return t.item()


class _Setup:
    """One expert-parallel workload on this rank: routing, weights, inputs, layer."""

    def __init__(self, cfg, world, rank, dev, count_group, weak, barrier="flags", placement="contiguous"):
        from gmm_b200.configs import history_loads
        from gmm_b200.ep import ExpertParallelGmm, balanced_placement
        self.cfg, self.world, self.rank, self.dev = cfg, world, rank, dev
        E = cfg.num_experts
        if E % world:
            raise SystemExit(f"cfg{cfg.cid}: {E} experts do not split over {world} ranks")
        self.El = El = E // world
        # expert placement: label l is expert perm[l]; rank r owns labels [r*El, (r+1)*El)
        self.placement = placement
        self.perm = (balanced_placement(history_loads(cfg), world) if placement == "balanced"
                     else list(range(E)))
        self.bs, self.tokens_r, self.tokens_total, all_bs = routing(
            cfg, world, rank, weak, self.perm if placement == "balanced" else None)
        self.rows_r = int(self.bs.sum())
        self.b_local = local_weights(cfg, [self.perm[l] for l in range(rank * El, (rank + 1) * El)], dev)
        self.ep = ExpertParallelGmm(E, count_group=count_group,
                                    transport=os.environ.get("GMM_EP_TRANSPORT", "auto"), barrier=barrier)
        self.ep.overlap = os.environ.get("GMM_EP_OVERLAP", "1") != "0"
        self.all_bs = self.ep.exchange_counts(self.bs)
        assert torch.equal(self.all_bs, all_bs), "count exchange disagrees with the routing draw"
        g = torch.Generator(device=dev).manual_seed(cfg.seed * 7919 + rank)
        cap = int(self.all_bs.sum(1).max())
        self.direct = self.ep._use_direct(self.b_local)
        if self.direct:
            # the layer's input rows live in this rank's symmetric token buffer and
            # its result stays in the symmetric output buffer (no copies)
            self.a = self.ep.input_buffer(cap, cfg.dim, cfg.dim_out, cfg.dtype, dev)[:self.rows_r]
            self.a.copy_(torch.randn(self.rows_r, cfg.dim, generator=g, device=dev))
            self.out = self.ep.output_buffer(cap, cfg.dim, cfg.dim_out, cfg.dtype, dev)[:self.rows_r]
        else:
            self.a = torch.randn(self.rows_r, cfg.dim, generator=g, device=dev).to(cfg.dtype)
            self.out = torch.empty(self.rows_r, cfg.dim_out, dtype=cfg.dtype, device=dev)
        self.rows_total = _sum_over_ranks(self.rows_r, dev)
        self.flops = 2.0 * self.rows_total * cfg.dim * cfg.dim_out
        # rows each rank's GEMM computes: every rank's rows for its local experts
        per_rank = self.all_bs.view(world, world, El).sum(dim=(0, 2)).double()
        self.imbalance = {"rows_per_rank_max": int(per_rank.max()), "rows_per_rank_mean": float(per_rank.mean()),
                          "efficiency_ceiling": round(float(per_rank.mean() / per_rank.max()), 4)}
        if placement == "balanced":  # what the contiguous placement would have given
            contig = routing(cfg, world, rank, weak)[3].view(world, world, El).sum(dim=(0, 2)).double()
            self.imbalance["efficiency_ceiling_contiguous"] = round(float(contig.mean() / contig.max()), 4)

    def exchange_us(self, calls=20):
        """Host microseconds per count exchange (mean of ``calls``, max over ranks)."""
        import time
        dist.barrier(group=self.ep.count_group)
        t0 = time.perf_counter()
        for _ in range(calls):
            got = self.ep.exchange_counts(self.bs)
        us = (time.perf_counter() - t0) / calls * 1e6
        assert torch.equal(got, self.all_bs)
        return round(_max_over_ranks(us, self.dev), 1)

    def step(self):
        return self.ep(self.a, self.b_local, self.bs, self.cfg.trans_b, all_bs=self.all_bs, out=self.out)

    def timed(self, steps, warmup):
        for _ in range(max(3, warmup)):
            self.step()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(steps):
            self.step()
        t1.record(stream)
        torch.cuda.synchronize()
        return _max_over_ranks(t0.elapsed_time(t1) / steps, self.dev)

    def parity(self):
        """This rank's output rows (the last step's) for every global expert."""
        cfg, El = self.cfg, self.El

        def get_b(label):
            if self.rank * El <= label < (self.rank + 1) * El:
                return self.b_local[label - self.rank * El]
            return expert_weight(cfg, self.perm[label], self.dev)

        res = check_parity(self.out, self.a, self.bs.tolist(), get_b, cfg.trans_b, seed=self.rank)
        ok = _sum_over_ranks(0 if res["ok"] else 1, self.dev) == 0
        return {"ok": ok, "rows_checked": int(_sum_over_ranks(res["rows"], self.dev)),
                "max_abs_err": _max_over_ranks(res["max_abs_err"], self.dev), "tol": res["tol"],
                "reference": res["reference"] + "; 2+ rows per (rank, global expert)"}

    def phases(self):
        if not self.direct:
            return None
        self.ep.record_phases = True
        self.step()
        torch.cuda.synchronize()
        ph = self.ep.phase_ms()
        self.ep.record_phases = False
        return {k: round(_max_over_ranks(v, self.dev), 4) for k, v in ph.items()}

    def close(self):
        del self.a, self.out, self.b_local, self.ep
        torch.cuda.empty_cache()


def ep_config_entry(setup, ms, world):
    cfg = setup.cfg
    return {"workload": f"cfg{cfg.cid}: {cfg.name}", "dtype": _dtype_name(cfg.dtype),
            "scaling": "strong", "tokens": setup.tokens_total, "experts_per_rank": setup.El,
            "placement": ("load-balanced: experts placed heaviest-first on the least-loaded rank, "
                          "by the routed rows of another batch of the same expert popularity"
                          if setup.placement == "balanced" else "contiguous blocks of E/N experts"),
            "ms_per_step": round(ms, 4), "tokens_per_s": round(setup.tokens_total / (ms * 1e-3), 1),
            "tflops": round(setup.flops / (ms * 1e-3) / 1e12, 2), "n_gpus": world,
            "load_imbalance": setup.imbalance}


def run(args, metric, load_peaks, clock_sampler):
    from gmm_b200.configs import CONFIGS, workload_config

    # NCCL keeps P2P tensors alive until wait() instead of recording them on its
    # stream, so the allocator can reuse them at once on the compute stream.
    os.environ.setdefault("TORCH_NCCL_AVOID_RECORD_STREAMS", "1")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    count_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    try:
        cid = args.config or 2
        cfg = CONFIGS[cid]
        weak = cid == 2
        s = _Setup(cfg, world, rank, dev, count_group, weak, barrier=os.environ.get("GMM_EP_BARRIER", "flags"))
        for _ in range(max(3, args.warmup)):
            s.step()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with clock_sampler(local_rank if rank == 0 else -1) as clk:
            # all ranks start the timed region together (the sampler start-up
            # on rank 0 must not count as a peer wait on the other ranks)
            dist.barrier()
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(args.steps):
                s.step()
            t1.record(stream)
            torch.cuda.synchronize()
        step_ms = _max_over_ranks(t0.elapsed_time(t1) / args.steps, dev)
        head_parity = s.parity()
        head_xchg = s.exchange_us()
        phases = s.phases() if args.phases else None
        dist.barrier()

        # e2e: A_r and this rank's expert weights from pinned host memory, result back to host
        a_h = s.a.cpu().pin_memory()
        b_h = s.b_local.cpu().pin_memory()
        b_d = torch.empty_like(s.b_local)
        out_h = torch.empty(s.rows_r, cfg.dim_out, dtype=cfg.dtype).pin_memory()

        def e2e_step():
            s.a.copy_(a_h, non_blocking=True)  # inputs land where the layer reads them
            b_d.copy_(b_h, non_blocking=True)
            o = s.ep(s.a, b_d, s.bs, cfg.trans_b, all_bs=s.all_bs, out=s.out)
            out_h.copy_(o, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e_steps = max(1, min(args.e2e_steps, args.steps))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / e_steps, dev)
        es = s.a.element_size()
        h2d = _sum_over_ranks((s.a.numel() + s.b_local.numel()) * es, dev)
        d2h = _sum_over_ranks(s.rows_r * cfg.dim_out * es, dev)
        head_imb = s.imbalance
        transport = s.direct
        overlap = s.ep.overlap
        barrier_kind = "flag-kernel" if s.ep.barrier == "flags" else "NCCL all-reduce"
        shm = s.ep._shm_counts is not None
        flops, tokens_total, rows_total, El = s.flops, s.tokens_total, s.rows_total, s.El
        s.close()
        del b_d, b_h, a_h

        # the north star's expert-parallel configurations, strong-scaled
        ep_configs = {}
        if not args.no_configs:
            for ecid in (5, 3):
                es_ = _Setup(CONFIGS[ecid], world, rank, dev, count_group, weak=False,
                             barrier=os.environ.get("GMM_EP_BARRIER", "flags"),
                             placement=os.environ.get("GMM_EP_PLACEMENT", "balanced"))
                ms = es_.timed(max(3, min(args.steps, 20)), args.warmup)
                entry = ep_config_entry(es_, ms, world)
                entry["count_exchange_us"] = es_.exchange_us()
                entry["parity"] = es_.parity()
                if args.phases:
                    entry["phases_ms"] = es_.phases()
                ep_configs[f"cfg{ecid}"] = entry
                es_.close()
                dist.barrier()

        if rank == 0:
            peaks, src = load_peaks()
            value = flops / (step_ms * 1e-3) / 1e12
            per_gpu = value / world
            line = {
                "metric": metric, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
                "tokens_per_s": round(tokens_total / (step_ms * 1e-3), 1),
                "higher_is_better": True, "scaling": "weak" if weak else "strong",
                "vs_baseline": None, "dtype": _dtype_name(cfg.dtype),
                "data": "synthetic (one seeded global routing draw, token-sharded; "
                        "A ~ N(0,1), B ~ N(0,1/dim))",
                "config": workload_config(cfg, world, weak),
                "ep": {"experts_per_rank": El, "rows": int(rows_total),
                       "exchange": (("shared-memory" if shm else "gloo") + " count all-gather; "
                                    + ("NVLink peer-load gather + combine fused into the GEMM "
                                       "epilogue (symmetric memory); own-rows GEMM overlapping the "
                                       "gather" if transport and overlap else
                                       "NVLink peer-load gather + combine fused into the GEMM "
                                       "epilogue (symmetric memory)" if transport
                                       else "NCCL P2P dispatch/combine")
                                    + f"; {barrier_kind} barriers"),
                       "load_imbalance": head_imb, "count_exchange_us": head_xchg},
                "parity": head_parity,
                "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                        "ms_per_step": round(e2e_ms, 3),
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                        "path": "pinned host A_r, B_local -> device; EP forward; out -> pinned host"},
                "gpu_launches": args.steps * (5 if transport and overlap else 4 if transport else 1),
                "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2),
                             "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": round(per_gpu / peaks["bf16_tflops"], 4), "traffic": None,
                             "peak_source": f"{src} (burst); achieved = whole-job TFLOP/s / N, "
                                            "including the exchange"},
                "clocks": clk.summary(),
                "ep_configs": ep_configs,
            }
            if phases:
                line["phases_ms"] = phases
            print(json.dumps(line), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()
