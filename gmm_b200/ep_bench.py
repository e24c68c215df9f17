"""Expert-parallel leg of ``bench.py`` (one process per GPU, launched by torchrun).

Workloads (``--config``):

* 2 (default): cfg2 shapes, weak scaling -- every rank routes 8192 tokens
  (top-2 over the 8 experts) and owns E/N experts; at N = 1 this is exactly
  the single-GPU cfg2 workload.
* 5: cfg5 (Mixtral-8x22B shapes), strong scaling -- 32768 tokens in total,
  split evenly over the ranks; 8/N experts per rank.
* 3: cfg3 (DeepSeek-V3 shapes, fp16 NT), strong scaling -- 4096 tokens in total,
  256/N experts per rank.

A step is the host count exchange + NCCL dispatch + local grouped GEMM +
NCCL combine (``gmm_b200.ep.ExpertParallelGmm``).  Time is measured with CUDA
events on each rank's stream between barriers and reduced with MAX over the
ranks; ``value`` is whole-job FLOPs per second, ``tokens_per_s`` pre-top-k
tokens per second.
"""

from __future__ import annotations

import datetime
import json
import math
import os
import statistics

import torch
import torch.distributed as dist


def _routing(cfg, world, rank):
    """This rank's token shard of one global routing draw (same on every rank)."""
    from gmm_b200.configs import route
    weak = cfg.cid == 2
    tokens_r = cfg.tokens if weak else cfg.tokens // world
    total = tokens_r * world
    gen = torch.Generator().manual_seed(cfg.seed)
    ids = route(cfg, gen, tokens=total)
    mine = ids[rank * tokens_r:(rank + 1) * tokens_r]
    bs = torch.bincount(mine.flatten(), minlength=cfg.num_experts).to(torch.int64)
    return bs, tokens_r, total, weak


def _local_weights(cfg, experts, device):
    from gmm_b200.configs import b_shape
    shape = b_shape(cfg, len(experts))
    b = torch.empty(*shape, dtype=cfg.dtype, device=device)
    s = 1.0 / math.sqrt(cfg.dim)
    for i, e in enumerate(experts):
        g = torch.Generator(device=device).manual_seed(cfg.seed * 100003 + e)
        b[i].copy_(torch.randn(*shape[1:], generator=g, device=device).mul_(s))
    return b


def run(args, metric, load_peaks, clock_sampler):
    from gmm_b200.configs import CONFIGS
    from gmm_b200.ep import ExpertParallelGmm

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
        E = cfg.num_experts
        if E % world:
            raise SystemExit(f"cfg{cid}: {E} experts do not split over {world} ranks")
        El = E // world
        bs, tokens_r, tokens_total, weak = _routing(cfg, world, rank)
        rows_r = int(bs.sum())
        b_local = _local_weights(cfg, list(range(rank * El, (rank + 1) * El)), dev)
        ep = ExpertParallelGmm(E, count_group=count_group,
                               transport=os.environ.get("GMM_EP_TRANSPORT", "auto"))
        all_bs = ep.exchange_counts(bs)
        g = torch.Generator(device=dev).manual_seed(cfg.seed * 7919 + rank)
        if ep._use_direct(b_local):
            # the layer's input rows live in this rank's symmetric token buffer
            a = ep.input_buffer(int(all_bs.sum(1).max()), cfg.dim, cfg.dim_out, cfg.dtype, dev)[:rows_r]
            a.copy_(torch.randn(rows_r, cfg.dim, generator=g, device=dev))
        else:
            a = torch.randn(rows_r, cfg.dim, generator=g, device=dev).to(cfg.dtype)

        rows_all = torch.tensor([rows_r], dtype=torch.float64, device=dev)
        dist.all_reduce(rows_all)
        flops = 2.0 * rows_all.item() * cfg.dim * cfg.dim_out

        for _ in range(max(3, args.warmup)):
            ep(a, b_local, bs, cfg.trans_b)
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
                ep(a, b_local, bs, cfg.trans_b)
            t1.record(stream)
            torch.cuda.synchronize()
        ms = torch.tensor([t0.elapsed_time(t1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        step_ms = ms.item()
        dist.barrier()

        # e2e: A_r and this rank's expert weights from pinned host memory, out back to host
        a_h = a.cpu().pin_memory()
        b_h = b_local.cpu().pin_memory()
        a_d, b_d = a, torch.empty_like(b_local)  # inputs land where the layer reads them
        out_h = torch.empty(rows_r, cfg.dim_out, dtype=cfg.dtype).pin_memory()

        def e2e_step():
            a_d.copy_(a_h, non_blocking=True)
            b_d.copy_(b_h, non_blocking=True)
            out = ep(a_d, b_d, bs, cfg.trans_b)
            out_h.copy_(out, non_blocking=True)

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
        ems = torch.tensor([e0.elapsed_time(e1) / e_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        es = a.element_size()
        h2d = torch.tensor([float((a.numel() + b_local.numel()) * es)], dtype=torch.float64, device=dev)
        d2h = torch.tensor([float(rows_r * cfg.dim_out * es)], dtype=torch.float64, device=dev)
        dist.all_reduce(h2d)
        dist.all_reduce(d2h)

        if rank == 0:
            peaks, src = load_peaks()
            value = flops / (step_ms * 1e-3) / 1e12
            per_gpu = value / world
            line = {
                "metric": metric, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
                "tokens_per_s": round(tokens_total / (step_ms * 1e-3), 1),
                "higher_is_better": True, "scaling": "weak" if weak else "strong",
                "vs_baseline": None,
                "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[cfg.dtype],
                "data": "synthetic (one seeded global routing draw, token-sharded; "
                        "A ~ N(0,1), B ~ N(0,1/dim))",
                "config": {"workload": f"cfg{cid}: {cfg.name}, expert parallel",
                           "experts": E, "experts_per_rank": El, "dim": cfg.dim,
                           "dim_out": cfg.dim_out, "tokens": tokens_total, "top_k": cfg.top_k,
                           "rows": int(rows_all.item()), "trans_b": cfg.trans_b,
                           "parallelism": f"ep{world}",
                           "l2": "inputs larger than L2 (126 MB)",
                           "exchange": (("shared-memory" if ep._shm_counts is not None else "gloo")
                                        + " count all-gather; "
                                        + ("NVLink peer-load gather + combine fused into the GEMM "
                                           "epilogue (symmetric memory)" if ep._use_direct(b_local)
                                           else "NCCL P2P dispatch/combine"))},
                "e2e": {"value": round(flops / (ems.item() * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                        "ms_per_step": round(ems.item(), 3),
                        "h2d_bytes_per_step": int(h2d.item()), "d2h_bytes_per_step": int(d2h.item()),
                        "path": "pinned host A_r, B_local -> device; EP forward; out -> pinned host"},
                "gpu_launches": args.steps * world,
                "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2),
                             "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": round(per_gpu / peaks["bf16_tflops"], 4), "traffic": None,
                             "peak_source": f"{src} (burst); achieved = whole-job TFLOP/s / N, "
                                            "including the NCCL exchange"},
                "clocks": clk.summary(),
            }
            print(json.dumps(line), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()
