"""Benchmark of the B200 grouped-GEMM forward (and its expert-parallel layer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

One JSON line on rank 0.  A "step" is one grouped-GEMM forward over the
configuration's full synthetic batch.

* N = 1 (default workload cfg2, the configuration the headline metric is
  quoted on): ``value`` = FLOPs / mean step time of ``hopper_gmm_fwd`` with
  inputs resident in HBM (CUDA events per step; the inputs are larger than
  the 126 MB L2); ``e2e`` = the same metric through the public host-operand
  call with A, B copied in from pinned host memory and D copied back every
  step; ``parity`` = sampled output rows of every expert against a PyTorch
  fp32 reference on the GPU; ``roofline.sustained_loop`` = >= 1 s of
  back-to-back steps after the timed region with the SM clock seen under
  load and the fraction of the dense tensor rate at that clock;
  ``configs`` = kernel time, roofline and parity of the other four
  workloads (cfg4's ``p50_us_per_call`` is its headline); ``ep_configs`` =
  the expert-parallel workloads (cfg5, cfg3) at N = 1, i.e. the local GEMM.
* N > 1 (launched by torchrun): expert parallelism -- each rank owns
  E/N experts and a 1/N share of the tokens (``gmm_b200.ep_bench``): the
  headline is cfg2 weak-scaled, ``ep_configs`` holds cfg5 and cfg3
  strong-scaled with in-run parity on every rank.  ``value`` = whole-job
  FLOPs / max-over-ranks step time; ``tokens_per_s`` = pre-top-k tokens /
  step time.
* ``--impl reference``: the reference's own CPU path (its per-expert
  ``ref_gmm`` loop, restated in ``oracle.ref_gmm_port``) on the host cores,
  on a bounded row sample of the same workload; rank 0 only; loads none of
  this repository's CUDA libraries.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ("grouped-GEMM TFLOP/s per B200 (% of tcgen05 peak); "
          "EP tokens/s at 1/2/4/8 GPUs")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=None,
                    help="workload config 1-5 (default: 2 at N=1, 2 with EP at N>1)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--max-experts", type=int, default=None,
                    help="keep only the first K experts (and their rows): a smaller case of the "
                         "same workload for ncu captures")
    ap.add_argument("--ffn", action="store_true",
                    help="time the MoE expert FFN (fused SwiGLU gate/up GEMM + down GEMM) on the "
                         "config's routing instead of the single grouped GEMM")
    ap.add_argument("--layer", action="store_true",
                    help="time the device-resident MoE layer (routing, permute, SwiGLU FFN, combine) "
                         "eagerly and as a replayed CUDA graph")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-configuration lines (configs / ep_configs)")
    ap.add_argument("--sustain-s", type=float, default=1.0,
                    help="seconds of back-to-back steps after the timed region, for the clock record")
    ap.add_argument("--phases", action="store_true",
                    help="N > 1: also time each phase of one expert-parallel step (barriers, gather, "
                         "GEMM + combine), max over ranks")
    ap.add_argument("--cublas", action="store_true",
                    help="N = 1: the configuration against cuBLAS (torch.matmul) per expert and as one GEMM")
    ap.add_argument("--cublas-variant", choices=["ours", "cublas_per", "cublas_one"], default=None,
                    help="with --cublas: time only this variant")
    ap.add_argument("--kernel-only", action="store_true",
                    help="warm-up + timed launches only (no e2e / CPU baseline / clocks): the "
                         "command profiled with ncu")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(key):
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling around the timed region.

    ``mark()`` notes host times; ``summary(window=i)`` restricts to the samples
    taken between mark i-1 and mark i (window 0: the whole span).  ``sm_mhz``
    is the median over the samples drawn under load (power above 40% of the
    largest sample), so idle samples around a short timed region do not count."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.marks = []
        self.lines = []

    def __enter__(self):
        if self.index < 0:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def mark(self):
        self.marks.append(time.time())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def _samples(self):
        import datetime
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, mx = float(parts[2]), float(parts[3])
                pw = float(parts[4]) if parts[4] not in ("", "[N/A]") else 0.0
            except ValueError:
                continue
            act = [n for n, v in zip(names, parts[6:10]) if v.lower().startswith("active")]
            yield ts, sm, mx, pw, act

    def summary(self, window=0):
        samples = list(self._samples())
        if window and len(self.marks) > window:
            lo, hi = self.marks[window - 1], self.marks[window]
            samples = [x for x in samples if lo <= x[0] <= hi]
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        pmax = max(x[3] for x in samples)
        loaded = [x for x in samples if x[3] >= 0.4 * pmax] or samples
        reasons = sorted({r for x in loaded for r in x[4]})
        return {"sm_mhz": statistics.median(x[1] for x in loaded), "sm_max_mhz": samples[-1][2],
                "reasons": reasons, "samples": len(samples), "samples_under_load": len(loaded),
                "power_w_max": pmax}


def cpu_rate(cfg, a_cpu, b_cpu, bs, budget_s=10.0):
    """Time the reference's CPU path (ref_gmm restated) on a bounded row sample.

    Returns (TFLOP/s, sample description, cores).  The sample keeps every
    expert's full B and takes the first r rows of each expert, r grown until
    one call takes about budget_s / 4 seconds."""
    import torch
    import oracle
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    bsl = [int(v) for v in bs]
    off = [0]
    for m in bsl:
        off.append(off[-1] + m)

    def sample(r):
        sub = [min(m, r) for m in bsl]
        idx = torch.cat([torch.arange(off[e], off[e] + sub[e]) for e in range(len(bsl)) if sub[e]])
        return a_cpu[idx], torch.tensor(sub, dtype=torch.int64), sum(sub)

    r = 8
    while True:
        a_s, bs_s, rows = sample(r)
        t0 = time.perf_counter()
        oracle.ref_gmm_port(a_s, b_cpu, bs_s, cfg.trans_b)
        dt = time.perf_counter() - t0
        if dt > budget_s / 4 or r >= max(bsl):
            break
        r = min(max(bsl), int(r * max(2.0, (budget_s / 4) / max(dt, 1e-4))))
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
        t0 = time.perf_counter()
        oracle.ref_gmm_port(a_s, b_cpu, bs_s, cfg.trans_b)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    flops = 2.0 * rows * cfg.dim * cfg.dim_out
    desc = (f"oracle.ref_gmm_port (torch CPU {oracle.dtype_name(cfg.dtype)}, per-expert matmul) "
            f"on the first {min(r, max(bsl))} rows of each expert ({rows} of {cfg.rows} rows, "
            f"all {len(bsl)} experts' B); median of {len(times)} runs")
    return flops / med / 1e12, desc, cores


# ------------------------------------------------------------------------ N = 1
def _workloads():
    """``gmm_b200/configs.py`` (seeded workload generators, no CUDA code) loaded by
    file path: importing it as ``gmm_b200.configs`` would run the package's
    ``__init__``, which loads the CUDA libraries -- the reference arm must not."""
    import importlib.util
    name = "gmm_b200_workloads"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "gmm_b200", "configs.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def _events_time(fn, steps, flush=None):
    """Per-step device milliseconds of ``fn`` (CUDA events on the current stream)."""
    import torch
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s_.elapsed_time(e) for s_, e in zip(starts, ends)]


def _pcie_bound(src_h, dst_h, h2d_bytes, d2h_bytes):
    """The e2e step's transfer bound on this box: one large pinned-host copy each
    way (from ``src_h``, into ``dst_h``), timed alone (CUDA events, median of
    3), and the step's bytes over those rates.  A full-duplex link overlaps the
    two directions, so the bound is the slower direction's time."""
    import torch
    n = min(src_h.numel(), dst_h.numel(), (256 << 20) // src_h.element_size())
    h = src_h.reshape(-1)[:n]
    o = dst_h.reshape(-1)[:n]
    d = torch.empty(n, dtype=h.dtype, device="cuda")

    def rate(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            fn()
            e_.record()
            torch.cuda.synchronize()
            ts.append(s_.elapsed_time(e_))
        return n * h.element_size() / (statistics.median(ts) * 1e-3) / 1e9

    h2d_gbs = rate(lambda: d.copy_(h, non_blocking=True))
    d2h_gbs = rate(lambda: o.copy_(d, non_blocking=True))
    bound_ms = max(h2d_bytes / h2d_gbs, d2h_bytes / d2h_gbs) / 1e6
    del d
    return {"h2d_gbs": round(h2d_gbs, 1), "d2h_gbs": round(d2h_gbs, 1), "bound_ms": round(bound_ms, 3),
            "note": "pinned-host copy rates measured alone on this box (256 MB each way); bound = the "
                    "slower direction's bytes / rate"}


DENSE_FLOP_PER_CLK = 148 * 8192  # B200: 148 SMs x 4096 bf16/fp16 FMA per clock each (dense)


def _config_inputs(W, cid, dev):
    import torch
    cfg = W.CONFIGS[cid]
    bs = W.batch_sizes_for(cfg)
    if cid == 1:
        a, b = [t.to(dev) for t in W.make_inputs(cfg, "cpu")]
    else:
        a, b = W.make_inputs(cfg, "cuda")
    torch.cuda.synchronize()
    return cfg, bs, a, b


def _config_entry(W, cid, dev, steps, warmup, peaks):
    """Kernel time, roofline and parity of one workload at N = 1."""
    import torch
    from gmm_b200 import hopper_gmm_fwd
    from gmm_b200.ep_bench import check_parity
    cfg, bs, a, b = _config_inputs(W, cid, dev)
    fn = lambda: hopper_gmm_fwd(a, b, bs, cfg.trans_b)  # noqa: E731
    for _ in range(max(3, warmup)):
        fn()
    alg = cfg.algorithmic_bytes(bs)
    flush = torch.empty(int(256e6), dtype=torch.uint8, device=dev) if alg <= 2 * 126e6 else None
    ms = _events_time(fn, steps, flush)
    mean = statistics.fmean(ms)
    out = fn()
    par = check_parity(out, a, bs.tolist(), lambda e: b[e], cfg.trans_b)
    tflops = cfg.flops() / (mean * 1e-3) / 1e12
    gbs = alg / (mean * 1e-3) / 1e9
    hbm_bound = cfg.dtype == torch.float32 or cid in (3, 4)
    entry = {"workload": f"cfg{cid}: {cfg.name}",
             "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[cfg.dtype],
             "ms_per_step": round(mean, 5), "p50_us_per_call": round(statistics.median(ms) * 1e3, 2),
             "tflops": round(tflops, 2), "gbs": round(gbs, 1),
             "tokens_per_s": round(cfg.tokens / (mean * 1e-3), 1),
             "roofline": {"bound": "hbm" if hbm_bound else "tensor",
                          "frac": round(gbs / peaks["hbm_gbs"] if hbm_bound else tflops / peaks["bf16_tflops"], 4),
                          "peak": peaks["hbm_gbs"] if hbm_bound else peaks["bf16_tflops"],
                          "unit": "GB/s" if hbm_bound else "TFLOP/s"},
             "l2": W.l2_note(cfg, bs), "steps": steps, "parity": par,
             "kernel_launches_per_step": 1}
    del a, b, out, flush
    torch.cuda.empty_cache()
    return entry


def run_single(args):
    import torch
    import gmm_b200  # noqa: F401  (loads the operator; fails loudly without it)
    from gmm_b200 import hopper_gmm_fwd
    from gmm_b200.ep_bench import check_parity
    W = _workloads()

    cid = args.config or 2
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = W.CONFIGS[cid]
    bs = W.batch_sizes_for(cfg)
    if args.max_experts:
        import dataclasses
        bs = bs[:args.max_experts].clone()
        cfg = dataclasses.replace(cfg, num_experts=len(bs), tokens=int(bs.sum()), top_k=1)
    if cid == 1:
        a, b = [t.to(dev) for t in W.make_inputs(cfg, "cpu")]
    else:
        a, b = W.make_inputs(cfg, "cuda")
    flops = cfg.flops()
    alg_bytes = cfg.algorithmic_bytes(bs)
    launches_per_step = 1  # one persistent kernel (fp32 included: TF32 split in shared memory)

    def step():
        return hopper_gmm_fwd(a, b, bs, cfg.trans_b)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    flush = torch.empty(int(256e6), dtype=torch.uint8, device=dev) if alg_bytes <= 2 * 126e6 else None

    peaks, peak_src = load_peaks()
    with ClockSampler(-1 if args.kernel_only else 0) as clk:
        kernel_ms = _events_time(step, args.steps, flush)
        # Sustained: back to back for >= args.sustain_s seconds right after the
        # timed region, so the clock sampler sees the kernel under load.
        sus = None
        if not args.kernel_only and args.sustain_s > 0:
            n = max(1, int(args.sustain_s * 1e3 / max(statistics.fmean(kernel_ms), 1e-3)))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            clk.mark()
            e0.record()
            for _ in range(n):
                if flush is not None:
                    flush.zero_()
                step()
            e1.record()
            torch.cuda.synchronize()
            clk.mark()
            sus = (n, e0.elapsed_time(e1) / n)
    step_ms = statistics.fmean(kernel_ms)
    value = flops / (step_ms * 1e-3) / 1e12
    if args.kernel_only:
        print(json.dumps({"config": f"cfg{cid}", "ms_per_step": step_ms, "value": value,
                          "unit": "TFLOP/s"}), flush=True)
        return
    p50_us = statistics.median(kernel_ms) * 1e3
    out = step()
    parity = check_parity(out, a, bs.tolist(), lambda e: b[e], cfg.trans_b)
    del out

    # ---------------- e2e: pinned host buffers, copies inside the timed region
    from gmm_b200 import hopper_gmm_fwd_host
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    d_h = torch.empty((cfg.rows, cfg.dim_out), dtype=cfg.dtype).pin_memory()

    def e2e_step():
        # per-expert-chunk H2D / GEMM / D2H pipeline (public host-operand API)
        hopper_gmm_fwd_host(a_h, b_h, bs, cfg.trans_b, out=d_h)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e_steps = max(1, min(args.e2e_steps, args.steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    es = a.element_size()
    h2d = (a.numel() + b.numel()) * es
    d2h = cfg.rows * cfg.dim_out * es
    pcie = _pcie_bound(b_h, d_h, h2d, d2h)

    if cfg.dtype == torch.float32 or cid in (3, 4):
        bound, achieved, peak, unit = "hbm", alg_bytes / (step_ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
    else:
        bound, achieved, peak, unit = "tensor", value, peaks["bf16_tflops"], "TFLOP/s"
    traffic = load_traffic(f"cfg{cid}")
    clocks = clk.summary()
    roof = {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": f"{peak_src} ({'burst' if unit == 'TFLOP/s' else 'copy'})",
            "algorithmic": {"flops": flops, "bytes": alg_bytes}}
    if unit == "TFLOP/s" and peaks.get("bf16_tflops_sustained"):
        roof["peak_sustained"] = peaks["bf16_tflops_sustained"]
        roof["frac_sustained"] = round(achieved / peaks["bf16_tflops_sustained"], 4)
    if sus is not None:
        n, sms = sus
        s_val = flops / (sms * 1e-3) / 1e12
        s_mhz = clk.summary(window=1).get("sm_mhz")
        roof["sustained_loop"] = {
            "steps": n, "ms_per_step": round(sms, 4), "achieved": round(s_val if unit == "TFLOP/s"
                                                                       else alg_bytes / (sms * 1e-3) / 1e9, 2),
            "sm_mhz_median": s_mhz, "power_w_max": clk.summary(window=1).get("power_w_max")}
        if s_mhz and unit == "TFLOP/s":
            per_ghz = s_val / (s_mhz / 1e3)
            roof["sustained_loop"]["tflops_per_ghz"] = round(per_ghz, 2)
            roof["sustained_loop"]["frac_at_clock"] = round(per_ghz / (DENSE_FLOP_PER_CLK / 1e3), 4)
            roof["sustained_loop"]["note"] = ("frac_at_clock = achieved / (148 SMs x 8192 dense FLOP/clk "
                                              "x median SM clock under load)")

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "p50_us_per_call": round(p50_us, 2),
        "tokens_per_s": round(cfg.tokens / (step_ms * 1e-3), 1),
        "higher_is_better": True, "scaling": "weak" if cid == 2 else "strong", "vs_baseline": None,
        "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[cfg.dtype],
        "data": "synthetic (seeded routing -> batch_sizes; A ~ N(0,1), B ~ N(0,1/dim))",
        "config": W.workload_config(cfg, 1, weak=cid == 2),
        "parity": parity,
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "pcie": pcie,
                "path": "gmm_b200.hopper_gmm_fwd_host: pinned host A,B -> device, GEMM, "
                        "D -> pinned host, pipelined per expert chunk on 3 streams"},
        "gpu_launches": args.steps * launches_per_step,
        "roofline": roof,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        a_c, b_c = a.cpu(), b.cpu()
        rate, desc, cores = cpu_rate(cfg, a_c, b_c, bs)
        line["cpu_baseline"] = {"value": round(rate, 4), "unit": "TFLOP/s", "cores": cores,
                                "kind": "port", "sample": desc}
        del a_c, b_c
    del a, b, a_h, b_h, d_h
    torch.cuda.empty_cache()
    if not args.no_configs and not args.max_experts:
        configs = {}
        for ocid in (1, 2, 3, 4, 5):
            if ocid != cid:
                configs[f"cfg{ocid}"] = _config_entry(W, ocid, dev, max(5, min(args.steps, 20)),
                                                      args.warmup, peaks)
        line["configs"] = configs
        # expert parallelism at N = 1 is the local grouped GEMM
        line["ep_configs"] = {
            k: {"workload": v["workload"], "dtype": v["dtype"], "scaling": "strong",
                "tokens": W.CONFIGS[int(k[3:])].tokens,
                "experts_per_rank": W.CONFIGS[int(k[3:])].num_experts,
                "ms_per_step": v["ms_per_step"], "tokens_per_s": v["tokens_per_s"],
                "tflops": v["tflops"], "n_gpus": 1, "parity": v["parity"],
                "load_imbalance": {"efficiency_ceiling": 1.0}}
            for k, v in configs.items() if k in ("cfg5", "cfg3")}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference's own CPU path on the host cores.  Imports torch, the
    workload generators (by file path) and ``oracle`` -- nothing that loads
    this repository's CUDA libraries."""
    import torch
    import oracle
    W = _workloads()

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    cid = args.config or 2
    cfg = W.CONFIGS[cid]
    bs = W.batch_sizes_for(cfg)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    # Bounded sample: every expert's full B, the first r rows of each expert,
    # r sized so one step takes about a second on this host.
    gen = torch.Generator().manual_seed(cfg.seed)
    shape = W.b_shape(cfg)
    b = torch.empty(*shape, dtype=cfg.dtype)
    for e in range(shape[0]):
        b[e] = (torch.randn(*shape[1:], generator=gen) / math.sqrt(cfg.dim)).to(cfg.dtype)
    bsl = [int(v) for v in bs]
    r = 4
    while True:
        sub = [min(m, r) for m in bsl]
        a = torch.randn(sum(sub), cfg.dim, generator=gen).to(cfg.dtype)
        bs_s = torch.tensor(sub, dtype=torch.int64)
        t0 = time.perf_counter()
        oracle.ref_gmm_port(a, b, bs_s, cfg.trans_b)
        dt = time.perf_counter() - t0
        if dt > 0.5 or r >= max(bsl):
            break
        r = min(max(bsl), int(r * max(2.0, 0.8 / max(dt, 1e-4))))
    for _ in range(max(1, args.warmup)):
        oracle.ref_gmm_port(a, b, bs_s, cfg.trans_b)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.ref_gmm_port(a, b, bs_s, cfg.trans_b)
        times.append(time.perf_counter() - t0)
        if sum(times) > 120:
            break
    step = statistics.fmean(times)
    rows = sum(sub)
    value = 2.0 * rows * cfg.dim * cfg.dim_out / step / 1e12
    desc = (f"reference ref_gmm restated (oracle.ref_gmm_port, torch CPU "
            f"{oracle.dtype_name(cfg.dtype)}) on the first {min(r, max(bsl))} rows of each expert "
            f"({rows} of {cfg.rows} rows, full B); {len(times)} timed steps")
    weak = cid == 2
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(step * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if weak else "strong",
        "vs_baseline": None, "dtype": oracle.dtype_name(cfg.dtype), "data": "synthetic",
        "config": W.workload_config(cfg, world, weak),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cores,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def run_cublas(args):
    """The configuration's grouped GEMM against cuBLAS on the same shapes, in one
    process: ``hopper_gmm_fwd``; ``torch.matmul`` per expert (the same work in E
    launches); ``torch.matmul`` of all rows with one expert's B (no grouping, no
    ragged tails: an upper bound for any grouped kernel).  Two passes of
    event-timed loops (the second runs hotter, nearer the power cap)."""
    import torch
    from gmm_b200 import hopper_gmm_fwd
    W = _workloads()
    cid = args.config or 2
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg, bs, a, b = _config_inputs(W, cid, dev)
    if args.max_experts:  # a smaller case of the same workload (the first experts and their rows)
        import dataclasses
        bs = bs[:args.max_experts].clone()
        rows = int(bs.sum())
        a, b = a[:rows], b[:args.max_experts]
        cfg = dataclasses.replace(cfg, num_experts=len(bs), tokens=rows, top_k=1)
    offs = [0]
    for m in bs.tolist():
        offs.append(offs[-1] + m)
    out = torch.empty(cfg.rows, cfg.dim_out, dtype=cfg.dtype, device=dev)
    bt = (lambda e: b[e].t()) if cfg.trans_b else (lambda e: b[e])  # noqa: E731

    def ours():
        hopper_gmm_fwd(a, b, bs, cfg.trans_b)

    def per_expert():
        for e in range(cfg.num_experts):
            if offs[e + 1] > offs[e]:
                torch.matmul(a[offs[e]:offs[e + 1]], bt(e), out=out[offs[e]:offs[e + 1]])

    def one_gemm():
        torch.matmul(a, bt(0), out=out)

    steps = max(5, min(args.steps, 50))
    res = {}
    variants = (("ours_grouped", ours), ("cublas_per_expert", per_expert),
                ("cublas_one_gemm_all_rows", one_gemm))
    if args.cublas_variant:  # one variant only (the command an ncu capture runs)
        variants = tuple(v for v in variants if v[0].startswith(args.cublas_variant))
    for rep in ((1,) if args.cublas_variant else (1, 2)):
        for name, fn in variants:
            for _ in range(max(3, args.warmup)):
                fn()
            ms = statistics.fmean(_events_time(fn, steps))
            res.setdefault(name, []).append({"pass": rep, "ms": round(ms, 4),
                                             "tflops": round(cfg.flops() / (ms * 1e-3) / 1e12, 1)})
    print(json.dumps({"workload": f"cfg{cid}: {cfg.name}", "steps": steps, "results": res}), flush=True)


def run_ffn(args):
    """MoE expert FFN forward: SwiGLU(A @ W1) @ W2 over the config's expert segments."""
    import torch
    import torch.nn.functional as F
    from gmm_b200 import hopper_gmm_fwd, moe_ffn
    from gmm_b200.configs import CONFIGS, batch_sizes_for
    cid = args.config or 2
    cfg = CONFIGS[cid]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bs = batch_sizes_for(cfg)
    E, dim = cfg.num_experts, cfg.dim
    inter = cfg.dim_out // 2 if cid == 3 else cfg.dim_out  # cfg3's dim_out is already gate+up
    g = torch.Generator(device=dev).manual_seed(cfg.seed)
    a = torch.randn(cfg.rows, dim, generator=g, device=dev).to(cfg.dtype)
    tb = cfg.trans_b
    w1 = torch.empty(*((E, 2 * inter, dim) if tb else (E, dim, 2 * inter)), dtype=cfg.dtype, device=dev)
    w2 = torch.empty(*((E, dim, inter) if tb else (E, inter, dim)), dtype=cfg.dtype, device=dev)
    for e in range(E):
        w1[e].copy_(torch.randn(w1.shape[1:], generator=g, device=dev) / math.sqrt(dim))
        w2[e].copy_(torch.randn(w2.shape[1:], generator=g, device=dev) / math.sqrt(inter))
    flops = 2.0 * cfg.rows * dim * 2 * inter + 2.0 * cfg.rows * inter * dim

    def fused():
        return moe_ffn(a, w1, w2, bs, tb, tb)

    def unfused():  # two plain grouped GEMMs with the activation as separate torch ops
        gu = hopper_gmm_fwd(a, w1, bs, tb)
        h = F.silu(gu[:, :inter]) * gu[:, inter:]
        return hopper_gmm_fwd(h, w2, bs, tb)

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    steps = max(1, min(args.steps, 50))
    ms = timed(fused, steps)
    ms_unfused = timed(unfused, steps)
    peaks, src = load_peaks()
    value = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "MoE expert FFN forward TFLOP/s (SwiGLU gate/up grouped GEMM + down grouped GEMM)",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16"}[cfg.dtype], "data": "synthetic",
        "config": {"workload": f"cfg{cid} routing, expert FFN", "experts": E, "dim": dim,
                   "inter": inter, "rows": cfg.rows, "trans_b": tb},
        "unfused_ms_per_step": round(ms_unfused, 4),
        "unfused_value": round(flops / (ms_unfused * 1e-3) / 1e12, 2),
        "roofline": {"bound": "tensor", "achieved": round(value, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(value / peaks["bf16_tflops"], 4),
                     "peak_source": f"{src} (burst)"},
        "gpu_launches": 2 * steps}), flush=True)


def run_layer(args):
    """Device-resident MoE layer on the config's shapes, eager and CUDA graph."""
    import torch
    from gmm_b200.configs import CONFIGS
    from gmm_b200.moe import moe_forward
    cid = args.config or 2
    cfg = CONFIGS[cid]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    E, dim, k, T = cfg.num_experts, cfg.dim, cfg.top_k, cfg.tokens
    inter = cfg.dim_out // 2 if cid == 3 else cfg.dim_out
    tb = cfg.trans_b
    g = torch.Generator(device=dev).manual_seed(cfg.seed)
    x = torch.randn(T, dim, generator=g, device=dev).to(cfg.dtype)
    logits = torch.randn(T, E, generator=g, device=dev)
    w1 = torch.empty(*((E, 2 * inter, dim) if tb else (E, dim, 2 * inter)), dtype=cfg.dtype, device=dev)
    w2 = torch.empty(*((E, dim, inter) if tb else (E, inter, dim)), dtype=cfg.dtype, device=dev)
    for e in range(E):
        w1[e].copy_(torch.randn(w1.shape[1:], generator=g, device=dev) / math.sqrt(dim))
        w2[e].copy_(torch.randn(w2.shape[1:], generator=g, device=dev) / math.sqrt(inter))
    flops = 2.0 * T * k * dim * 2 * inter + 2.0 * T * k * inter * dim

    def step():
        return moe_forward(x, logits, w1, w2, k, tb, tb)

    steps = max(1, min(args.steps, 50))
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1) / steps
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    graph_ms = e0.elapsed_time(e1) / steps
    del graph
    print(json.dumps({
        "metric": "device-resident MoE layer forward (route + permute + SwiGLU FFN + combine)",
        "value": round(flops / (graph_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(graph_ms, 4),
        "eager_ms_per_step": round(eager_ms, 4), "tokens_per_s": round(T / (graph_ms * 1e-3), 1),
        "higher_is_better": True, "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16"}[cfg.dtype],
        "data": "synthetic (router logits ~ N(0,1))",
        "config": {"workload": f"cfg{cid} shapes, MoE layer", "tokens": T, "top_k": k, "experts": E,
                   "dim": dim, "inter": inter, "trans_b": tb},
        "gpu_launches": 7 * steps}), flush=True)


def main():
    args = parse()
    if args.layer and args.impl == "ours":
        run_layer(args)
        return
    if args.ffn and args.impl == "ours":
        run_ffn(args)
        return
    if args.cublas and args.impl == "ours":
        run_cublas(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        from gmm_b200 import ep_bench
        ep_bench.run(args, METRIC, load_peaks, ClockSampler)
        return
    run_single(args)


if __name__ == "__main__":
    main()
