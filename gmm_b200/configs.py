"""Seeded synthetic workloads for the five grouped-GEMM configurations.

The reference publishes no dataset or benchmark inputs; its own benchmark
draws synthetic tensors (reference ``tests/bench_moe_forward.py:105-117``).
These generators stand in for the five configurations the project is
measured on.  Every configuration is a grouped GEMM ``D[rows_g] = A[rows_g] @
B[g]`` (``B[g]^T`` when ``trans_b``) whose row segments come from a routing
draw: ``batch_sizes = bincount(topk_expert_ids, minlength=E)``.

Draw order for one configuration: routing on a CPU ``torch.Generator`` seeded
with the configuration's seed, then A, then B.  Routing (and therefore
``batch_sizes``) is always drawn on the CPU and is frozen as a fixture under
``tests/golden``.  A and B are drawn on the CPU with the same generator for
configurations small enough for that (cfg1), and on the device with a CUDA
generator seeded the same way for the large ones, where a CPU draw of B
(up to 15 GB) would take minutes; the parity checks copy the device-drawn
inputs back so the oracle always sees exactly the bytes the kernel saw.
"""

from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import torch


@dataclasses.dataclass(frozen=True)
class GmmConfig:
    """One grouped-GEMM workload."""

    cid: int
    name: str
    num_experts: int
    dim: int
    dim_out: int
    tokens: int          # pre-top-k tokens (the EP tokens/s numerator)
    top_k: int
    dtype: torch.dtype
    trans_b: bool
    seed: int
    routing: str         # "uniform", "softmax_topk", "zipf", "dirichlet"
    b_scale: str         # "unit" -> N(0,1); "inv_sqrt_dim" -> N(0, 1/dim)

    @property
    def rows(self) -> int:
        return self.tokens * self.top_k

    def flops(self) -> float:
        return 2.0 * self.rows * self.dim * self.dim_out

    def elem_bytes(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    def algorithmic_bytes(self, batch_sizes) -> float:
        """A + (nonzero experts' B) + D, each read or written once."""
        nz = int((torch.as_tensor(batch_sizes) > 0).sum())
        e = self.elem_bytes()
        return float((self.rows * self.dim + nz * self.dim * self.dim_out
                      + self.rows * self.dim_out) * e)


CONFIGS = {
    1: GmmConfig(1, "fp32 NN tiny (reference CPU case)", 8, 128, 256, 512, 1,
                 torch.float32, False, 0, "uniform", "unit"),
    2: GmmConfig(2, "bf16 NN Mixtral-8x7B up-proj prefill", 8, 4096, 14336, 8192, 2,
                 torch.bfloat16, False, 1, "softmax_topk", "inv_sqrt_dim"),
    3: GmmConfig(3, "fp16 NT DeepSeek-V3 fine-grained experts", 256, 7168, 4096, 4096, 8,
                 torch.float16, True, 2, "zipf", "inv_sqrt_dim"),
    4: GmmConfig(4, "bf16 NN decode small-M down-proj", 128, 768, 2048, 128, 8,
                 torch.bfloat16, False, 3, "softmax_topk", "inv_sqrt_dim"),
    5: GmmConfig(5, "bf16 NN Mixtral-8x22B EP prefill", 8, 6144, 16384, 32768, 2,
                 torch.bfloat16, False, 4, "dirichlet", "inv_sqrt_dim"),
}


def route(cfg: GmmConfig, gen: torch.Generator, tokens: Optional[int] = None,
          sample_gen: Optional[torch.Generator] = None) -> torch.Tensor:
    """Top-k expert ids ``[tokens, top_k]`` (int64, CPU) for ``cfg``'s routing law.

    ``sample_gen`` (zipf / dirichlet laws): draw the tokens' experts from it
    instead of ``gen``, keeping the expert popularity ``gen`` fixes -- another
    batch of the same model, as a load balancer's history would see it."""
    n_tok = cfg.tokens if tokens is None else tokens
    sg = gen if sample_gen is None else sample_gen
    E, k = cfg.num_experts, cfg.top_k
    if cfg.routing == "uniform":
        # bs = [tokens/E]*E exactly: token t goes to expert t // (tokens/E).
        per = n_tok // E
        return (torch.arange(n_tok, dtype=torch.int64) // per).clamp_max(E - 1).view(n_tok, 1)
    if cfg.routing == "softmax_topk":
        logits = torch.randn(n_tok, E, generator=gen)
        return torch.topk(torch.softmax(logits, dim=-1), k, dim=-1).indices
    if cfg.routing == "zipf":
        # Zipf(s=1.1) weights r^-1.1 handed to experts in a random order; the
        # 16 lightest experts get weight 0 so the draw has zero-row experts.
        perm = torch.randperm(E, generator=gen)
        w = torch.empty(E, dtype=torch.float64)
        w[perm] = torch.arange(1, E + 1, dtype=torch.float64).pow(-1.1)
        w[perm[E - 16:]] = 0.0
        return torch.multinomial(w.expand(n_tok, E), k, replacement=False, generator=sg)
    if cfg.routing == "dirichlet":
        conc = torch.full((E,), 5.0, dtype=torch.float64)
        # Dirichlet(alpha) = normalised Gamma(alpha, 1) draws.
        g = torch._standard_gamma(conc.unsqueeze(0).expand(1, E).contiguous(), generator=gen)[0]
        p = g / g.sum()
        return torch.multinomial(p.expand(n_tok, E), k, replacement=False, generator=sg)
    raise ValueError(cfg.routing)


def batch_sizes_for(cfg: GmmConfig) -> torch.Tensor:
    """Frozen-recipe ``batch_sizes`` (CPU int64) for a configuration."""
    gen = torch.Generator().manual_seed(cfg.seed)
    ids = route(cfg, gen)
    return torch.bincount(ids.flatten(), minlength=cfg.num_experts).to(torch.int64)


def b_shape(cfg: GmmConfig, num_experts: Optional[int] = None) -> List[int]:
    e = cfg.num_experts if num_experts is None else num_experts
    return [e, cfg.dim_out, cfg.dim] if cfg.trans_b else [e, cfg.dim, cfg.dim_out]


def make_inputs(cfg: GmmConfig, device: str = "cpu", rows: Optional[int] = None,
                num_experts: Optional[int] = None, seed_offset: int = 0):
    """Draw A ``[rows, dim]`` and B (N(0,1) or N(0,1/dim)) in ``cfg.dtype``.

    On the CPU the generator follows the routing draw (same generator); on a
    CUDA device a CUDA generator seeded with ``cfg.seed + seed_offset`` is
    used.  ``rows``/``num_experts`` override the full sizes (EP shards).
    """
    n_rows = cfg.rows if rows is None else rows
    dev = torch.device(device)
    if dev.type == "cpu":
        gen = torch.Generator().manual_seed(cfg.seed + seed_offset)
        route(cfg, gen)  # advance past the routing draw
    else:
        gen = torch.Generator(device=dev).manual_seed(cfg.seed + seed_offset)
    a = torch.randn(n_rows, cfg.dim, generator=gen, device=dev, dtype=torch.float32).to(cfg.dtype)
    shape = b_shape(cfg, num_experts)
    if dev.type == "cpu":
        b = torch.randn(*shape, generator=gen, dtype=torch.float32)
        if cfg.b_scale == "inv_sqrt_dim":
            b = b / math.sqrt(cfg.dim)
        b = b.to(cfg.dtype)
    else:
        # Draw in the target dtype directly (chunked per expert) to bound the
        # fp32 temporary: cfg3's B is 7.5e9 elements.
        b = torch.empty(*shape, dtype=cfg.dtype, device=dev)
        s = 1.0 / math.sqrt(cfg.dim) if cfg.b_scale == "inv_sqrt_dim" else 1.0
        for e in range(shape[0]):
            t = torch.randn(*shape[1:], generator=gen, device=dev, dtype=torch.float32)
            b[e].copy_(t.mul_(s))
    return a, b


TOLERANCE = {torch.bfloat16: 1.6e-2, torch.float16: 2e-3, torch.float32: 5e-3}  # rtol = atol


def l2_note(cfg: GmmConfig, batch_sizes) -> str:
    """How a timed loop over this workload avoids L2 reuse between steps."""
    return ("inputs larger than L2 (126 MB)" if cfg.algorithmic_bytes(batch_sizes) > 2 * 126e6
            else "L2 flushed between steps (256 MB write)")


def workload_config(cfg: GmmConfig, world: int = 1, weak: bool = False) -> dict:
    """The ``config`` object of a bench line: the workload alone, identical in
    every arm that measures it (no arm- or implementation-specific keys)."""
    tokens = cfg.tokens * world if weak else cfg.tokens
    return {"workload": f"cfg{cfg.cid}: {cfg.name}", "experts": cfg.num_experts, "dim": cfg.dim,
            "dim_out": cfg.dim_out, "tokens": tokens, "top_k": cfg.top_k,
            "rows": tokens * cfg.top_k, "trans_b": cfg.trans_b, "parallelism": f"ep{world}",
            "scaling": "weak" if weak else "strong",
            "l2": l2_note(cfg, batch_sizes_for(cfg))}


def history_loads(cfg: GmmConfig, tokens: Optional[int] = None) -> torch.Tensor:
    """Rows per expert of another batch with the same expert popularity (a
    different token sample): what a load balancer would have measured before
    placing the experts.  ``[num_experts]`` int64."""
    gen = torch.Generator().manual_seed(cfg.seed)
    sample = torch.Generator().manual_seed(cfg.seed + 7777)
    ids = route(cfg, gen, tokens=tokens, sample_gen=sample)
    return torch.bincount(ids.flatten(), minlength=cfg.num_experts).to(torch.int64)
