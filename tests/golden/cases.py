"""Golden-case recipes shared by ``make_golden.py`` and the tests.

A case is fully determined by its fields: inputs are re-drawn from a CPU
``torch.Generator`` seeded with ``seed`` (A first, then B), optionally scaled
by ``1/sqrt(dim*dim_out)`` as the reference's correctness test does
(reference ``tests/test_forward.py:30-37``), then cast to the case dtype.
"""

from __future__ import annotations

import math

import torch

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _case(name, bs, dim, dim_out, dtype, trans_b, seed, scaled):
    return dict(name=name, bs=list(bs), dim=dim, dim_out=dim_out, dtype=dtype,
                trans_b=bool(trans_b), seed=seed, scaled=bool(scaled))


def all_cases():
    cases = []
    # The reference's own shape table (tests/test_forward.py:57-62) and dtype /
    # layout matrix (tests/test_forward.py:67-77), inputs scaled as it does.
    for E, per, dim, dim_out in [(4, 128, 128, 256), (8, 64, 256, 512), (16, 128, 128, 128)]:
        for dt in ("fp32", "bf16", "fp16"):
            for tb in ((False,) if dt == "fp32" else (False, True)):
                cases.append(_case(f"ref_{E}x{per}_{dim}x{dim_out}_{dt}_{'NT' if tb else 'NN'}",
                                   [per] * E, dim, dim_out, dt, tb, 0, True))
    # Unscaled N(0,1) inputs: the tolerance-critical distribution of the
    # five workload configurations.
    for dt in ("fp32", "bf16", "fp16"):
        cases.append(_case(f"unit_8x64_256x512_{dt}_NN", [64] * 8, 256, 512, dt, False, 5, False))
    cases.append(_case("unit_8x64_256x512_fp32_NT", [64] * 8, 256, 512, "fp32", True, 6, False))
    # The reference's zero-size-expert case (tests/test_forward.py:79-87),
    # here with its values pinned too.
    cases.append(_case("zero_experts_fp16_NN", [0, 32, 0, 64, 0], 128, 256, "fp16", False, 7, False))
    # Ragged segments: 1-row experts, tile tails in M, N and K, empty experts.
    for dt in ("bf16", "fp16", "fp32"):
        for tb in (False, True):
            cases.append(_case(f"ragged_{dt}_{'NT' if tb else 'NN'}", [1, 0, 130, 7, 255, 0, 64, 3],
                               192, 328, dt, tb, 8, False))
    # cfg1 of the workload table: E=8, 128->256, bs=[64]*8, N(0,1) fp32.
    cases.append(_case("cfg1_fp32_NN", [64] * 8, 128, 256, "fp32", False, 0, False))
    return cases


def make_case_inputs(case):
    """Re-draw a case's A ``[T, dim]`` and B (CPU tensors, case dtype)."""
    bs = case["bs"]
    E, dim, dim_out = len(bs), case["dim"], case["dim_out"]
    T = sum(bs)
    gen = torch.Generator().manual_seed(case["seed"])
    a = torch.randn(T, dim, generator=gen, dtype=torch.float32)
    shape = (E, dim_out, dim) if case["trans_b"] else (E, dim, dim_out)
    b = torch.randn(*shape, generator=gen, dtype=torch.float32)
    if case["scaled"]:
        s = 1.0 / math.sqrt(dim * dim_out)
        a, b = a * s, b * s
    dt = DTYPES[case["dtype"]]
    return a.to(dt), b.to(dt), torch.tensor(bs, dtype=torch.int64)


def sample_rows(bs, seed=1234, per_expert=4):
    """Row indices checked against the golden output: first/last + random rows of each expert."""
    g = torch.Generator().manual_seed(seed)
    rows, start = [], 0
    for m in bs:
        if m > 0:
            pick = {start, start + m - 1}
            if m > 2:
                extra = torch.randint(start + 1, start + m - 1, (per_expert - 2,), generator=g)
                pick.update(int(v) for v in extra)
            rows.extend(sorted(pick))
        start += m
    return rows
