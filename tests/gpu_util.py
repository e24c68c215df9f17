"""Shared helpers for the GPU parity tests (checker side only)."""

from __future__ import annotations

import contextlib
import json
import os

import numpy as np
import torch

import oracle

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden():
    gold = np.load(os.path.join(GOLDEN_DIR, "ref_gmm_golden.npz"))
    cases = json.loads(bytes(gold["__meta__"]).decode())
    return gold, cases


def golden_values(gold, case):
    raw = gold[case["name"] + "__out"]
    if case["dtype"] == "fp32":
        return raw.view(np.float32)
    if case["dtype"] == "bf16":
        return (raw.astype(np.uint32) << 16).view(np.float32)
    return raw.view(np.float16).astype(np.float32)


def check_rows(got_rows: torch.Tensor, a_rows, b_sub, bs_sub, trans_b, dtype_name, what=""):
    """Compare device output rows with the oracle run on the same rows/experts."""
    want = oracle.round_to(oracle.gmm_oracle_np(a_rows, b_sub, bs_sub, trans_b), dtype_name)
    got = got_rows.float().cpu().numpy()
    tol = oracle.TOLERANCE[dtype_name]
    ok, nbad, maxerr = oracle.allclose_report(got, want, tol)
    assert ok, f"{what}: {nbad}/{got.size} elements outside rtol=atol={tol}; max abs err {maxerr:.3e}"
    return maxerr


def sampled_subproblem(bs, rows_per_expert=4, max_experts=8, seed=0):
    """Pick rows from a few non-empty experts; returns (row_index, experts, sub_batch_sizes)."""
    g = np.random.default_rng(seed)
    bs = [int(v) for v in bs]
    off = np.concatenate([[0], np.cumsum(bs)])
    nz = [e for e, m in enumerate(bs) if m > 0]
    pick = sorted(g.choice(nz, size=min(max_experts, len(nz)), replace=False).tolist())
    # always include the first, the last and the largest non-empty expert
    for e in (nz[0], nz[-1], int(np.argmax(bs))):
        if e not in pick:
            pick.append(e)
    pick = sorted(pick)
    rows, sub_bs = [], []
    for e in pick:
        m = bs[e]
        cand = {int(off[e]), int(off[e] + m - 1)}
        if m > 2:
            cand.update(int(v) for v in g.integers(off[e], off[e] + m, size=rows_per_expert))
        r = sorted(cand)
        rows.extend(r)
        sub_bs.append(len(r))
    return np.asarray(rows, dtype=np.int64), pick, sub_bs


@contextlib.contextmanager
def forced_tile(kind):
    """Force one kernel family ("auto", "128", "256", "swap") for the calls made
    inside the block (``gmm_sm100_set_tile_kind``), then restore the previous one."""
    from gmm_b200 import capi
    prev = capi.set_tile_kind(kind)
    try:
        yield kind
    finally:
        capi.set_tile_kind(prev)
