"""The CPU oracle pinned against the reference's own ``ref_gmm`` outputs."""

import json
import os

import numpy as np
import pytest
import torch

import oracle
from cases import all_cases, make_case_inputs

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_gmm_golden.npz"))
CASES = json.loads(bytes(GOLD["__meta__"]).decode())


def _golden_values(case):
    raw = GOLD[case["name"] + "__out"]
    if case["dtype"] == "fp32":
        return raw.view(np.float32)
    if case["dtype"] == "bf16":
        return (raw.astype(np.uint32) << 16).view(np.float32)
    return raw.view(np.float16).astype(np.float32)


def test_golden_covers_every_case():
    assert [c["name"] for c in CASES] == [c["name"] for c in all_cases()]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracles_match_reference_ref_gmm(case):
    a, b, bs = make_case_inputs(case)
    rows = GOLD[case["name"] + "__rows"]
    want = _golden_values(case)
    tol = oracle.TOLERANCE[case["dtype"]]
    c64 = oracle.gmm_oracle_c(a, b, bs, case["trans_b"])
    n32 = oracle.gmm_oracle_np(a, b, bs, case["trans_b"])
    for name, acc in (("c_f64", c64), ("np_f32", n32)):
        got = oracle.round_to(acc[rows], case["dtype"])
        ok, nbad, maxerr = oracle.allclose_report(got, want, tol)
        assert ok, f"{name}: {nbad} elements outside tol {tol}, max err {maxerr}"
        if case["dtype"] != "fp32":
            # Rounding (nearly) the same fp32 accumulator to 16 bits: almost
            # every element is bit-identical to the reference's.
            same = np.mean(got == want)
            assert same > 0.97, f"{name}: only {same:.3f} of elements bit-identical"
        else:
            # fp32 differs only by summation order.
            scale = np.abs(want).max() + 1e-30
            assert maxerr <= 1e-5 * scale, f"{name}: fp32 max err {maxerr} vs scale {scale}"


def test_ref_gmm_port_matches_reference():
    """The literal torch-CPU port reproduces the reference's own outputs.  It
    runs the same bf16 matmuls as the reference's ref_gmm, so on the CPU the
    golden vectors were made on it is bit-identical; another CPU's BLAS may
    order the fp32 accumulation differently and round a rare element to the
    neighbouring bf16 value (seen: 1 element in 6,560 on an AMD EPYC host)."""
    case = next(c for c in CASES if c["name"] == "ragged_bf16_NT")
    a, b, bs = make_case_inputs(case)
    rows = GOLD[case["name"] + "__rows"]
    got = oracle.ref_gmm_port(a, b, bs, True)[rows].float().numpy()
    want = _golden_values(case)
    assert np.mean(got == want) > 0.999
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)  # bf16 spacing at |want|
    assert np.all(np.abs(got - want) <= ulp)


def test_oracle_rejects_bad_sum():
    a = torch.zeros(10, 8)
    b = torch.zeros(2, 8, 4)
    with pytest.raises(ValueError, match="Sum of batch_sizes"):
        oracle.gmm_oracle_c(a, b, torch.tensor([3, 4]))
    with pytest.raises(ValueError, match="Sum of batch_sizes"):
        oracle.gmm_oracle_np(a, b, torch.tensor([3, 4]))


def test_round_bf16_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], dtype=np.float32)
    want = torch.tensor(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(oracle.round_bf16(x), want)
    r = np.random.default_rng(0).standard_normal(100000).astype(np.float32)
    np.testing.assert_array_equal(oracle.round_bf16(r), torch.tensor(r).to(torch.bfloat16).float().numpy())


def test_config_batch_sizes_are_frozen():
    from gmm_b200.configs import CONFIGS, batch_sizes_for
    with open(os.path.join(os.path.dirname(__file__), "golden", "config_batch_sizes.json")) as f:
        frozen = json.load(f)
    for cid, cfg in CONFIGS.items():
        bs = batch_sizes_for(cfg)
        assert bs.tolist() == frozen[str(cid)]
        assert int(bs.sum()) == cfg.rows
    assert min(frozen["3"]) == 0 and sum(v > 0 for v in frozen["3"]) == 240
    assert max(frozen["4"]) <= 16


def test_routing_and_permutation_oracles_agree_with_loops():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((50, 12)).astype(np.float32)
    logits[3, 5] = logits[3, 7] = 9.0  # a tie: the lower index wins
    ids, w = oracle.topk_oracle(logits, 3, renormalize=True)
    assert ids[3, 0] == 5 and ids[3, 1] == 7
    for t in range(50):
        want = sorted(range(12), key=lambda e: (-logits[t, e], e))[:3]
        assert list(ids[t]) == want
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-12)
    bs, dst, src = oracle.permute_oracle(ids, 12)
    rows = [(e, t, j) for t in range(50) for j in range(3) for e in [ids[t, j]]]
    rows.sort(key=lambda r: r[0])  # stable: (token, slot) order kept within an expert
    for pos, (e, t, j) in enumerate(rows):
        assert dst[t, j] == pos and src[pos] == t
    assert bs.sum() == 150 and list(bs) == [sum(1 for r in rows if r[0] == e) for e in range(12)]
    y = rng.standard_normal((150, 4)).astype(np.float32)
    out = oracle.unpermute_oracle(y, dst, w)
    np.testing.assert_allclose(out[7], sum(w[7, j] * y[dst[7, j]].astype(np.float64) for j in range(3)),
                               rtol=1e-6)
