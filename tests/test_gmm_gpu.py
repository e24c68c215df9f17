"""Parity of the sm_100a grouped-GEMM kernels with the reference's math.

The reference's own correctness test (reference tests/test_forward.py) is the
model: the same shape table, dtypes and layouts, compared with per-expert
fp32-accumulated matmuls -- here the pinned CPU oracle and the reference's
own ``ref_gmm`` golden outputs.  Tolerances (rtol = atol): bf16 1.6e-2,
fp16 2e-3, fp32 5e-3; row placement is checked bit-exactly.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from cases import make_case_inputs
from gpu_util import check_rows, forced_tile, golden, golden_values, sampled_subproblem

pytestmark = pytest.mark.gpu

GOLD, CASES = golden()


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gmm_b200  # noqa: F401  (loads the op)
    torch.cuda.set_device(0)
    yield
    from gmm_b200 import capi
    assert capi.device_error(clear=True) == 0, "a kernel recorded a device-side timeout"


@pytest.fixture(params=["128", "256", "swap"])
def tile(request):
    """Run a test with one kernel forced: single-CTA 128-row tiles, CTA-pair
    256-row tiles, or swap-AB tiles (16-bit problems only; fp32 keeps its own
    kernel)."""
    with forced_tile(request.param):
        yield request.param


def _fwd(a, b, bs, trans_b):
    from gmm_b200 import hopper_gmm_fwd
    return hopper_gmm_fwd(a, b, bs, trans_b=trans_b)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden_case(case, tile):
    a, b, bs = make_case_inputs(case)
    out = _fwd(a.cuda(), b.cuda(), bs, case["trans_b"])
    torch.cuda.synchronize()
    assert out.shape == (a.shape[0], b.shape[1] if case["trans_b"] else b.shape[2])
    assert out.dtype == a.dtype
    tol = oracle.TOLERANCE[case["dtype"]]
    # 1) against the reference's own ref_gmm outputs (sampled rows)
    rows = GOLD[case["name"] + "__rows"]
    got = out.float().cpu().numpy()
    ok, nbad, err = oracle.allclose_report(got[rows], golden_values(GOLD, case), tol)
    assert ok, f"vs reference ref_gmm: {nbad} bad, max err {err:.3e}"
    # 2) against the oracle on every row
    want = oracle.round_to(oracle.gmm_oracle_c(a, b, bs, case["trans_b"]), case["dtype"])
    ok, nbad, err = oracle.allclose_report(got, want, tol)
    assert ok, f"vs oracle: {nbad} bad, max err {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("trans_b", [False, True])
def test_placement_is_exact(dtype, trans_b, tile):
    """B[e] = (e+1) * I: every output row must be exactly (e+1) * its input row."""
    bs = [5, 0, 300, 1, 129, 0, 128, 17, 0, 64]
    dim = 256
    T = sum(bs)
    g = torch.Generator().manual_seed(3)
    a = torch.randint(-8, 9, (T, dim), generator=g).to(dtype)
    eye = torch.eye(dim)
    b = torch.stack([(e + 1) * eye for e in range(len(bs))]).to(dtype)
    out = _fwd(a.cuda(), b.cuda(), torch.tensor(bs), trans_b).cpu()
    scale = torch.repeat_interleave(torch.arange(1, len(bs) + 1, dtype=torch.float32), torch.tensor(bs))
    want = (a.float() * scale[:, None]).to(dtype)
    assert torch.equal(out, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_canary_rows_untouched(dtype, tile):
    """Drive the C ABI into the middle of a NaN-filled buffer: nothing outside D is written."""
    from gmm_b200 import capi
    bs = [3, 0, 200, 0, 70]
    T, dim, dim_out, pad = sum(bs), 136, 264, 37
    a = torch.randn(T, dim, device="cuda").to(dtype)
    b = torch.randn(len(bs), dim, dim_out, device="cuda").to(dtype)
    big = torch.full((T + 2 * pad, dim_out), float("nan"), device="cuda", dtype=dtype)
    d = big[pad:pad + T]
    capi.forward(a, b, bs, d, trans_b=False)
    torch.cuda.synchronize()
    assert torch.isnan(big[:pad]).all() and torch.isnan(big[pad + T:]).all()
    assert not torch.isnan(d).any()
    check_rows(d, a.cpu(), b.cpu(), bs, False, oracle.dtype_name(dtype), "canary")


def test_more_groups_than_inline_table():
    """1500 non-empty experts: the tile table goes through the device workspace."""
    E = 1500
    g = torch.Generator().manual_seed(11)
    bs = torch.randint(1, 5, (E,), generator=g)
    bs[::7] = 0
    T, dim, dim_out = int(bs.sum()), 64, 128
    a = torch.randn(T, dim, generator=g).to(torch.bfloat16)
    b = (torch.randn(E, dim_out, dim, generator=g) / 8).to(torch.bfloat16)
    out = _fwd(a.cuda(), b.cuda(), bs, True)
    want = oracle.round_to(oracle.gmm_oracle_np(a, b, bs, True), "bf16")
    ok, nbad, err = oracle.allclose_report(out.float().cpu().numpy(), want, 1.6e-2)
    assert ok, (nbad, err)


@pytest.mark.parametrize("groups", [127, 128, 129, 1024, 1025])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_table_size_boundaries(groups, dtype, tile):
    """Non-empty expert counts either side of the two inline-table sizes (128
    groups travel in the small parameter block, up to 1024 in the full one,
    more in the workspace): every kernel family gets its whole table."""
    g = torch.Generator().manual_seed(groups)
    bs = torch.randint(1, 4, (groups + groups // 9,), generator=g)
    bs[torch.randperm(bs.numel(), generator=g)[:groups // 9]] = 0  # empty experts between the others
    assert int((bs > 0).sum()) == groups
    T, dim, dim_out = int(bs.sum()), 64, 96
    a = torch.randn(T, dim, generator=g).to(dtype)
    b = (torch.randn(bs.numel(), dim, dim_out, generator=g) / 8).to(dtype)
    out = _fwd(a.cuda(), b.cuda(), bs, False)
    name = oracle.dtype_name(dtype)
    want = oracle.gmm_oracle_np(a, b, bs, False)
    if dtype != torch.float32:
        want = oracle.round_to(want, name)
    ok, nbad, err = oracle.allclose_report(out.float().cpu().numpy(), want, oracle.TOLERANCE[name])
    assert ok, (groups, nbad, err)


def test_degenerate_sizes(tile):
    dev = "cuda"
    # all experts empty -> T = 0
    out = _fwd(torch.empty(0, 64, device=dev, dtype=torch.bfloat16),
               torch.randn(3, 64, 32, device=dev).bfloat16(), torch.zeros(3, dtype=torch.int64), False)
    assert out.shape == (0, 32)
    # dim = 0 -> zeros
    out = _fwd(torch.empty(5, 0, device=dev, dtype=torch.float16),
               torch.empty(2, 0, 16, device=dev, dtype=torch.float16), torch.tensor([2, 3]), False)
    assert out.shape == (5, 16) and (out == 0).all()
    # one row, one expert, tiny dims (M, N and K tails all at once)
    a = torch.randn(1, 8, device=dev).bfloat16()
    b = torch.randn(1, 8, 8, device=dev).bfloat16()
    out = _fwd(a, b, torch.tensor([1]), False)
    check_rows(out, a.cpu(), b.cpu(), [1], False, "bf16", "1x8x8")


def test_reference_error_messages():
    dev = "cuda"
    a = torch.randn(10, 64, device=dev).bfloat16()
    b = torch.randn(2, 64, 32, device=dev).bfloat16()
    with pytest.raises(RuntimeError, match=r"Sum of batch_sizes \(9\) must equal A.size\(0\) \(10\)"):
        _fwd(a, b, torch.tensor([4, 5]), False)
    with pytest.raises(RuntimeError, match="batch_sizes must be a 1D CPU int64 tensor"):
        _fwd(a, b, torch.tensor([4, 6], device=dev), False)
    with pytest.raises(RuntimeError, match="A and B must have the same dtype"):
        _fwd(a, b.half(), torch.tensor([4, 6]), False)
    with pytest.raises(RuntimeError, match=r"B.size\(0\) must equal num_experts"):
        _fwd(a, b, torch.tensor([4, 3, 3]), False)
    with pytest.raises(RuntimeError, match=r"B.size\(1\) must equal A.size\(1\) \(dim\)"):
        _fwd(a, torch.randn(2, 32, 64, device=dev).bfloat16(), torch.tensor([4, 6]), False)
    with pytest.raises(RuntimeError, match="Unsupported dtype"):
        _fwd(a.double(), b.double(), torch.tensor([4, 6]), False)
    with pytest.raises(RuntimeError, match="A must be a contiguous CUDA tensor"):
        _fwd(torch.randn(64, 10, device=dev).bfloat16().t(), b, torch.tensor([4, 6]), False)


def test_deterministic_and_stream_ordered(tile):
    a = torch.randn(3000, 512, device="cuda").bfloat16()
    b = (torch.randn(4, 512, 768, device="cuda") / 16).bfloat16()
    bs = torch.tensor([1000, 0, 1500, 500])
    ref = _fwd(a, b, bs, False)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        outs = [_fwd(a, b, bs, False) for _ in range(3)]
    s.synchronize()
    for o in outs:
        assert torch.equal(o, ref)


# ------------------------------------------------------------ workload configs
def _config_inputs(cid):
    from gmm_b200.configs import CONFIGS, batch_sizes_for, make_inputs
    cfg = CONFIGS[cid]
    bs = batch_sizes_for(cfg)
    if cid == 1:
        a, b = make_inputs(cfg, "cpu")
        a, b = a.cuda(), b.cuda()
    else:
        a, b = make_inputs(cfg, "cuda")
    return cfg, bs, a, b


def _column_slice(dim_out, bn=256):
    """Output columns checked on every row: 64 straddling each of the first two
    n-tile boundaries and the two half-tile boundaries next to them (a CTA
    pair splits a tile's columns in halves), plus the last 64 (the ragged
    last n-tile)."""
    cols = set()
    for edge in (bn // 2, bn, bn + bn // 2, 2 * bn):
        if edge < dim_out:
            cols.update(range(edge - 32, min(edge + 32, dim_out)))
    cols.update(range(max(0, dim_out - 64), dim_out))
    return np.asarray(sorted(cols), dtype=np.int64)


@pytest.mark.parametrize("cid", [1, 2, 3, 4, 5])
def test_config_parity(cid, tile):
    """Every row of every configuration against the oracle: cfg1 and cfg4 on
    every column, cfg2/3/5 on a column slice around the n-tile boundaries
    (the oracle then costs seconds on the CPU), plus sampled rows of every
    column on the largest, first and last experts."""
    if tile == "swap" and cid == 1:
        pytest.skip("fp32 has no swap-AB kernel")
    cfg, bs, a, b = _config_inputs(cid)
    out = _fwd(a, b, bs, cfg.trans_b)
    torch.cuda.synchronize()
    assert out.shape == (cfg.rows, cfg.dim_out)
    assert torch.isfinite(out.float()).all()
    name = oracle.dtype_name(cfg.dtype)
    tol = oracle.TOLERANCE[name]
    if cid in (1, 4):  # small enough for the oracle on every element
        cols = np.arange(cfg.dim_out)
        b_sub = b.cpu()
    else:
        cols = _column_slice(cfg.dim_out)
        idx = torch.as_tensor(cols, device="cuda")
        b_sub = (b.index_select(1, idx) if cfg.trans_b else b.index_select(2, idx)).cpu()
    want = oracle.round_to(oracle.gmm_oracle_np(a.cpu(), b_sub, bs, cfg.trans_b), name)
    got = out[:, torch.as_tensor(cols, device="cuda")].float().cpu().numpy()
    ok, nbad, err = oracle.allclose_report(got, want, tol)
    assert ok, f"cfg{cid}: {nbad} of {got.size} elements (all {cfg.rows} rows x {len(cols)} cols) off, max {err:.3e}"
    rows, experts, sub_bs = sampled_subproblem(bs.tolist())
    ridx = torch.as_tensor(rows, device="cuda")
    check_rows(out[ridx], a[ridx].cpu(), b[experts].cpu(), sub_bs, cfg.trans_b, name,
               f"cfg{cid} sampled rows, every column")
    del a, b, out
    torch.cuda.empty_cache()


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_config_placement_is_exact(cid, tile):
    """Row placement on the configuration's own ragged expert table (cfg2's
    1-row tail, cfg3's 13..3555-row experts and zero-row experts, cfg5's
    Dirichlet loads): with B[e] = c_e * I and small integer A every output row
    must be exactly c_e times its input row."""
    from gmm_b200.configs import CONFIGS, batch_sizes_for
    cfg = CONFIGS[cid]
    bs = batch_sizes_for(cfg)
    E, T, dim = cfg.num_experts, cfg.rows, 128
    g = torch.Generator(device="cuda").manual_seed(cid)
    a = torch.randint(-8, 9, (T, dim), generator=g, device="cuda").to(cfg.dtype)
    scale = (torch.arange(E, device="cuda") % 7 + 1).to(torch.float32)  # neighbours differ
    b = (scale[:, None, None] * torch.eye(dim, device="cuda")).to(cfg.dtype)
    out = _fwd(a, b, bs, cfg.trans_b)
    want = (a.float() * torch.repeat_interleave(scale, bs.cuda())[:, None]).to(cfg.dtype)
    assert torch.equal(out, want)


@pytest.mark.parametrize("cid", [2, 3, 5])
def test_config_checksum_of_checksums(cid):
    """Size-independent property on the full output: row sums of D equal
    A @ (row sums of B[e]) per expert (linearity), checked at fp32 tolerance
    scaled for the rounding of dim_out outputs per row."""
    cfg, bs, a, b = _config_inputs(cid)
    out = _fwd(a, b, bs, cfg.trans_b)
    got = out.float().sum(dim=1)
    bsum = b.float().sum(dim=1 if cfg.trans_b else 2)  # [E, dim]
    off = 0
    want = torch.empty_like(got)
    for e, m in enumerate(bs.tolist()):
        if m:
            want[off:off + m] = a[off:off + m].float() @ bsum[e]
        off += m
    ulp = 2 ** -8 if cfg.dtype == torch.bfloat16 else 2 ** -11
    tol = 4.0 * math.sqrt(cfg.dim_out) * ulp * out.float().abs().mean().item() + 1e-2
    err = (got - want).abs().max().item()
    assert err < tol, (err, tol)
    del a, b, out
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype,trans_b", [(torch.bfloat16, False), (torch.float16, True),
                                           (torch.float32, False)])
def test_host_streamed_matches_device_op(dtype, trans_b):
    """hopper_gmm_fwd_host (pipelined PCIe transfers) gives the device op's bytes,
    in one piece (the default for a problem this small) and cut into chunks."""
    from gmm_b200 import hopper_gmm_fwd, hopper_gmm_fwd_host
    from gmm_b200.streaming import HostStreamedGmm
    g = torch.Generator().manual_seed(9)
    bs = torch.tensor([300, 0, 17, 512, 1, 0, 260, 99, 4])
    T, dim, dim_out = int(bs.sum()), 256, 384
    a = torch.randn(T, dim, generator=g).to(dtype).pin_memory()
    shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
    b = (torch.randn(*shape, generator=g) / 16).to(dtype).pin_memory()
    want = hopper_gmm_fwd(a.cuda(), b.cuda(), bs, trans_b=trans_b).cpu()
    chunked = HostStreamedGmm(n_chunks=4, min_chunk_bytes=1)
    for _ in range(2):  # the second call reuses the pipeline's buffers
        got = hopper_gmm_fwd_host(a, b, bs, trans_b=trans_b)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        got = chunked(a, b, bs, trans_b)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def test_default_swap_tiles_match_the_128_row_kernel_and_the_oracle():
    """Decode-shaped routing (small experts) takes swap-AB tiles by default;
    their output must agree with the 128-row kernel and the oracle."""
    g = torch.Generator().manual_seed(21)
    bs = torch.randint(0, 17, (96,), generator=g)
    bs[::5] = 0
    bs[7] = 64
    T, dim, dim_out = int(bs.sum()), 384, 1000
    for dtype, trans_b in ((torch.bfloat16, False), (torch.float16, True)):
        a = torch.randn(T, dim, generator=g).to(dtype)
        shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
        b = (torch.randn(*shape, generator=g) / dim ** 0.5).to(dtype)
        with forced_tile("auto"):
            auto = _fwd(a.cuda(), b.cuda(), bs, trans_b).cpu()
        with forced_tile("128"):
            big = _fwd(a.cuda(), b.cuda(), bs, trans_b).cpu()
        name = oracle.dtype_name(dtype)
        want = oracle.round_to(oracle.gmm_oracle_c(a, b, bs, trans_b), name)
        for got in (auto, big):
            ok, nbad, err = oracle.allclose_report(got.float().numpy(), want, oracle.TOLERANCE[name])
            assert ok, (name, nbad, err)


@pytest.mark.parametrize("dtype,trans_b", [(torch.bfloat16, False), (torch.float16, True),
                                           (torch.float32, False), (torch.bfloat16, True)])
def test_plan_then_launch_matches_forward(dtype, trans_b):
    """gmm_sm100_plan once, gmm_sm100_launch on two operand sets (two GEMMs that
    share the routing): each bit-identical to a gmm_sm100_forward call."""
    from gmm_b200 import capi
    bs = [130, 0, 1, 700, 64, 0, 255, 9]
    T, dim, dim_out = sum(bs), 192, 320
    plan = capi.Plan(bs, T, dim, dim_out, capi.dtype_code(dtype), trans_b)
    g = torch.Generator().manual_seed(41)
    shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
    for _ in range(2):
        a = torch.randn(T, dim, generator=g).to(dtype).cuda()
        b = (torch.randn(*shape, generator=g) / dim ** 0.5).to(dtype).cuda()
        got = plan.launch(a, b, torch.empty(T, dim_out, dtype=dtype, device="cuda"))
        want = capi.forward(a, b, bs, torch.empty(T, dim_out, dtype=dtype, device="cuda"), trans_b=trans_b)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    plan.close()


def test_concurrent_host_threads_on_their_own_streams():
    """Calls from four host threads at once, each on its own stream and dtype:
    no host-side state is shared between calls, so every result equals the
    single-threaded one (the reference's static host parameter buffer races
    here, reference csrc/hopper_gmm_forward.cu:196)."""
    import threading
    g = torch.Generator().manual_seed(51)
    cases = []
    for i, dtype in enumerate([torch.bfloat16, torch.float16, torch.float32, torch.bfloat16]):
        bs = torch.randint(0, 200, (6 + i,), generator=g)
        bs[i] = 0
        T = int(bs.sum())
        a = torch.randn(T, 128, generator=g).to(dtype).cuda()
        b = (torch.randn(len(bs), 128, 192, generator=g) / 12).to(dtype).cuda()
        cases.append((a, b, bs, _fwd(a, b, bs, False)))
    torch.cuda.synchronize()
    errors = []

    def work(i):
        try:
            torch.cuda.set_device(0)
            s = torch.cuda.Stream()
            a, b, bs, want = cases[i]
            with torch.cuda.stream(s):
                outs = [_fwd(a, b, bs, False) for _ in range(20)]
            s.synchronize()
            if not all(torch.equal(o, want) for o in outs):
                errors.append(f"thread {i}: result differs")
        except Exception as exc:  # noqa: BLE001
            errors.append(f"thread {i}: {exc!r}")

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors


@pytest.mark.parametrize("max_rows", [16, 32, 64, 128])
@pytest.mark.parametrize("trans_b", [False, True])
def test_swap_row_blocks(max_rows, trans_b):
    """Swap-AB tiles whose tallest row block is 16, 32, 64 or 128 rows (the
    MMA's N), zero-row experts between them, against the oracle."""
    g = torch.Generator().manual_seed(max_rows)
    bs = torch.randint(1, max_rows + 1, (40,), generator=g)
    bs[3] = max_rows
    bs[::9] = 0
    T, dim, dim_out = int(bs.sum()), 320, 520
    a = torch.randn(T, dim, generator=g).to(torch.bfloat16)
    shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
    b = (torch.randn(*shape, generator=g) / dim ** 0.5).to(torch.bfloat16)
    with forced_tile("swap"):
        out = _fwd(a.cuda(), b.cuda(), bs, trans_b).cpu()
    want = oracle.round_to(oracle.gmm_oracle_c(a, b, bs, trans_b), "bf16")
    ok, nbad, err = oracle.allclose_report(out.float().numpy(), want, oracle.TOLERANCE["bf16"])
    assert ok, (max_rows, nbad, err)
