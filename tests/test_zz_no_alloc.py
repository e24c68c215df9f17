"""The allocation-free fp32 entry point, ``gmm_sm100_forward_f32_noalloc``.

It serves callers that cannot allocate device memory themselves (a plugin
inside an engine that owns every allocation, or a caller that cannot let
cudaMalloc / cudaFree synchronise the device): the one device buffer the fp32
path can need -- the tile table of more than 1024 non-empty experts -- lives
in a fixed array compiled into the library.  These tests drive it through the
C ABI and check it against the CPU oracle at the fp32 tolerance used by every
other test, and against the regular entry point, on two calls in a row (so a
second call that reuses the shared array is covered too), including a
problem whose table does go through the array.

This file is named to be collected last.
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = oracle.TOLERANCE["fp32"]


def _noalloc(a, b, bs, trans_b, d):
    from gmm_b200 import capi
    lib = capi.load()
    arr = np.ascontiguousarray(np.asarray(bs, dtype=np.int64))
    dim_out = b.shape[1] if trans_b else b.shape[2]
    rc = lib.gmm_sm100_forward_f32_noalloc(
        a.data_ptr(), b.data_ptr(), arr.ctypes.data, arr.shape[0], a.shape[0], a.shape[1], dim_out,
        int(trans_b), d.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return rc, lib.gmm_sm100_last_error().decode()


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def _problem(g, bs, dim, dim_out, trans_b):
    T = int(sum(bs))
    a = torch.randn(T, dim, generator=g)
    shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
    b = torch.randn(*shape, generator=g)
    return a, b


@pytest.mark.parametrize("trans_b", [False, True])
def test_noalloc_matches_oracle_and_regular_entry_twice(trans_b):
    from gmm_b200 import hopper_gmm_fwd
    g = torch.Generator().manual_seed(21)
    many = torch.randint(1, 4, (1200,), generator=g)
    many[::11] = 0  # 1090 non-empty experts, some empty ones between them
    problems = [([64, 0, 130, 1, 57], 192, 320),  # inline tile table
                (many.tolist(), 32, 64),           # more than 1024 non-empty experts: table in the array
                ([512] * 8, 128, 256)]             # inline again, after the array was used
    assert sum(1 for m in problems[1][0] if m > 0) > 1024
    for bs, dim, dim_out in problems:  # calls in a row on the shared array
        a, b = _problem(g, bs, dim, dim_out, trans_b)
        d = torch.full((a.shape[0], dim_out), float("nan"), device="cuda")
        rc, msg = _noalloc(a.cuda(), b.cuda(), bs, trans_b, d)
        assert rc == 0, msg
        torch.cuda.synchronize()
        got = d.cpu().numpy()
        want = oracle.gmm_oracle_c(a, b, bs, trans_b)
        ok, nbad, err = oracle.allclose_report(got, want, TOL)
        assert ok, f"{len(bs)} experts: {nbad} elements off the oracle beyond {TOL}, max err {err}"
        regular = hopper_gmm_fwd(a.cuda(), b.cuda(), torch.tensor(bs), trans_b=trans_b).cpu().numpy()
        ok, nbad, err = oracle.allclose_report(got, regular, TOL)
        assert ok, f"{len(bs)} experts: {nbad} elements off the regular entry point, max err {err}"


def test_noalloc_rejects_tables_beyond_its_array():
    """800,000 one-row experts need a 9.6 MB tile table: more than the fixed
    8 MiB array, so the call is rejected on the host, before any GPU work."""
    E = 800_000
    bs = np.ones(E, dtype=np.int64)
    a = torch.zeros(E, 4, device="cuda")
    b = torch.zeros(E, 4, 4, device="cuda")
    d = torch.zeros(E, 4, device="cuda")
    rc, msg = _noalloc(a, b, bs, False, d)
    assert rc == -8 and "scratch" in msg
