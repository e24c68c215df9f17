"""The allocation-free fp32 entry point, ``gmm_sm100_forward_f32_noalloc``.

It serves callers that cannot allocate device memory themselves (a plugin
inside an engine that owns every allocation, or a caller that cannot let
cudaMalloc / cudaFree synchronise the device): its scratch is a fixed array
compiled into the library.  These tests drive it through the C ABI and check
it against the regular entry point (``hopper_gmm_fwd`` -> ``gmm_sm100_forward``)
at the fp32 tolerance used by every other test, on two calls in a row, so a
second call that reuses the shared scratch is covered too.

This file is named to be collected last.
"""

import ctypes

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


@pytest.mark.parametrize("trans_b", [False, True])
def test_noalloc_matches_regular_entry_twice(trans_b):
    from gmm_b200 import hopper_gmm_fwd
    g = torch.Generator().manual_seed(21)
    problems = [([64, 0, 130, 1, 57], 192, 320), ([512] * 8, 128, 256)]
    for bs, dim, dim_out in problems:  # two calls in a row on the shared scratch
        T = sum(bs)
        a = torch.randn(T, dim, generator=g).cuda()
        shape = (len(bs), dim_out, dim) if trans_b else (len(bs), dim, dim_out)
        b = torch.randn(*shape, generator=g).cuda()
        d = torch.full((T, dim_out), float("nan"), device="cuda")
        rc, msg = _noalloc(a, b, bs, trans_b, d)
        assert rc == 0, msg
        want = hopper_gmm_fwd(a, b, torch.tensor(bs), trans_b=trans_b)
        torch.cuda.synchronize()
        ok, nbad, err = oracle.allclose_report(d.cpu().numpy(), want.cpu().numpy(), TOL)
        assert ok, f"bs={bs}: {nbad} elements differ beyond {TOL}, max err {err}"


def test_noalloc_rejects_problems_beyond_its_scratch():
    bs = [1024] * 8
    a = torch.zeros(8192, 256, device="cuda")
    b = torch.zeros(8, 256, 512, device="cuda")
    d = torch.zeros(8192, 512, device="cuda")
    rc, msg = _noalloc(a, b, bs, False, d)
    assert rc == -8 and "scratch" in msg
