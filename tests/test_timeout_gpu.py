"""The bounded-wait path of the persistent kernels, made to run out on purpose.

Every mbarrier wait in the 128-row and CTA-pair kernels gives up after a time
limit, raises the CTA's abort flag, lets the copies it has in flight land,
frees its tensor memory and records GMM_ERR_DEVICE_TIMEOUT in the device error
word.  ``gmm_sm100_forward_inject_timeout`` shortens that limit to 50 ms and
has the producer of CTA (pair) 0 skip one k-block's loads, so the MMA warp
waits for data that never comes.  The test checks that the kernel returns,
that the host reads the timeout status, and that the next ordinary call on
the same stream is correct -- the context survives.  No GPU fault, trap or
hang is involved: the kernel ends by its own bounded waits.
"""

import numpy as np
import pytest
import torch

import oracle
from gpu_util import forced_tile

pytestmark = pytest.mark.gpu

GMM_ERR_DEVICE_TIMEOUT = -9


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    from gmm_b200 import capi
    capi.device_error(clear=True)
    yield
    capi.device_error(clear=True)


@pytest.mark.parametrize("tile", ["128", "256"])
def test_wait_runs_out_and_the_context_survives(tile):
    from gmm_b200 import capi, hopper_gmm_fwd
    lib = capi.load()
    bs = [300, 0, 200, 17]
    T, dim, dim_out = sum(bs), 512, 512  # 8 k-blocks of 64
    g = torch.Generator().manual_seed(5)
    a = torch.randn(T, dim, generator=g).to(torch.bfloat16).cuda()
    b = (torch.randn(len(bs), dim, dim_out, generator=g) / dim ** 0.5).to(torch.bfloat16).cuda()
    d = torch.empty(T, dim_out, dtype=torch.bfloat16, device="cuda")
    arr = np.asarray(bs, dtype=np.int64)
    stream = torch.cuda.current_stream()
    try:
        with forced_tile(tile):
            rc = lib.gmm_sm100_forward_inject_timeout(
                a.data_ptr(), b.data_ptr(), arr.ctypes.data, len(bs), T, dim, dim_out,
                capi.GMM_DTYPE_BF16, 0, d.data_ptr(), 2, 0.05, stream.cuda_stream)
            assert rc == 0, lib.gmm_sm100_last_error().decode()
            stream.synchronize()  # the kernel returns by itself
            assert capi.device_error(clear=True) == GMM_ERR_DEVICE_TIMEOUT
            # the same stream, an ordinary call: correct, and no new error
            out = hopper_gmm_fwd(a, b, torch.tensor(bs), trans_b=False)
            stream.synchronize()
        assert capi.device_error(clear=True) == 0
        want = oracle.round_to(oracle.gmm_oracle_c(a.cpu(), b.cpu(), bs, False), "bf16")
        ok, nbad, err = oracle.allclose_report(out.float().cpu().numpy(), want, oracle.TOLERANCE["bf16"])
        assert ok, (nbad, err)
    finally:
        capi.device_error(clear=True)


def test_inject_rejects_what_it_cannot_run():
    from gmm_b200 import capi
    lib = capi.load()
    arr = np.asarray([64], dtype=np.int64)
    # fp32, a k-block past the end, a limit beyond 2 s: rejected on the host
    assert lib.gmm_sm100_forward_inject_timeout(16, 16, arr.ctypes.data, 1, 64, 64, 64,
                                                capi.GMM_DTYPE_F32, 0, 16, 0, 0.05, None) == -3
    assert lib.gmm_sm100_forward_inject_timeout(16, 16, arr.ctypes.data, 1, 64, 64, 64,
                                                capi.GMM_DTYPE_BF16, 0, 16, 5, 0.05, None) == -1
    assert lib.gmm_sm100_forward_inject_timeout(16, 16, arr.ctypes.data, 1, 64, 64, 64,
                                                capi.GMM_DTYPE_BF16, 0, 16, 0, 3.0, None) == -1
