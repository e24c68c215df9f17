"""Variable-K grouped GEMM (MoE backward weight gradient) against the fp64 oracle:
D[e] = A[rows_e]^T @ B[rows_e].  Ragged row counts that are not multiples of the
64-row contraction block make the kernel zero the next expert's rows in shared
memory; empty experts must come out as exact zeros."""

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bs,M,N", [([100, 0, 1, 300, 64, 0, 129], 192, 320),
                                    ([64] * 8, 128, 256),
                                    ([0, 0, 5], 64, 64),
                                    ([1000, 37], 256, 512)])
def test_vark_parity(dtype, bs, M, N):
    from gmm_b200 import gmm_vark
    g = torch.Generator().manual_seed(len(bs) + M)
    T = sum(bs)
    # scaled so the fp16 sums over ~1000 rows stay well inside range
    a = (torch.randn(T, M, generator=g) / 4).to(dtype)
    b = (torch.randn(T, N, generator=g) / 4).to(dtype)
    got = gmm_vark(a.cuda(), b.cuda(), torch.tensor(bs)).float().cpu().numpy()
    name = oracle.dtype_name(dtype)
    want = oracle.round_to(oracle.vark_oracle(a, b, bs), name)
    ok, nbad, err = oracle.allclose_report(got, want, oracle.TOLERANCE[name])
    assert ok, f"{nbad} bad, max err {err:.3e}"
    for e, m in enumerate(bs):
        if m == 0:
            assert (got[e] == 0).all()


def test_vark_next_expert_rows_do_not_leak():
    """Expert 0 has 10 rows; expert 1's rows are huge: any leak would show."""
    from gmm_b200 import gmm_vark
    a = torch.ones(74, 64, dtype=torch.bfloat16)
    b = torch.ones(74, 64, dtype=torch.bfloat16)
    a[10:] = 1000.0
    got = gmm_vark(a.cuda(), b.cuda(), torch.tensor([10, 64])).float().cpu()
    assert torch.equal(got[0], torch.full((64, 64), 10.0))
    assert torch.equal(got[1], torch.full((64, 64), 64000.0))


def test_vark_rejects_bad_sum():
    from gmm_b200 import gmm_vark
    a = torch.ones(10, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="Sum of batch_sizes"):
        gmm_vark(a, a, torch.tensor([4, 5]))
