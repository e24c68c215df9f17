"""Fused MoE FFN forward: SwiGLU gate/up grouped GEMM (activation in the
epilogue) followed by the down grouped GEMM, against the fp64 oracle.

The oracle applies silu(gate) * up to fp64 per-expert products and rounds
once, which is what the fused epilogue does from its fp32 accumulators; the
tolerances are the grouped GEMM's (bf16 1.6e-2, fp16 2e-3)."""

import pytest
import torch

import oracle
from gpu_util import forced_tile, sampled_subproblem

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


@pytest.fixture(params=["128", "256", "swap"])
def tile(request):
    with forced_tile(request.param):
        yield request.param


def _inputs(bs, dim, inter, dtype, trans_b, seed=0):
    g = torch.Generator().manual_seed(seed)
    T = sum(bs)
    a = torch.randn(T, dim, generator=g).to(dtype)
    shape = (len(bs), 2 * inter, dim) if trans_b else (len(bs), dim, 2 * inter)
    w1 = (torch.randn(*shape, generator=g) / dim ** 0.5).to(dtype)
    return a, w1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("trans_b", [False, True])
def test_swiglu_parity(dtype, trans_b, tile):
    from gmm_b200 import gmm_swiglu
    bs = [1, 0, 300, 7, 129, 0, 520, 33]
    a, w1 = _inputs(bs, 192, 200, dtype, trans_b)  # I=200: a partial 128-column act tile
    got = gmm_swiglu(a.cuda(), w1.cuda(), torch.tensor(bs), trans_b=trans_b)
    torch.cuda.synchronize()
    assert got.shape == (sum(bs), 200) and got.dtype == dtype
    name = oracle.dtype_name(dtype)
    want = oracle.round_to(oracle.swiglu_oracle(a, w1, bs, trans_b), name)
    ok, nbad, err = oracle.allclose_report(got.float().cpu().numpy(), want, oracle.TOLERANCE[name])
    assert ok, f"{nbad} bad, max err {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_moe_ffn_parity(dtype, tile):
    from gmm_b200 import moe_ffn
    bs = [64, 0, 250, 3, 400]
    dim, inter = 256, 384
    a, w1 = _inputs(bs, dim, inter, dtype, False, seed=1)
    g = torch.Generator().manual_seed(2)
    w2 = (torch.randn(len(bs), inter, dim, generator=g) / inter ** 0.5).to(dtype)
    got = moe_ffn(a.cuda(), w1.cuda(), w2.cuda(), torch.tensor(bs))
    torch.cuda.synchronize()
    name = oracle.dtype_name(dtype)
    h = torch.from_numpy(oracle.round_to(oracle.swiglu_oracle(a, w1, bs, False), name)).to(dtype)
    want = oracle.round_to(oracle.gmm_oracle_c(h, w2, bs, False), name)
    # two roundings of the hidden activation may differ by an ulp: allow a
    # second tolerance step for the down projection of a rounded input
    ok, nbad, err = oracle.allclose_report(got.float().cpu().numpy(), want, 2 * oracle.TOLERANCE[name])
    assert ok, f"{nbad} bad, max err {err:.3e}"


def test_swiglu_mixtral_shape_sampled_rows():
    """Mixtral-8x7B expert FFN shapes (dim 4096, I 14336, cfg2 routing): sampled rows."""
    from gmm_b200 import gmm_swiglu
    from gmm_b200.configs import CONFIGS, batch_sizes_for
    cfg = CONFIGS[2]
    bs = batch_sizes_for(cfg)
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(cfg.rows, 4096, generator=g, device="cuda").bfloat16()
    w1 = (torch.randn(8, 4096, 2 * 14336, generator=g, device="cuda") / 64).bfloat16()
    got = gmm_swiglu(a, w1, bs)
    rows, experts, sub_bs = sampled_subproblem(bs.tolist(), rows_per_expert=3)
    ridx = torch.as_tensor(rows, device="cuda")
    want = oracle.round_to(oracle.swiglu_oracle(a[ridx].cpu(), w1[experts].cpu(), sub_bs, False), "bf16")
    ok, nbad, err = oracle.allclose_report(got[ridx].float().cpu().numpy(), want, 1.6e-2)
    assert ok, (nbad, err)
