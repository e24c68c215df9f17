"""Device-resident MoE layer: routing, permutation, grouped GEMMs with device
batch sizes, combine -- each against the CPU oracle, and the whole layer
captured and replayed as a CUDA graph (it never synchronises with the host).

Index work (expert ids, batch sizes, row positions, permuted rows) must be
bit-exact; floating-point results use the grouped GEMM's tolerances."""

import numpy as np
import pytest
import torch

import oracle
from gpu_util import forced_tile

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    yield
    from gmm_b200 import capi
    capi.device_error(clear=True)


@pytest.fixture(params=["128", "256", "swap"])
def tile(request):
    with forced_tile(request.param):
        yield request.param


@pytest.mark.parametrize("E,k,dtype", [(8, 2, torch.float32), (128, 8, torch.bfloat16),
                                       (256, 8, torch.float32), (1000, 4, torch.float16)])
def test_topk_route(E, k, dtype):
    from gmm_b200.moe import topk_route
    g = torch.Generator().manual_seed(E)
    logits = torch.randn(777, E, generator=g).to(dtype)
    logits[5, 3] = logits[5, 1] = 50.0  # a tie at the top: lower index first
    ids, w = topk_route(logits.cuda(), k)
    want_ids, want_w = oracle.topk_oracle(logits, k, renormalize=True)
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-5, atol=1e-6)
    ids2, w2 = topk_route(logits.cuda(), k, renormalize=False)
    np.testing.assert_array_equal(ids2.cpu().numpy(), want_ids)
    _, raw = oracle.topk_oracle(logits, k, renormalize=False)
    np.testing.assert_allclose(w2.cpu().numpy(), raw, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T,k,E", [(1, 1, 4), (1000, 2, 8), (4096, 8, 256), (9000, 3, 1024)])
def test_permute_is_a_stable_sort(T, k, E):
    from gmm_b200.moe import permute
    g = torch.Generator().manual_seed(T)
    ids = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32)
    x = torch.randn(T, 64, generator=g).bfloat16()
    xp, bs, dst, src = permute(x.cuda(), ids.cuda(), E)
    want_bs, want_dst, want_src = oracle.permute_oracle(ids.numpy(), E)
    np.testing.assert_array_equal(bs.cpu().numpy(), want_bs)
    np.testing.assert_array_equal(dst.cpu().numpy(), want_dst)
    np.testing.assert_array_equal(src.cpu().numpy(), want_src)
    assert torch.equal(xp.cpu(), x[torch.from_numpy(want_src).long()])


def test_permute_ignores_out_of_range_ids():
    from gmm_b200.moe import permute
    ids = torch.tensor([[0, 5], [9, 1], [-2, 1]], dtype=torch.int32)
    x = torch.arange(3 * 8, dtype=torch.float32).view(3, 8)
    xp, bs, dst, src = permute(x.cuda(), ids.cuda(), 6)
    assert bs.cpu().tolist() == [1, 2, 0, 0, 0, 1]
    d = dst.cpu()
    assert d[1, 0] == -1 and d[2, 0] == -1
    assert torch.equal(xp[:4].cpu(), x[[0, 1, 2, 0]])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_unpermute(dtype):
    from gmm_b200.moe import unpermute
    g = torch.Generator().manual_seed(1)
    T, k, N = 300, 4, 136
    y = torch.randn(T * k, N, generator=g).to(dtype)
    dst = torch.randperm(T * k, generator=g).view(T, k).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    got = unpermute(y.cuda(), dst.cuda(), w.cuda()).float().cpu().numpy()
    want = oracle.round_to(oracle.unpermute_oracle(y, dst.numpy(), w), oracle.dtype_name(dtype))
    name = oracle.dtype_name(dtype)
    ok, nbad, err = oracle.allclose_report(got, want, oracle.TOLERANCE[name])
    assert ok, (nbad, err)


@pytest.mark.parametrize("dtype,trans_b", [(torch.bfloat16, False), (torch.float16, True),
                                           (torch.float32, False)])
def test_device_batch_sizes_match_host_batch_sizes(dtype, trans_b, tile):
    """Same kernel, table built on the device: bit-identical to the host-table op."""
    from gmm_b200 import hopper_gmm_fwd
    from gmm_b200.moe import grouped_gemm_dev
    bs = [130, 0, 1, 700, 64, 0, 255]
    cap = sum(bs) + 50  # spare rows past the experts' total are left alone
    g = torch.Generator().manual_seed(2)
    a = torch.randn(cap, 192, generator=g).to(dtype).cuda()
    shape = (len(bs), 320, 192) if trans_b else (len(bs), 192, 320)
    b = (torch.randn(*shape, generator=g) / 14).to(dtype).cuda()
    got = grouped_gemm_dev(a, b, torch.tensor(bs, dtype=torch.int32, device="cuda"), trans_b)
    want = hopper_gmm_fwd(a[:sum(bs)], b, torch.tensor(bs), trans_b=trans_b)
    torch.cuda.synchronize()
    assert torch.equal(got[:sum(bs)], want)


def test_device_batch_sizes_swiglu_matches_host(tile):
    from gmm_b200 import gmm_swiglu
    from gmm_b200.moe import grouped_gemm_dev
    bs = [40, 300, 0, 90]
    g = torch.Generator().manual_seed(3)
    a = torch.randn(sum(bs), 128, generator=g).bfloat16().cuda()
    b = (torch.randn(4, 128, 2 * 136, generator=g) / 11).bfloat16().cuda()
    got = grouped_gemm_dev(a, b, torch.tensor(bs, dtype=torch.int32, device="cuda"), swiglu=True)
    want = gmm_swiglu(a, b, torch.tensor(bs))
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_device_batch_sizes_errors_are_recorded_not_faulted():
    from gmm_b200 import capi
    from gmm_b200.moe import grouped_gemm_dev
    capi.device_error(clear=True)
    a = torch.randn(100, 64, device="cuda").bfloat16()
    b = torch.randn(2, 64, 64, device="cuda").bfloat16()
    grouped_gemm_dev(a, b, torch.tensor([80, 30], dtype=torch.int32, device="cuda"))  # 110 > 100 rows
    torch.cuda.synchronize()
    assert capi.device_error(clear=True) == -2
    grouped_gemm_dev(a, b, torch.tensor([-1, 30], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert capi.device_error(clear=True) == -1


def _layer_inputs(T=2000, E=16, k=2, dim=256, inter=320, dtype=torch.bfloat16, seed=4):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, dim, generator=g).to(dtype)
    logits = torch.randn(T, E, generator=g)
    w1 = (torch.randn(E, dim, 2 * inter, generator=g) / dim ** 0.5).to(dtype)
    w2 = (torch.randn(E, inter, dim, generator=g) / inter ** 0.5).to(dtype)
    return x, logits, w1, w2


def test_moe_forward_matches_oracle(tile):
    from gmm_b200.moe import moe_forward
    x, logits, w1, w2 = _layer_inputs()
    got = moe_forward(x.cuda(), logits.cuda(), w1.cuda(), w2.cuda(), k=2).float().cpu().numpy()
    ids, w = oracle.topk_oracle(logits, 2)
    bs, dst, src = oracle.permute_oracle(ids, 16)
    xp = x[torch.from_numpy(src).long()]
    h = torch.from_numpy(oracle.round_to(oracle.swiglu_oracle(xp, w1, bs, False), "bf16")).bfloat16()
    y = torch.from_numpy(oracle.round_to(oracle.gmm_oracle_c(h, w2, bs, False), "bf16"))
    want = oracle.round_to(oracle.unpermute_oracle(y, dst, w.astype(np.float32)), "bf16")
    ok, nbad, err = oracle.allclose_report(got, want, 2 * 1.6e-2)
    assert ok, (nbad, err)


def test_moe_forward_captured_in_a_cuda_graph():
    from gmm_b200.moe import moe_forward
    x, logits, w1, w2 = _layer_inputs(seed=5)
    xs, ls, w1d, w2d = x.cuda(), logits.cuda(), w1.cuda(), w2.cuda()
    eager = moe_forward(xs, ls, w1d, w2d, k=2)  # first call also sets kernel attributes
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe_forward(xs, ls, w1d, w2d, k=2)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = moe_forward(xs, ls, w1d, w2d, k=2)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new routing and activations through the same graph
    x2, logits2, _, _ = _layer_inputs(seed=6)
    xs.copy_(x2.cuda())
    ls.copy_(logits2.cuda())
    graph.replay()
    want = moe_forward(xs, ls, w1d, w2d, k=2)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
