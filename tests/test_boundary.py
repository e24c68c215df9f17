"""The drop-in boundary, checked without a GPU: op schema, fake impl, Python
signature, the C ABI's exported symbols and its host-side validation."""

import ctypes
import inspect
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gmm_sm100.h")


def test_header_symbols_exported():
    from gmm_b200 import capi
    lib = capi.load()
    declared = set(re.findall(r"\b(gmm_sm100_\w+)\s*\(", open(HEADER).read()))
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert declared == set(capi._SIGNATURES), "ctypes binding out of sync with the header"


def test_op_schema_matches_reference():
    import gmm_b200  # noqa: F401
    schema = str(torch.ops.hopper_gmm_fwd.gmm.default._schema)
    assert schema == ("hopper_gmm_fwd::gmm(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor")


def test_python_signature_matches_reference():
    from gmm_b200 import hopper_gmm_fwd
    import hopper_gmm_forward
    sig = inspect.signature(hopper_gmm_fwd)
    assert list(sig.parameters) == ["a", "b", "batch_sizes", "trans_b"]
    assert sig.parameters["trans_b"].default is False
    assert hopper_gmm_forward.hopper_gmm_fwd is hopper_gmm_fwd
    assert hopper_gmm_forward.__all__ == ["hopper_gmm_fwd"]


@pytest.mark.parametrize("trans_b", [False, True])
def test_fake_impl_shapes(trans_b):
    import gmm_b200  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        bs = torch.tensor([128, 0, 384])
        a = torch.empty(512, 64, dtype=torch.float16, device="cuda")
        b = torch.empty(3, 96, 64, dtype=torch.float16, device="cuda") if trans_b else \
            torch.empty(3, 64, 96, dtype=torch.float16, device="cuda")
        out = torch.ops.hopper_gmm_fwd.gmm(a, b, bs, trans_b)
        assert tuple(out.shape) == (512, 96) and out.dtype == torch.float16
        assert out.device.type == "cuda"


def test_cpu_tensors_have_no_kernel():
    """Like the reference, only the CUDA dispatch key is implemented: no CPU fallback."""
    import gmm_b200  # noqa: F401
    with pytest.raises(NotImplementedError):
        torch.ops.hopper_gmm_fwd.gmm(torch.zeros(4, 8), torch.zeros(1, 8, 8), torch.tensor([4]), False)


def _cabi_forward(bs, T, dim=16, dim_out=16, dtype=1, trans_b=0):
    from gmm_b200 import capi
    lib = capi.load()
    arr = np.asarray(bs, dtype=np.int64)
    # Non-null dummy pointers: validation fails before any CUDA call.
    rc = lib.gmm_sm100_forward(16, 16, arr.ctypes.data, len(bs), T, dim, dim_out, dtype, trans_b,
                               16, None, 0, None)
    return rc, lib.gmm_sm100_last_error().decode()


def test_cabi_validates_on_host():
    rc, msg = _cabi_forward([3, 4], 10)
    assert rc == -2 and msg == "Sum of batch_sizes (7) must equal A.size(0) (10)"
    rc, msg = _cabi_forward([3, -1], 2)
    assert rc == -1 and "negative" in msg
    rc, msg = _cabi_forward([3], 3, dtype=7)
    assert rc == -3 and msg.startswith("Unsupported dtype")
    rc, _ = _cabi_forward([0, 0], 0)  # T = 0: nothing to do, no CUDA call
    assert rc == 0


def test_cabi_errstr_and_workspace():
    from gmm_b200 import capi
    lib = capi.load()
    for code in range(0, -10, -1):
        assert lib.gmm_sm100_errstr(code) not in (None, b"unknown status")
    assert lib.gmm_sm100_errstr(-100) == b"unknown status"
    # bf16/fp16 with a small table: no workspace
    assert capi.workspace_size([64] * 8, 512, 128, 256, capi.GMM_DTYPE_BF16, False) == 0
    # fp32: none either (the TF32 hi/lo split is made in shared memory)
    assert capi.workspace_size([64] * 8, 512, 128, 256, capi.GMM_DTYPE_F32, False) == 0
    assert capi.workspace_size([64] * 8, 512, 128, 256, capi.GMM_DTYPE_F32, True) == 0
    # more than 1024 non-empty experts: the table moves to the workspace
    ws = capi.workspace_size([1] * 2000, 2000, 64, 64, capi.GMM_DTYPE_F16, True)
    assert ws == ((3 * 2000 + 2) * 4 + 255) // 256 * 256


def test_swiglu_op_schema_and_fake():
    import gmm_b200  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    assert str(torch.ops.hopper_gmm_fwd.gmm_swiglu.default._schema) == (
        "hopper_gmm_fwd::gmm_swiglu(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor")
    with FakeTensorMode():
        a = torch.empty(64, 32, dtype=torch.bfloat16, device="cuda")
        b = torch.empty(2, 32, 96, dtype=torch.bfloat16, device="cuda")
        out = gmm_b200.gmm_swiglu(a, b, torch.tensor([30, 34]))
        assert tuple(out.shape) == (64, 48)


def test_cabi_other_entries_validate_on_host():
    """Every entry point rejects bad arguments with a status and a message
    before it touches the GPU (dummy non-null pointers, no device here)."""
    from gmm_b200 import capi
    lib = capi.load()
    P = 256  # a non-null, 16-byte-aligned dummy address; never dereferenced

    def last():
        return lib.gmm_sm100_last_error().decode()

    bs = np.asarray([3, 4], dtype=np.int64)
    # variable-K: sum, dtype, row pitch
    assert lib.gmm_sm100_forward_vark(P, P, bs.ctypes.data, 2, 9, 64, 64, 1, P, None) == -2
    assert "Sum of batch_sizes (7)" in last()
    assert lib.gmm_sm100_forward_vark(P, P, bs.ctypes.data, 2, 7, 64, 64, 0, P, None) == -3
    assert lib.gmm_sm100_forward_vark(P, P, bs.ctypes.data, 2, 7, 12, 64, 1, P, None) == -4
    # SwiGLU: 16-bit only, gate/up width a multiple of 8
    assert lib.gmm_sm100_forward_swiglu(P, P, bs.ctypes.data, 2, 7, 64, 128, 0, 0, P, None, 0, None) == -3
    assert lib.gmm_sm100_forward_swiglu(P, P, bs.ctypes.data, 2, 7, 64, 40, 1, 0, P, None, 0, None) == -4
    # device batch sizes: expert count, SwiGLU dtype, alignment of D and of the sizes
    assert lib.gmm_sm100_forward_dev(P, P, P, 0, 8, 64, 64, 1, 0, 0, P, None, 0, None) == -1
    assert lib.gmm_sm100_forward_dev(P, P, P, 1025, 8, 64, 64, 1, 0, 0, P, None, 0, None) == -1
    assert lib.gmm_sm100_forward_dev(P, P, P, 4, 8, 64, 64, 0, 0, 1, P, None, 0, None) == -1
    assert lib.gmm_sm100_forward_dev(P, P, P, 4, 8, 64, 64, 1, 0, 0, P + 8, None, 0, None) == -4
    assert lib.gmm_sm100_forward_dev(P, P, P + 2, 4, 8, 64, 64, 1, 0, 0, P, None, 0, None) == -4
    # the allocation-free fp32 entry: a tile table (800,000 non-empty experts)
    # larger than the fixed array
    big = np.ones(800_000, dtype=np.int64)
    rc = lib.gmm_sm100_forward_f32_noalloc(P, P, big.ctypes.data, big.shape[0], big.shape[0], 64, 64, 0, P, None)
    assert rc == -8 and "fixed scratch holds 8388608 bytes" in last()
    assert lib.gmm_sm100_forward_f32_noalloc(P, P, bs.ctypes.data, 2, 9, 64, 64, 0, P, None) == -2
    # routing and permutation
    moe_last = lambda: lib.gmm_sm100_moe_last_error().decode()  # noqa: E731
    assert lib.gmm_sm100_moe_topk(P, 0, 16, 8, 0, 1, P, P, None) == -1
    assert lib.gmm_sm100_moe_topk(P, 0, 16, 8, 9, 1, P, P, None) == -1
    assert lib.gmm_sm100_moe_topk(P, 0, 16, 2000, 2, 1, P, P, None) == -1 and "1024" in moe_last()
    assert lib.gmm_sm100_moe_permute(P, 16, 24, P, 2, 8, P, P, P, P, None, 0, None) == -4
    assert lib.gmm_sm100_moe_permute(P, 16, 32, P, 2, 0, P, P, P, P, None, 0, None) == -1
    assert lib.gmm_sm100_moe_unpermute(P, P, P, 16, 2, 12, 1, P, None) == -4
    assert lib.gmm_sm100_moe_unpermute(P, P, P, 16, 0, 64, 1, P, None) == -1


def test_plan_is_host_only_and_agrees_with_workspace_size():
    """gmm_sm100_plan makes no CUDA call (this host has no GPU) and asks for
    the workspace gmm_sm100_workspace_size reports for the same problem."""
    import ctypes
    from gmm_b200 import capi
    lib = capi.load()
    cases = [([64] * 8, 512, 128, 256, capi.GMM_DTYPE_F32, False),
             ([5, 0, 300, 1], 306, 64, 128, capi.GMM_DTYPE_BF16, False),
             ([2000] * 8, 16000, 64, 64, capi.GMM_DTYPE_BF16, True),
             ([1] * 2000, 2000, 64, 64, capi.GMM_DTYPE_F16, True)]
    for bs, T, dim, dim_out, dt, tb in cases:
        p = capi.Plan(bs, T, dim, dim_out, dt, tb)
        assert p.workspace_size == capi.workspace_size(bs, T, dim, dim_out, dt, tb)
        p.close()
    with pytest.raises(capi.GmmError, match=r"Sum of batch_sizes \(7\) must equal A.size\(0\) \(9\)"):
        capi.Plan([3, 4], 9, 64, 64, capi.GMM_DTYPE_BF16)
    with pytest.raises(capi.GmmError, match="Unsupported dtype"):
        capi.Plan([3, 4], 7, 64, 64, 9)
    arr = np.asarray([1, 2], dtype=np.int64)
    assert lib.gmm_sm100_plan(arr.ctypes.data, 2, 3, 64, 64, 1, 0, None) == -1
    assert lib.gmm_sm100_launch(None, 16, 16, 16, None, 0, None) == -1
    # an empty problem launches as a no-op, without touching the device
    h = ctypes.c_void_p()
    zero = np.zeros(3, dtype=np.int64)
    assert lib.gmm_sm100_plan(zero.ctypes.data, 3, 0, 64, 64, 1, 0, ctypes.byref(h)) == 0
    assert lib.gmm_sm100_launch(h, 16, 16, 16, None, 0, None) == 0
    lib.gmm_sm100_plan_free(h)
    lib.gmm_sm100_plan_free(None)


def test_tile_kind_override_roundtrip():
    """The process-wide kernel-family override (gmm_sm100_set_tile_kind)
    returns the previous setting and rejects unknown kinds."""
    from gmm_b200 import capi
    prev = capi.set_tile_kind("128")
    try:
        assert capi.set_tile_kind("swap") == "128"
        assert capi.set_tile_kind("256") == "swap"
        assert capi.load().gmm_sm100_set_tile_kind(9) == -1
        assert capi.set_tile_kind("auto") == "256"
    finally:
        capi.set_tile_kind(prev)


def test_host_pipeline_chunking():
    """hopper_gmm_fwd_host moves a small problem in one piece and cuts a large
    one into expert chunks of at least min_chunk_bytes each (host logic only)."""
    from gmm_b200.configs import CONFIGS, batch_sizes_for
    from gmm_b200.streaming import _chunks, chunk_count
    mb = 1 << 20
    assert chunk_count(2 * mb, 8, 32 * mb) == 1           # cfg1-sized: one chunk
    assert chunk_count(0, 8, 32 * mb) == 1
    assert chunk_count(100 * mb, 8, 32 * mb) == 3
    assert chunk_count(1544 * mb, 8, 32 * mb) == 8        # cfg2-sized: the full pipeline
    assert chunk_count(10 * mb, 8, 0) == 8                 # no floor: n_chunks
    for cid in (1, 2, 3, 4, 5):
        bs = [int(v) for v in batch_sizes_for(CONFIGS[cid]).tolist()]
        for n in (1, 3, 8):
            spans = _chunks(bs, n)
            assert spans[0][0] == 0 and spans[-1][1] == len(bs)
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert 1 <= len(spans) <= n
