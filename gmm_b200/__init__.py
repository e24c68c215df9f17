"""gmm_b200 -- B200-native (sm_100a) MoE grouped-GEMM forward.

Drop-in for the reference's Python surface (reference
``hopper_gmm_forward/__init__.py:59-88``)::

    from gmm_b200 import hopper_gmm_fwd          # or: from hopper_gmm_forward import ...
    d = hopper_gmm_fwd(a, b, batch_sizes)        # d[rows_e] = a[rows_e] @ b[e]

The operator is registered as ``torch.ops.hopper_gmm_fwd.gmm`` (schema
``gmm(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor``) by
the in-tree ``_C.so``, loaded with ``torch.ops.load_library`` like the
reference's extension (reference ``hopper_gmm_forward/__init__.py:19-46``);
its fake (meta) implementation is registered here for ``torch.compile`` /
export.  There is no CPU fallback: without the native library the call
raises ``RuntimeError``.
"""

from __future__ import annotations

import os
import warnings

import torch

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_TORCH_OP = os.path.join(_PKG_DIR, "_C.so")
_HAS_C = False


def _load_c_ext() -> bool:
    if not os.path.exists(_TORCH_OP):
        return False
    try:
        torch.ops.load_library(_TORCH_OP)
    except Exception as e:  # noqa: BLE001
        warnings.warn(f"gmm_b200: failed to load {_TORCH_OP}: {e}", RuntimeWarning)
        return False
    return True


def load_native() -> bool:
    """Load ``_C.so`` (registering the ops and their fake impls) if not done yet.

    Called at import; a build run in the same process calls it again once the
    library exists."""
    global _HAS_C
    if _HAS_C:
        return True
    if not _load_c_ext():
        return False
    _HAS_C = True
    _register_fakes()
    return True


def hopper_gmm_fwd(a: torch.Tensor,
                   b: torch.Tensor,
                   batch_sizes: torch.Tensor,
                   trans_b: bool = False) -> torch.Tensor:
    """Forward-only grouped GEMM on B200 (sm_100a).

    Args:
        a: ``[num_tokens, dim]`` contiguous CUDA, fp32/bf16/fp16.
        b: ``[num_experts, dim, dim_out]`` (or ``[num_experts, dim_out, dim]``
           if ``trans_b=True``) contiguous CUDA, same dtype as ``a``.
        batch_sizes: ``[num_experts]`` int64 tensor on CPU; rows
           ``[sum(batch_sizes[:e]), sum(batch_sizes[:e+1]))`` of ``a`` belong
           to expert ``e`` and ``sum(batch_sizes)`` must equal ``num_tokens``.
        trans_b: ``b`` holds each expert's matrix transposed. For fp32 the
           products run as three TF32 tensor-core passes (near-fp32 accuracy).

    Returns:
        ``[num_tokens, dim_out]`` tensor, same dtype/device as ``a``:
        ``out[rows_e] = a[rows_e] @ (b[e].T if trans_b else b[e])``.
    """
    if not _HAS_C:
        raise RuntimeError("gmm_b200._C is not available. Build with `python -m gmm_b200.build`.")
    return torch.ops.hopper_gmm_fwd.gmm(a, b, batch_sizes, trans_b)


def gmm_swiglu(a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor,
               trans_b: bool = False) -> torch.Tensor:
    """Fused MoE gate/up projection: ``silu(a @ gate[e]) * (a @ up[e])`` per expert segment.

    ``b`` holds each expert's gate and up projections side by side:
    ``[E, dim, 2*I]`` with columns ``[gate | up]`` (``trans_b=False``) or
    ``[E, 2*I, dim]`` with rows ``[gate | up]`` (``trans_b=True``).  Returns
    ``[num_tokens, I]``; the activation is applied to the fp32 accumulators
    inside the GEMM epilogue (bf16 / fp16).
    """
    if not _HAS_C:
        raise RuntimeError("gmm_b200._C is not available. Build with `python -m gmm_b200.build`.")
    return torch.ops.hopper_gmm_fwd.gmm_swiglu(a, b, batch_sizes, trans_b)


def moe_ffn(a: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
            batch_sizes: torch.Tensor, trans_gate_up: bool = False,
            trans_down: bool = False) -> torch.Tensor:
    """MoE expert FFN forward on expert-grouped rows: SwiGLU(a @ w_gate_up) @ w_down.

    Two grouped GEMMs over the same ``batch_sizes``: the gate/up projection
    with SiLU-and-multiply fused into its epilogue, then the down projection
    (``w_down`` is ``[E, I, dim]``, or ``[E, dim, I]`` with ``trans_down``).
    """
    h = gmm_swiglu(a, w_gate_up, batch_sizes, trans_gate_up)
    return hopper_gmm_fwd(h, w_down, batch_sizes, trans_down)


def gmm_vark(a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor) -> torch.Tensor:
    """Variable-K grouped GEMM (MoE backward weight gradient).

    For each expert ``e`` with rows ``rows_e`` (from the CPU int64
    ``batch_sizes``): ``out[e] = a[rows_e].T @ b[rows_e]``; ``a`` is
    ``[T, M]``, ``b`` is ``[T, N]`` (bf16/fp16, CUDA), ``out`` is ``[E, M, N]``
    with fp32 accumulation; an expert with no rows gets zeros.  The sibling of
    the forward kernel that the reference removed from its extract.
    """
    from gmm_b200 import capi
    import numpy as np
    if a.dim() != 2 or b.dim() != 2 or a.shape[0] != b.shape[0]:
        raise RuntimeError("a and b must be 2D with the same number of rows")
    if not (a.is_cuda and b.is_cuda) or a.dtype != b.dtype:
        raise RuntimeError("a and b must be CUDA tensors of one dtype")
    a, b = a.contiguous(), b.contiguous()
    bs = np.ascontiguousarray(batch_sizes.cpu().numpy().astype(np.int64))
    out = torch.empty(bs.shape[0], a.shape[1], b.shape[1], dtype=a.dtype, device=a.device)
    capi._check(capi.load().gmm_sm100_forward_vark(
        a.data_ptr(), b.data_ptr(), bs.ctypes.data, bs.shape[0], a.shape[0], a.shape[1], b.shape[1],
        capi.dtype_code(a.dtype), out.data_ptr(), torch.cuda.current_stream(a.device).cuda_stream))
    return out


def hopper_gmm_fwd_host(a, b, batch_sizes, trans_b=False, out=None, device=None):
    """``hopper_gmm_fwd`` on host-resident (pinned) operands, with the transfers pipelined
    against the GEMM; see :mod:`gmm_b200.streaming`."""
    if not _HAS_C:
        raise RuntimeError("gmm_b200._C is not available. Build with `python -m gmm_b200.build`.")
    from gmm_b200.streaming import hopper_gmm_fwd_host as _f
    return _f(a, b, batch_sizes, trans_b=trans_b, out=out, device=device)


def _register_fakes() -> None:
    @torch.library.register_fake("hopper_gmm_fwd::gmm")
    def _hopper_gmm_fwd_fake(a, b, batch_sizes, trans_b):
        num_tokens = a.shape[0]
        n = b.shape[1] if trans_b else b.shape[2]
        return torch.empty(num_tokens, n, dtype=a.dtype, device=a.device)

    def _gmm_swiglu_fake(a, b, batch_sizes, trans_b):
        n = b.shape[1] if trans_b else b.shape[2]
        return torch.empty(a.shape[0], n // 2, dtype=a.dtype, device=a.device)

    try:  # absent only in a stale build; `python -m gmm_b200.build` refreshes it
        torch.library.register_fake("hopper_gmm_fwd::gmm_swiglu")(_gmm_swiglu_fake)
    except RuntimeError:
        warnings.warn("gmm_b200._C predates gmm_swiglu; rebuild with `python -m gmm_b200.build`",
                      RuntimeWarning)


if not load_native():
    warnings.warn("gmm_b200._C not built; run `python -m gmm_b200.build`. "
                  f"No loadable _C.so in {_PKG_DIR}", RuntimeWarning)


__all__ = ["hopper_gmm_fwd"]
