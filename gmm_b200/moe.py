"""A device-resident MoE expert layer built on the grouped GEMM.

``moe_forward(x, router_logits, w_gate_up, w_down, k)`` runs

1. top-k routing (softmax, k largest, optional renormalisation),
2. the permutation of the token rows into expert order (stable counting sort),
3. the fused SwiGLU gate/up grouped GEMM and the down grouped GEMM, both
   reading the per-expert row counts from device memory,
4. the weighted combine back into token order,

as seven kernel launches with no host synchronisation, so the layer can be
captured in a CUDA graph.  The reference only provides step 3's grouped GEMM
(with host ``batch_sizes``); its benchmark leaves routing and gather/scatter
out (reference ``tests/bench_moe_forward.py:216-217``).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from gmm_b200 import capi


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_moe(rc):
    if rc != 0:
        raise RuntimeError(capi.load().gmm_sm100_moe_last_error().decode() or f"status {rc}")


def topk_route(logits: torch.Tensor, k: int, renormalize: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """(ids int32 [T, k], weights fp32 [T, k]) from router logits [T, E]."""
    if not logits.is_cuda or logits.dim() != 2:
        raise ValueError("logits must be a 2D CUDA tensor")
    logits = logits.contiguous()
    T, E = logits.shape
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    _check_moe(capi.load().gmm_sm100_moe_topk(logits.data_ptr(), capi.dtype_code(logits.dtype), T, E, k,
                                              int(renormalize), ids.data_ptr(), w.data_ptr(),
                                              _stream(logits)))
    return ids, w


def permute(x: torch.Tensor, ids: torch.Tensor, num_experts: int):
    """Token rows in expert order.

    Returns ``(x_perm [T*k, dim], batch_sizes int32 [E], dst_pos int32 [T, k],
    src_token int32 [T*k])``; all stay on the device."""
    if ids.dtype != torch.int32 or ids.dim() != 2 or not ids.is_cuda:
        raise ValueError("ids must be a 2D CUDA int32 tensor [T, k]")
    x = x.contiguous()
    T, k = ids.shape
    if x.shape[0] != T:
        raise ValueError("x and ids must have the same number of tokens")
    dev = x.device
    n = T * k
    x_perm = torch.empty(n, x.shape[1], dtype=x.dtype, device=dev)
    bs = torch.empty(num_experts, dtype=torch.int32, device=dev)
    dst_pos = torch.empty(T, k, dtype=torch.int32, device=dev)
    src_token = torch.empty(n, dtype=torch.int32, device=dev)
    lib = capi.load()
    need = int(lib.gmm_sm100_moe_permute_workspace_size(n, num_experts))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    _check_moe(lib.gmm_sm100_moe_permute(x.data_ptr(), T, x.shape[1] * x.element_size(),
                                         ids.contiguous().data_ptr(), k, num_experts, x_perm.data_ptr(),
                                         bs.data_ptr(), dst_pos.data_ptr(), src_token.data_ptr(),
                                         ws.data_ptr(), need, _stream(x)))
    return x_perm, bs, dst_pos, src_token


def unpermute(y: torch.Tensor, dst_pos: torch.Tensor, weights: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[t] = sum_j weights[t, j] * y[dst_pos[t, j]]`` (fp32 accumulation)."""
    T, k = dst_pos.shape
    y = y.contiguous()
    out = torch.empty(T, y.shape[1], dtype=y.dtype, device=y.device)
    wp = weights.contiguous().float().data_ptr() if weights is not None else None
    _check_moe(capi.load().gmm_sm100_moe_unpermute(y.data_ptr(), dst_pos.contiguous().data_ptr(), wp, T, k,
                                                   y.shape[1], capi.dtype_code(y.dtype), out.data_ptr(),
                                                   _stream(y)))
    return out


def grouped_gemm_dev(a: torch.Tensor, b: torch.Tensor, batch_sizes: torch.Tensor,
                     trans_b: bool = False, swiglu: bool = False) -> torch.Tensor:
    """Grouped GEMM with device-resident int32 ``batch_sizes`` (no host sync).

    ``a`` has capacity rows; the first ``sum(batch_sizes)`` are used and only
    those rows of the result are written."""
    if batch_sizes.dtype != torch.int32 or not batch_sizes.is_cuda:
        raise ValueError("batch_sizes must be a CUDA int32 tensor")
    a = a.contiguous()
    b = b.contiguous()
    E = b.shape[0]
    dim_out = b.shape[1] if trans_b else b.shape[2]
    n_out = dim_out // 2 if swiglu else dim_out
    d = torch.empty(a.shape[0], n_out, dtype=a.dtype, device=a.device)
    dt = capi.dtype_code(a.dtype)
    lib = capi.load()
    need = int(lib.gmm_sm100_dev_workspace_size(E, a.shape[0], a.shape[1], dim_out, dt))
    ws = torch.empty(need, dtype=torch.uint8, device=a.device) if need else None
    capi._check(lib.gmm_sm100_forward_dev(a.data_ptr(), b.data_ptr(), batch_sizes.data_ptr(), E, a.shape[0],
                                          a.shape[1], dim_out, dt, int(trans_b), int(swiglu), d.data_ptr(),
                                          ws.data_ptr() if need else None, need, _stream(a)))
    return d


def moe_forward(x: torch.Tensor, router_logits: torch.Tensor, w_gate_up: torch.Tensor,
                w_down: torch.Tensor, k: int, trans_gate_up: bool = False, trans_down: bool = False,
                renormalize: bool = True) -> torch.Tensor:
    """MoE expert layer forward (SwiGLU experts) for tokens ``x [T, dim]``."""
    E = w_gate_up.shape[0]
    ids, w = topk_route(router_logits, k, renormalize)
    xp, bs, dst_pos, _ = permute(x, ids, E)
    h = grouped_gemm_dev(xp, w_gate_up, bs, trans_gate_up, swiglu=True)
    y = grouped_gemm_dev(h, w_down, bs, trans_down)
    return unpermute(y, dst_pos, w)
