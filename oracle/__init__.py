"""CPU oracle for the grouped-GEMM forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arms may import this package, and only as the checker or as the
timed CPU baseline.  The product path (``gmm_b200``) never imports it and has
no CPU fallback.

Three restatements of the reference's per-expert matmul oracle ``ref_gmm``
(reference ``tests/test_forward.py:8-15``), with the row segmentation of the
reference host entry (reference ``csrc/hopper_gmm_forward.cu:454-471``):

* :func:`gmm_oracle_c`   -- plain C (``gmm_oracle.c``), fp64 accumulation.
* :func:`gmm_oracle_np`  -- numpy BLAS, fp32 accumulation (fast, for large
  sampled checks).
* :func:`ref_gmm_port`   -- the literal torch-CPU form of ``ref_gmm`` in the
  input dtype; this is the reference's own CPU path and is what the CPU
  baseline times.

Parity is pinned: ``tests/test_oracle.py`` checks the C and numpy oracles
against golden outputs of the reference's own ``ref_gmm`` stored in
``tests/golden`` (made by ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "gmm_oracle.c")
_LIB_PATH = os.path.join(_HERE, "libgmm_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile ``gmm_oracle.c`` into ``oracle/libgmm_oracle.so``."""
    if force or not os.path.exists(_LIB_PATH) or \
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(_SRC):
        subprocess.check_call(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared",
                               "-o", _LIB_PATH, _SRC])
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        f = lib.gmm_oracle_f64acc
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                      ctypes.c_void_p]
        _lib = lib
    return _lib


def to_f32(x) -> np.ndarray:
    """Exact widening of a torch/numpy tensor (fp32/bf16/fp16) to numpy fp32."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", torch.float32).contiguous().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _bs_list(batch_sizes):
    return [int(v) for v in (batch_sizes.tolist() if hasattr(batch_sizes, "tolist")
                             else batch_sizes)]


def gmm_oracle_c(a, b, batch_sizes, trans_b: bool = False) -> np.ndarray:
    """fp64-accumulated grouped GEMM (plain C). Returns ``[T, dim_out]`` float64."""
    a32, b32 = to_f32(a), to_f32(b)
    bs = np.ascontiguousarray(np.asarray(_bs_list(batch_sizes), dtype=np.int64))
    T, dim = a32.shape
    E = b32.shape[0]
    dim_out = b32.shape[1] if trans_b else b32.shape[2]
    if bs.shape[0] != E:
        raise ValueError("batch_sizes length must equal the number of experts")
    out = np.empty((T, dim_out), dtype=np.float64)
    rc = _load().gmm_oracle_f64acc(a32.ctypes.data, b32.ctypes.data, bs.ctypes.data, E, T, dim,
                                   dim_out, int(bool(trans_b)), out.ctypes.data)
    if rc == -2:
        raise ValueError(f"Sum of batch_sizes ({int(bs.sum())}) must equal A.size(0) ({T})")
    if rc != 0:
        raise ValueError(f"gmm_oracle_f64acc failed ({rc})")
    return out


def gmm_oracle_np(a, b, batch_sizes, trans_b: bool = False) -> np.ndarray:
    """fp32-accumulated grouped GEMM via numpy BLAS. Returns ``[T, dim_out]`` float32."""
    a32, b32 = to_f32(a), to_f32(b)
    bs = _bs_list(batch_sizes)
    T = a32.shape[0]
    if sum(bs) != T:
        raise ValueError(f"Sum of batch_sizes ({sum(bs)}) must equal A.size(0) ({T})")
    dim_out = b32.shape[1] if trans_b else b32.shape[2]
    out = np.empty((T, dim_out), dtype=np.float32)
    start = 0
    for i, m in enumerate(bs):
        if m:
            rhs = b32[i].T if trans_b else b32[i]
            np.matmul(a32[start:start + m], rhs, out=out[start:start + m])
        start += m
    return out


def swiglu_oracle(a, b, batch_sizes, trans_b: bool = False) -> np.ndarray:
    """silu(gate) * up of the fp64 grouped GEMM, B holding [gate | up] (float64).

    The MoE FFN's activation (SiLU(x) = x / (1 + exp(-x))) applied to the
    reference per-expert matmul; no reference counterpart of its own."""
    acc = gmm_oracle_c(a, b, batch_sizes, trans_b)
    half = acc.shape[1] // 2
    g, u = acc[:, :half], acc[:, half:]
    return g / (1.0 + np.exp(-g)) * u


def vark_oracle(a, b, batch_sizes) -> np.ndarray:
    """D[e] = a[rows_e]^T @ b[rows_e] in float64 ([E, M, N]); zeros for empty experts."""
    a64, b64 = to_f32(a).astype(np.float64), to_f32(b).astype(np.float64)
    bs = _bs_list(batch_sizes)
    out = np.zeros((len(bs), a64.shape[1], b64.shape[1]))
    start = 0
    for e, m in enumerate(bs):
        if m:
            out[e] = a64[start:start + m].T @ b64[start:start + m]
        start += m
    return out


def topk_oracle(logits, k: int, renormalize: bool = True):
    """(ids [T, k], weights [T, k]) of softmax top-k routing, ties to the lower index."""
    x = to_f32(logits).astype(np.float64)
    order = np.argsort(-x, axis=1, kind="stable")[:, :k]
    p = np.exp(x - x.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    w = np.take_along_axis(p, order, axis=1)
    if renormalize:
        w = w / w.sum(axis=1, keepdims=True)
    return order.astype(np.int32), w


def permute_oracle(ids, num_experts: int):
    """Stable expert order of the (token, slot) pairs: (batch_sizes, dst_pos [T, k], src_token)."""
    ids = np.asarray(ids)
    T, k = ids.shape
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")
    dst = np.empty(T * k, dtype=np.int32)
    dst[order] = np.arange(T * k, dtype=np.int32)
    return (np.bincount(flat, minlength=num_experts).astype(np.int32), dst.reshape(T, k),
            (order // k).astype(np.int32))


def unpermute_oracle(y, dst_pos, weights=None) -> np.ndarray:
    """out[t] = sum_j w[t, j] * y[dst_pos[t, j]] in float64."""
    y64 = to_f32(y).astype(np.float64)
    dst = np.asarray(dst_pos)
    w = np.ones(dst.shape) if weights is None else to_f32(weights).astype(np.float64)
    return np.einsum("tk,tkn->tn", w, y64[dst])


def ref_gmm_port(a, b, batch_sizes, trans_b: bool = False):
    """The reference's ``ref_gmm`` (tests/test_forward.py:8-15) on torch CPU tensors.

    Runs in the inputs' own dtype, exactly as the reference's oracle does.
    """
    import torch
    bs = _bs_list(batch_sizes)
    out, start = [], 0
    for i, size in enumerate(bs):
        rhs = b[i].t() if trans_b else b[i]
        out.append(a[start:start + size] @ rhs)
        start += size
    return torch.cat(out)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 (round-to-nearest-even) and return as float32."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def round_to(x: np.ndarray, dtype_name: str) -> np.ndarray:
    """Round an accumulator array to the output dtype ("fp32", "bf16", "fp16"), as float32."""
    x32 = np.asarray(x, dtype=np.float32)
    if dtype_name == "fp32":
        return x32
    if dtype_name == "bf16":
        return round_bf16(x32)
    if dtype_name == "fp16":
        return x32.astype(np.float16).astype(np.float32)
    raise ValueError(dtype_name)


def dtype_name(torch_dtype) -> str:
    import torch
    return {torch.float32: "fp32", torch.bfloat16: "bf16", torch.float16: "fp16"}[torch_dtype]


# Parity tolerances (rtol = atol) per output dtype: bf16 1.6e-2, fp16 2e-3,
# fp32 (computed through TF32 tensor cores) 5e-3.
TOLERANCE = {"bf16": 1.6e-2, "fp16": 2e-3, "fp32": 5e-3}


def allclose_report(got: np.ndarray, want: np.ndarray, tol: float):
    """(ok, n_bad, max_abs_err) under |got - want| <= tol + tol * |want|."""
    g = np.asarray(got, dtype=np.float64)
    w = np.asarray(want, dtype=np.float64)
    err = np.abs(g - w)
    bad = ~(err <= tol + tol * np.abs(w))
    return (not bad.any()), int(bad.sum()), float(err.max() if err.size else 0.0)
