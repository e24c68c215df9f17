"""ctypes binding of the C ABI in ``include/gmm_sm100.h`` (``libgmm_sm100.so``).

This is what a non-torch caller binds; the tests use it to drive the kernels
through the C ABI directly.  Pointers are passed as integers (e.g.
``tensor.data_ptr()``), streams as ``torch.cuda.current_stream().cuda_stream``.
"""

from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libgmm_sm100.so")

GMM_DTYPE_F32, GMM_DTYPE_BF16, GMM_DTYPE_F16 = 0, 1, 2

# Every symbol the header declares, with its ctypes signature.
_SIGNATURES = {
    "gmm_sm100_errstr": (ctypes.c_char_p, [ctypes.c_int]),
    "gmm_sm100_last_error": (ctypes.c_char_p, []),
    "gmm_sm100_check_device": (ctypes.c_int, [ctypes.c_int]),
    "gmm_sm100_set_tile_kind": (ctypes.c_int, [ctypes.c_int]),
    "gmm_sm100_workspace_size": (ctypes.c_size_t, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                                   ctypes.c_int]),
    "gmm_sm100_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_void_p]),
    "gmm_sm100_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "gmm_sm100_forward_swiglu": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                                ctypes.c_void_p]),
    "gmm_sm100_forward_vark": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                              ctypes.c_void_p]),
    "gmm_sm100_forward_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.c_void_p]),
    "gmm_sm100_dev_workspace_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                       ctypes.c_int64, ctypes.c_int]),
    "gmm_sm100_moe_topk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p]),
    "gmm_sm100_moe_permute": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.c_void_p]),
    "gmm_sm100_moe_permute_workspace_size": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int]),
    "gmm_sm100_moe_unpermute": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_int64, ctypes.c_int, ctypes.c_int64,
                                               ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "gmm_sm100_moe_last_error": (ctypes.c_char_p, []),
    "gmm_sm100_ep_gather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int64, ctypes.c_void_p]),
    "gmm_sm100_forward_inject_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                        ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_double,
                                                        ctypes.c_void_p]),
    "gmm_sm100_ep_barrier": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_double, ctypes.c_void_p]),
    "gmm_sm100_forward_ep": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "gmm_sm100_ep_workspace_size": (ctypes.c_size_t, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                      ctypes.c_int]),
    "gmm_sm100_plan": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_void_p)]),
    "gmm_sm100_plan_workspace_size": (ctypes.c_size_t, [ctypes.c_void_p]),
    "gmm_sm100_launch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_void_p]),
    "gmm_sm100_plan_free": (None, [ctypes.c_void_p]),
    "gmm_sm100_forward_f32_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_void_p, ctypes.c_int64,
                                                     ctypes.c_int64, ctypes.c_int64,
                                                     ctypes.c_int64, ctypes.c_int,
                                                     ctypes.c_void_p, ctypes.c_void_p]),
}

_lib = None


def load():
    """Load ``libgmm_sm100.so`` (raises ``OSError`` if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} not built; run `python -m gmm_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class GmmError(RuntimeError):
    def __init__(self, status, detail):
        super().__init__(f"{detail} (status {status})")
        self.status = status


def _check(rc):
    if rc != 0:
        lib = load()
        raise GmmError(rc, lib.gmm_sm100_last_error().decode() or lib.gmm_sm100_errstr(rc).decode())


def dtype_code(torch_dtype) -> int:
    import torch
    return {torch.float32: GMM_DTYPE_F32, torch.bfloat16: GMM_DTYPE_BF16,
            torch.float16: GMM_DTYPE_F16}[torch_dtype]


def workspace_size(batch_sizes, num_tokens, dim, dim_out, dtype, trans_b) -> int:
    import numpy as np
    bs = np.ascontiguousarray(np.asarray(batch_sizes, dtype=np.int64))
    return int(load().gmm_sm100_workspace_size(bs.ctypes.data, bs.shape[0], num_tokens, dim, dim_out,
                                               dtype, int(bool(trans_b))))


def forward(a, b, batch_sizes, d, trans_b=False, workspace=None, stream=None):
    """Run ``gmm_sm100_forward`` on torch CUDA tensors through the C ABI (no torch op)."""
    import numpy as np
    import torch
    bs = np.ascontiguousarray(np.asarray(batch_sizes, dtype=np.int64))
    dtype = dtype_code(a.dtype)
    dim = a.shape[1]
    dim_out = b.shape[1] if trans_b else b.shape[2]
    need = workspace_size(bs, a.shape[0], dim, dim_out, dtype, trans_b)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
    s = torch.cuda.current_stream(a.device).cuda_stream if stream is None else stream
    _check(load().gmm_sm100_forward(a.data_ptr(), b.data_ptr(), bs.ctypes.data, bs.shape[0],
                                    a.shape[0], dim, dim_out, dtype, int(bool(trans_b)),
                                    d.data_ptr(), workspace.data_ptr() if need else None, need, s))
    return d


class Plan:
    """``gmm_sm100_plan``: the host half of a grouped GEMM (tile table, kernel
    choice), built once from host batch sizes and launched any number of times
    on operands of its shapes with ``launch`` (``gmm_sm100_launch``)."""

    def __init__(self, batch_sizes, num_tokens, dim, dim_out, dtype, trans_b=False):
        import numpy as np
        bs = np.ascontiguousarray(np.asarray(batch_sizes, dtype=np.int64))
        self._lib = load()
        handle = ctypes.c_void_p()
        _check(self._lib.gmm_sm100_plan(bs.ctypes.data, bs.shape[0], num_tokens, dim, dim_out, dtype,
                                        int(bool(trans_b)), ctypes.byref(handle)))
        self._h = handle.value
        self.workspace_size = int(self._lib.gmm_sm100_plan_workspace_size(self._h))

    def launch(self, a, b, d, workspace=None, stream=None):
        import torch
        need = self.workspace_size
        if need and workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
        s = torch.cuda.current_stream(a.device).cuda_stream if stream is None else stream
        _check(self._lib.gmm_sm100_launch(self._h, a.data_ptr(), b.data_ptr(), d.data_ptr(),
                                          workspace.data_ptr() if need else None, need, s))
        return d

    def close(self):
        if getattr(self, "_h", None):
            self._lib.gmm_sm100_plan_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


TILE_KINDS = {"auto": 0, "128": 1, "256": 2, "swap": 3}


def set_tile_kind(kind: str) -> str:
    """Force a kernel family for 16-bit problems ("auto", "128", "256" or "swap",
    ``gmm_sm100_set_tile_kind``); returns the previous setting."""
    prev = load().gmm_sm100_set_tile_kind(TILE_KINDS[kind])
    if prev < 0:
        _check(prev)
    return {v: k for k, v in TILE_KINDS.items()}[prev]


def device_error(clear=True) -> int:
    v = ctypes.c_int(0)
    _check(load().gmm_sm100_device_error(ctypes.byref(v), int(bool(clear))))
    return v.value


def _i64(values):
    import numpy as np
    return np.ascontiguousarray(np.asarray(values, dtype=np.int64).reshape(-1))


def _ptrs(values):
    return (ctypes.c_void_p * len(values))(*[int(v) for v in values])


def ep_gather(x, src_ptrs, counts, src_rows, num_local_experts, row_bytes, rank_base=0, stream=None):
    """Pull the (expert, segment) row chunks into ``x`` (see ``gmm_sm100_ep_gather``)."""
    import torch
    c, r = _i64(counts), _i64(src_rows)
    s = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    _check(load().gmm_sm100_ep_gather(x.data_ptr(), _ptrs(src_ptrs), c.ctypes.data, r.ctypes.data,
                                      num_local_experts, len(src_ptrs), rank_base, row_bytes, s))


def ep_barrier(flag_ptrs, rank, epoch, device, timeout_s=5.0, stream=None):
    """Cross-rank barrier over peer memory (``gmm_sm100_ep_barrier``)."""
    import torch
    s = torch.cuda.current_stream(device).cuda_stream if stream is None else stream
    _check(load().gmm_sm100_ep_barrier(_ptrs(flag_ptrs), len(flag_ptrs), rank, epoch, timeout_s, s))


def forward_ep(x, b, counts, dst_rows, num_local_experts, out_ptrs, trans_b=False, rank_base=0,
               stream=None):
    """Local grouped GEMM whose epilogue writes each row back to its source rank."""
    import torch
    c, d = _i64(counts), _i64(dst_rows)
    W = len(out_ptrs)
    dtype = dtype_code(x.dtype)
    dim = x.shape[1]
    dim_out = b.shape[1] if trans_b else b.shape[2]
    lib = load()
    need = int(lib.gmm_sm100_ep_workspace_size(c.ctypes.data, num_local_experts, W, x.shape[0], dim,
                                               dim_out, dtype))
    ws = torch.empty(need, dtype=torch.uint8, device=x.device) if need else None
    s = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    _check(lib.gmm_sm100_forward_ep(x.data_ptr(), b.data_ptr(), c.ctypes.data, d.ctypes.data,
                                    num_local_experts, W, rank_base, _ptrs(out_ptrs), x.shape[0], dim, dim_out,
                                    dtype, int(bool(trans_b)), ws.data_ptr() if need else None, need, s))
