"""ctypes binding of the C ABI in ``include/fa8.h`` (``libfa8.so``).

This is the binding a non-torch caller (or a test) uses to reach the kernels
without the PyTorch extension: plain pointers, sizes and integer status
codes. ``Fa8FwdParams`` mirrors ``struct fa8_fwd_params`` field for field.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import _build

FA8_OK = 0
FA8_ERR_INVALID_ARG = 1
FA8_ERR_UNSUPPORTED = 2
FA8_ERR_ALIGNMENT = 3
FA8_ERR_CUDA = 4
FA8_ERR_DRIVER = 5
FA8_ERR_NO_DEVICE = 6
FA8_V_BHDS = 0
FA8_V_BHSD = 1
FA8_OUT_F16 = 0
FA8_OUT_E4M3 = 1

# Every symbol include/fa8.h declares.
EXPORTED = [
    "fa8_fwd_params_init",
    "fa8_fwd",
    "fa8_fwd_workspace_size",
    "fa8_fwd_static_scratch",
    "fa8_static_scratch_bytes",
    "fa8_lse_merge",
    "fa8_quantize_e4m3",
    "fa8_bwd_params_init",
    "fa8_bwd_workspace_size",
    "fa8_bwd",
    "fa8_status_string",
    "fa8_last_error_message",
    "fa8_launch_count",
]


class Fa8FwdParams(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
        ("lse", C.c_void_p), ("status", C.c_void_p),
        ("batch", C.c_int64), ("heads", C.c_int64), ("heads_kv", C.c_int64),
        ("seqlen_q", C.c_int64), ("seqlen_kv", C.c_int64), ("head_dim", C.c_int64),
        ("q_stride_b", C.c_int64), ("q_stride_h", C.c_int64), ("q_stride_s", C.c_int64),
        ("k_stride_b", C.c_int64), ("k_stride_h", C.c_int64), ("k_stride_s", C.c_int64),
        ("v_stride_b", C.c_int64), ("v_stride_h", C.c_int64), ("v_stride_r", C.c_int64),
        ("o_stride_b", C.c_int64), ("o_stride_h", C.c_int64), ("o_stride_s", C.c_int64),
        ("lse_stride_b", C.c_int64), ("lse_stride_h", C.c_int64),
        ("softmax_scale", C.c_float), ("causal", C.c_int32), ("v_layout", C.c_int32),
        ("out_dtype", C.c_int32),
        ("q_offset", C.c_int64), ("kv_offset", C.c_int64),
        ("split_keys", C.c_int32), ("sm_budget", C.c_int32),
        ("descale_q", C.c_float), ("descale_k", C.c_float), ("descale_v", C.c_float),
        ("reserved0", C.c_int32),
        ("cu_seqlens_q", C.c_void_p), ("cu_seqlens_kv", C.c_void_p),
        ("max_seqlen_q", C.c_int64),
        ("wait_timeout_cycles", C.c_int64), ("debug_skip_kv_loads", C.c_int32),
        ("reserved1", C.c_int32),
        ("descale_q_bh", C.c_void_p), ("descale_k_bh", C.c_void_p), ("descale_v_bh", C.c_void_p),
        ("descale_q_stride_b", C.c_int64), ("descale_q_stride_h", C.c_int64),
        ("descale_kv_stride_b", C.c_int64), ("descale_kv_stride_h", C.c_int64),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_int64), ("kv_splits", C.c_int32),
        ("reserved3", C.c_int32),
    ]


class Fa8BwdParams(C.Structure):
    """Mirror of ``struct fa8_bwd_params``."""
    _fields_ = [
        ("batch", C.c_int64), ("heads", C.c_int64), ("heads_kv", C.c_int64),
        ("seqlen_q", C.c_int64), ("seqlen_kv", C.c_int64), ("head_dim", C.c_int64),
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
        ("d_o", C.c_void_p), ("lse", C.c_void_p),
        ("dq", C.c_void_p), ("dk", C.c_void_p), ("dv", C.c_void_p),
        ("causal", C.c_int32), ("softmax_scale", C.c_float), ("v_layout", C.c_int32),
        ("status", C.c_void_p), ("timeout_cycles", C.c_longlong),
    ]


_lib = None


def lib(path: Path | None = None) -> C.CDLL:
    """Load libfa8.so (raises OSError if it has not been built)."""
    global _lib
    if _lib is None or path is not None:
        p = Path(path) if path is not None else _build.LIB
        L = C.CDLL(str(p))
        L.fa8_fwd_params_init.argtypes = [C.POINTER(Fa8FwdParams)] + [C.c_int64] * 6
        L.fa8_fwd_params_init.restype = None
        L.fa8_fwd.argtypes = [C.POINTER(Fa8FwdParams), C.c_void_p]
        L.fa8_fwd.restype = C.c_int
        L.fa8_fwd_workspace_size.argtypes = [C.POINTER(Fa8FwdParams)]
        L.fa8_fwd_workspace_size.restype = C.c_int64
        L.fa8_fwd_static_scratch.argtypes = [C.POINTER(Fa8FwdParams), C.c_void_p]
        L.fa8_fwd_static_scratch.restype = C.c_int
        L.fa8_static_scratch_bytes.argtypes = []
        L.fa8_static_scratch_bytes.restype = C.c_int64
        L.fa8_lse_merge.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.c_int,
                                    C.POINTER(C.c_void_p), C.c_int64, C.c_int64, C.c_void_p,
                                    C.c_int64, C.c_void_p, C.c_void_p]
        L.fa8_lse_merge.restype = C.c_int
        L.fa8_quantize_e4m3.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64,
                                        C.c_int64, C.c_float, C.c_int, C.c_void_p]
        L.fa8_quantize_e4m3.restype = C.c_int
        L.fa8_bwd_params_init.argtypes = [C.POINTER(Fa8BwdParams)] + [C.c_int64] * 6
        L.fa8_bwd_params_init.restype = None
        L.fa8_bwd_workspace_size.argtypes = [C.POINTER(Fa8BwdParams)]
        L.fa8_bwd_workspace_size.restype = C.c_int64
        L.fa8_bwd.argtypes = [C.POINTER(Fa8BwdParams), C.c_void_p, C.c_int64, C.c_void_p]
        L.fa8_bwd.restype = C.c_int
        L.fa8_status_string.argtypes = [C.c_int]
        L.fa8_status_string.restype = C.c_char_p
        L.fa8_last_error_message.argtypes = []
        L.fa8_last_error_message.restype = C.c_char_p
        L.fa8_launch_count.argtypes = []
        L.fa8_launch_count.restype = C.c_uint64
        if path is not None:
            return L
        _lib = L
    return _lib


def params(batch, heads, heads_kv, seqlen_q, seqlen_kv, head_dim) -> Fa8FwdParams:
    p = Fa8FwdParams()
    lib().fa8_fwd_params_init(C.byref(p), batch, heads, heads_kv, seqlen_q, seqlen_kv, head_dim)
    return p


def check(status: int) -> None:
    if status != FA8_OK:
        L = lib()
        raise RuntimeError(f"fa8 status {status}: {L.fa8_status_string(status).decode()}: "
                           f"{L.fa8_last_error_message().decode()}")


def fwd(p: Fa8FwdParams, stream: int = 0) -> int:
    return lib().fa8_fwd(C.byref(p), C.c_void_p(stream))


def fwd_static_scratch(p: Fa8FwdParams, stream: int = 0) -> int:
    """fa8_fwd for callers that cannot allocate: split-KV scratch from the library's fixed array."""
    return lib().fa8_fwd_static_scratch(C.byref(p), C.c_void_p(stream))


def workspace_size(p: Fa8FwdParams) -> int:
    """Split-KV workspace bytes fa8_fwd would use for these parameters (0: no split)."""
    return int(lib().fa8_fwd_workspace_size(C.byref(p)))


def lse_merge(o_ptrs, o_is_f16, lse_ptrs, rows, head_dim, o_out, o_out_stride, lse_out,
              stream: int = 0) -> int:
    n = len(o_ptrs)
    oa = (C.c_void_p * n)(*o_ptrs)
    la = (C.c_void_p * n)(*lse_ptrs)
    return lib().fa8_lse_merge(n, oa, int(o_is_f16), la, rows, head_dim, o_out, o_out_stride,
                               lse_out, C.c_void_p(stream))


def quantize_e4m3(x_ptr, in_dtype, y_ptr, batch, rows, cols, scale, transpose,
                  stream: int = 0) -> int:
    return lib().fa8_quantize_e4m3(x_ptr, in_dtype, y_ptr, batch, rows, cols, scale,
                                   int(transpose), C.c_void_p(stream))


def bwd_params(batch, heads, heads_kv, seqlen_q, seqlen_kv, head_dim) -> Fa8BwdParams:
    p = Fa8BwdParams()
    lib().fa8_bwd_params_init(C.byref(p), batch, heads, heads_kv, seqlen_q, seqlen_kv, head_dim)
    return p


def bwd_workspace_size(p: Fa8BwdParams) -> int:
    """Device workspace bytes fa8_bwd needs for these parameters (-1: invalid)."""
    return int(lib().fa8_bwd_workspace_size(C.byref(p)))


def bwd(p: Fa8BwdParams, workspace: int, workspace_bytes: int, stream: int = 0) -> int:
    return lib().fa8_bwd(C.byref(p), C.c_void_p(workspace), workspace_bytes, C.c_void_p(stream))
