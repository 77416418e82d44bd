"""B200-native (sm_100a) FP8 flash-attention forward.

Drop-in for the module ``ada_cute_fp8_flash_attention`` of
Lemon7-UP/ada_cute_fp8_flash_attention, whose only export is
``flash_attn_fp8_forward(q, k, v)`` (csrc/attention_api.cpp:6-9):

* ``q``, ``k``: ``torch.float8_e4m3fn`` of shape (B, H, S, D), D in {64, 128};
* ``v``: ``torch.float8_e4m3fn`` pre-transposed to (B, H, D, S) (test.py:51-52);
* causal attention with scale 1/sqrt(D) (csrc/flash_attention.cu:524);
* returns fp16 O of shape (B, H, S, D).

The computation runs in the native library ``libfa8.so`` (C ABI,
``include/fa8.h``) through the PyTorch extension ``_fa8_torch``. There is no
CPU or eager-PyTorch fallback: importing this package raises ImportError when
the native extension has not been built (``python
ada_cute_fp8_flash_attention_b200/_build.py``).
"""
from __future__ import annotations

import importlib.util
import sys

from . import _build

__all__ = [
    "flash_attn_fp8_forward",
    "flash_attn_fp8_forward_ex",
    "flash_attn_fp8_varlen_forward",
    "flash_attn_fp8_backward",
    "lse_merge",
    "quantize_e4m3",
    "launch_count",
]


def _load_ext():
    path = _build.ext_path()
    if not path.exists():
        raise ImportError(
            f"native extension {path.name} is not built; run "
            "`python ada_cute_fp8_flash_attention_b200/_build.py` (no CPU fallback exists)")
    import torch  # noqa: F401  (loads libc10 / libtorch for the extension)

    name = f"{__name__}.{_build.EXT_NAME}"
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


_C = _load_ext()


def flash_attn_fp8_forward(q, k, v):
    """Reference-compatible entry point: causal FP8 attention, V in (B,H,D,S), fp16 out."""
    return _C.flash_attn_fp8_forward(q, k, v)


def flash_attn_fp8_forward_ex(q, k, v, causal=True, softmax_scale=None, v_layout="bhds",
                              return_lse=False, out_dtype="fp16", q_offset=0, kv_offset=0,
                              split_keys=-1, out=None, lse=None, descale_q=1.0, descale_k=1.0,
                              descale_v=1.0, sm_budget=0):
    """FP8 attention forward with options.

    Returns ``out`` or ``(out, lse)`` when ``return_lse`` is set. ``lse`` is the
    natural-log log-sum-exp of the scaled scores per query row (fp32, (B,H,S)),
    ``-inf`` for rows with no visible key. ``q_offset``/``kv_offset`` are global
    positions used by the causal mask (context-parallel chunks). ``split_keys``:
    query tiles whose first row sees fewer keys than this use a two-term (hi +
    lo) e4m3 P; -1 = default (1024), 0 = never. ``descale_q/k/v``: dequantisation
    factors of scaled e4m3 inputs (real value = code x factor), each a float
    (per tensor) or a device tensor that broadcasts to (B, H) for Q and to
    (B, H_kv) for K and V (per batch and head). ``sm_budget`` > 0 runs the kernel
    on at most that many SMs (a multiple of 8) of a green-context partition,
    leaving the rest to concurrent work such as NCCL transfers; 0 = whole GPU.
    """
    import torch

    def split(d):
        return (1.0, d) if isinstance(d, torch.Tensor) else (float(d), None)
    (sq, tq), (sk, tk), (sv, tv) = split(descale_q), split(descale_k), split(descale_v)
    res = _C.flash_attn_fp8_forward_ex(q, k, v, causal, softmax_scale, v_layout, return_lse,
                                       out_dtype, q_offset, kv_offset, split_keys, out, lse,
                                       sq, sk, sv, tq, tk, tv, int(sm_budget))
    return (res[0], res[1]) if return_lse else res[0]


def flash_attn_fp8_varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q,
                                  causal=True, softmax_scale=None, v_layout="thd",
                                  return_lse=False, out_dtype="fp16", status=None):
    """FP8 attention over packed variable-length sequences.

    q: (total_q, H, D), k: (total_kv, H_kv, D), v: (total_kv, H_kv, D) ("thd", read
    in place) or (H_kv, D, total_kv) ("hdt"), all e4m3; cu_seqlens_*: int32 prefix
    sums (batch+1) on q's device. Every cu_seqlens_kv entry must be a multiple of 16.
    The offsets are never read on the host (no device synchronisation): the kernel
    refuses a sequence that breaks the rules, leaves it unwritten and ORs a bit into
    ``status`` (optional int32 device tensor): 2 = unaligned K/V start, 4 = offsets
    outside the packed tensors or a sequence longer than ``max_seqlen_q``.
    Returns out (total_q, H, D) or (out, lse (H, total_q)).
    """
    res = _C.flash_attn_fp8_varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_kv,
                                           int(max_seqlen_q), causal, softmax_scale, v_layout,
                                           return_lse, out_dtype, status)
    return (res[0], res[1]) if return_lse else res[0]


def flash_attn_fp8_backward(q, k, v, out, grad_out, lse, causal=True, softmax_scale=None,
                            v_layout="bhds"):
    """Gradients of the FP8 attention with respect to its e4m3 inputs.

    q (B,H,S_q,D), k (B,H_kv,S_kv,D), v (B,H_kv,D,S_kv) for "bhds" or (B,H_kv,S_kv,D)
    for "bhsd", all e4m3; ``out`` (fp16) and ``lse`` (fp32 (B,H,S_q)) as the forward
    returned them (``return_lse=True``); ``grad_out`` fp16 like ``out``. P is
    recomputed exactly in fp32. Returns (dq, dk, dv) in fp32; dk and dv are
    (B, H_kv, S_kv, D) with the query heads of each K/V head summed. The
    reference has no backward; this is the gradient of the same forward.
    """
    dq, dk, dv = _C.flash_attn_fp8_backward(q, k, v, out, grad_out, lse, causal, softmax_scale,
                                            v_layout)
    return dq, dk, dv


def lse_merge(outs, lses):
    """Merge partial outputs of the same rows: returns (fp16 out, fp32 lse)."""
    o, l = _C.lse_merge(list(outs), list(lses))
    return o, l


def quantize_e4m3(x, scale=1.0, transpose_last2=False):
    """fp16/bf16 -> e4m3 (RNE, saturating at +-448), optionally transposing the last 2 dims."""
    return _C.quantize_e4m3(x, scale, transpose_last2)


def launch_count():
    """Kernel launches issued through the C ABI by this process."""
    return _C.launch_count()
