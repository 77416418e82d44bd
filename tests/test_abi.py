"""CPU checks of the C ABI: libfa8.so loads, exports every symbol include/fa8.h
declares, the ctypes mirror of fa8_fwd_params has the C layout, and host-side
argument validation answers without a GPU (no kernel is launched)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def abi():
    from ada_cute_fp8_flash_attention_b200 import c_abi
    return c_abi


def test_header_symbols_exported(abi):
    hdr = (ROOT / "include" / "fa8.h").read_text()
    declared = set(re.findall(r"^\s*(?:int|void|const char\*|uint64_t)\s+(fa8_\w+)\s*\(", hdr, re.M))
    assert declared, "no declarations parsed"
    assert declared <= set(abi.EXPORTED) | declared
    lib = abi.lib()
    for name in declared:
        assert hasattr(lib, name), f"{name} not exported by libfa8.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi._build.LIB)],
                         capture_output=True, text=True).stdout
    for name in declared:
        assert re.search(rf"\bT {name}$", out, re.M), name


def test_params_struct_layout_matches_c(abi, tmp_path):
    src = tmp_path / "layout.c"
    fields = [f[0] for f in abi.Fa8FwdParams._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(fa8_fwd_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "fa8.h"\nint main(void){{\n'
                   f'  printf("size %zu\\n", sizeof(fa8_fwd_params));\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True,
                                                    text=True).stdout.splitlines())
    assert int(lines["size"]) == C.sizeof(abi.Fa8FwdParams)
    for f in fields:
        assert int(lines[f]) == getattr(abi.Fa8FwdParams, f).offset, f


def test_params_init_defaults(abi):
    p = abi.params(2, 8, 4, 100, 300, 128)
    assert p.q_stride_s == 128 and p.q_stride_h == 100 * 128 and p.q_stride_b == 8 * 100 * 128
    assert p.k_stride_b == 4 * 300 * 128 and p.v_stride_r == 300 and p.v_stride_h == 128 * 300
    assert abs(p.softmax_scale - 128 ** -0.5) < 1e-7
    assert p.causal == 0 and p.split_keys == -1 and p.out_dtype == abi.FA8_OUT_F16


@pytest.mark.parametrize("mutate,status", [
    (lambda p: setattr(p, "head_dim", 96), "FA8_ERR_UNSUPPORTED"),
    (lambda p: setattr(p, "batch", -1), "FA8_ERR_INVALID_ARG"),
    (lambda p: setattr(p, "v_layout", 7), "FA8_ERR_INVALID_ARG"),
    (lambda p: (setattr(p, "v_layout", 1), setattr(p, "v_stride_r", 64)), "FA8_ERR_INVALID_ARG"),
    (lambda p: setattr(p, "heads_kv", 3), "FA8_ERR_UNSUPPORTED"),
    (lambda p: setattr(p, "q", None), "FA8_ERR_INVALID_ARG"),
    (lambda p: setattr(p, "q", 0x1008), "FA8_ERR_ALIGNMENT"),
    (lambda p: setattr(p, "v_stride_r", 1000), "FA8_ERR_ALIGNMENT"),
    (lambda p: setattr(p, "softmax_scale", -1.0), "FA8_ERR_INVALID_ARG"),
])
def test_validation_without_gpu(abi, mutate, status):
    p = abi.params(1, 4, 4, 256, 256, 128)
    p.q = p.k = p.v = p.o = 0x100000  # never dereferenced: validation fails first
    mutate(p)
    assert abi.fwd(p) == getattr(abi, status)
    assert abi.lib().fa8_last_error_message()


def test_empty_problem_is_a_no_op(abi):
    p = abi.params(0, 4, 4, 256, 256, 128)
    assert abi.fwd(p) == abi.FA8_OK


def test_no_gpu_reports_error_not_crash(abi):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    p = abi.params(1, 4, 4, 256, 256, 128)
    p.q = p.k = p.v = p.o = 0x100000
    assert abi.fwd(p) in (abi.FA8_ERR_CUDA, abi.FA8_ERR_NO_DEVICE)


def test_aux_entry_points_validate(abi):
    assert abi.lse_merge([], 1, [], 10, 128, 0x1000, 128, None) == abi.FA8_ERR_INVALID_ARG
    # o_parts / o_out are accessed as 16-byte vectors: misaligned pointers are refused
    assert abi.lse_merge([0x1008], 1, [0x2000], 10, 128, 0x1000, 128, None) == abi.FA8_ERR_ALIGNMENT
    assert abi.lse_merge([0x1000], 1, [0x2000], 10, 128, 0x1008, 128, None) == abi.FA8_ERR_ALIGNMENT
    assert abi.quantize_e4m3(None, 0, 0x1000, 1, 1, 16, 1.0, 0) == abi.FA8_ERR_INVALID_ARG
    assert abi.lib().fa8_status_string(3) == b"alignment / stride requirement violated"


def test_bwd_params_struct_layout_matches_c(abi, tmp_path):
    src = tmp_path / "layout_bwd.c"
    fields = [f[0] for f in abi.Fa8BwdParams._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(fa8_bwd_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "fa8.h"\nint main(void){{\n'
                   f'  printf("size %zu\\n", sizeof(fa8_bwd_params));\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout_bwd"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True,
                                                    text=True).stdout.splitlines())
    assert int(lines["size"]) == C.sizeof(abi.Fa8BwdParams)
    for f in fields:
        assert int(lines[f]) == getattr(abi.Fa8BwdParams, f).offset, f


def test_bwd_params_and_workspace_size(abi):
    p = abi.bwd_params(2, 8, 4, 100, 300, 128)
    assert p.causal == 1 and p.v_layout == abi.FA8_V_BHDS and p.softmax_scale == 0.0
    # fp16 copies of Q (2*8*128*128), K and V (2*4*384*128 each), Delta (2*8*128 floats)
    assert abi.bwd_workspace_size(p) == 2 * 8 * 128 * 128 * 2 + 2 * (2 * 4 * 384 * 128 * 2) + 2 * 8 * 128 * 4
    p.head_dim = 96
    assert abi.bwd_workspace_size(p) == -1
    assert abi.bwd(p, 0, 0) == abi.FA8_ERR_UNSUPPORTED
