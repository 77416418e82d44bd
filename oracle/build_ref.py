"""Build the reference extension from its own sources, for sm_100a — TEST INFRASTRUCTURE.

Compiles Lemon7-UP/ada_cute_fp8_flash_attention's three translation units
(csrc/attention_api.cpp, csrc/flash_attention.cu, csrc/flash_api.cpp) where
they lie under the reference checkout, with the vendored CUTLASS 3.4 headers
(deps/cutlass/include), into ``oracle/_ref/ada_cute_fp8_flash_attention*.so``.
The reference's own build system (setup.py) is not run: this recipe passes the
compile flags that setup.py:47-66 lists, but targets ``compute_100a/sm_100a``
instead of ``sm_89`` (setup.py:19-20). Its Ada ``mma.sync`` code compiles and
runs on B200 unchanged (legacy tensor-core path).

Do not run the result on a GPU. On B200 it faulted with an illegal memory
access on a repeat call at test.py's shape: for the first query block it
prefetches K/V tile -1 (csrc/flash_attention.cu:260-268), reading 64 rows
before the first (batch, head)'s K and V^T, which faults whenever nothing is
mapped in front of the allocation. It is built only as a record of the reference's code path; nothing in this repository
imports or runs it, and no loader for it is provided. Outputs go to
oracle/_ref/ (git-ignored).

Usage: python oracle/build_ref.py /path/to/reference
   or: FA8_REFERENCE_ROOT=/path/to/reference python oracle/build_ref.py
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULE = "ada_cute_fp8_flash_attention"


def build(ref_root: str, verbose: bool = False) -> Path:
    import torch
    import torch.utils.cpp_extension as ce

    ref = Path(ref_root)
    if not (ref / "csrc" / "flash_attention.cu").exists():
        raise FileNotFoundError(f"reference sources not found under {ref}")
    OUT.mkdir(exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = OUT / f"{MODULE}{suffix}"
    srcs = [ref / "csrc" / "attention_api.cpp", ref / "csrc" / "flash_attention.cu",
            ref / "csrc" / "flash_api.cpp"]
    if target.exists() and all(target.stat().st_mtime > s.stat().st_mtime for s in srcs):
        return target
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    abi = "1" if torch._C._GLIBCXX_USE_CXX11_ABI else "0"
    incs = [ref / "csrc", ref / "include", ref / "deps/cutlass/include",
            ref / "deps/cutlass/tools/utils/include", ref / "deps/cutlass/examples/common",
            *ce.include_paths(), Path(cuda_home) / "include", sysconfig.get_paths()["include"]]
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
    inc_flags = [f"-I{p}" for p in incs]
    objs = []
    for src in srcs:
        obj = OUT / (src.stem + ".o")
        if src.suffix == ".cu":
            cmd = [str(Path(cuda_home) / "bin" / "nvcc"), "-c", str(src), "-o", str(obj),
                   "-O3", "-std=c++17", "--use_fast_math", "-lineinfo",
                   "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                   "-U__CUDA_NO_HALF2_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                   "--expt-relaxed-constexpr", "--expt-extended-lambda",
                   "-gencode", "arch=compute_100a,code=sm_100a",
                   "-Xcompiler", "-fPIC", *defs, *inc_flags]
        else:
            cmd = ["g++", "-c", str(src), "-o", str(obj), "-O3", "-std=c++17", "-fPIC",
                   *defs, *inc_flags]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stderr[-4000:]}")
        objs.append(str(obj))
    libdirs = ce.library_paths()
    cmd = ["g++", "-shared", "-o", str(target) + ".tmp", *objs,
           *[f"-L{p}" for p in libdirs], f"-L{Path(cuda_home) / 'lib64'}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stderr[-4000:]}")
    os.replace(str(target) + ".tmp", target)
    for o in objs:
        os.remove(o)
    return target


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FA8_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: build_ref.py REFERENCE_ROOT (or set FA8_REFERENCE_ROOT)")
    print(build(root, verbose=True))
