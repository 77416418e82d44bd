"""In-tree build of the native pieces (no JIT cache, no pip install).

* ``libfa8.so``      — the C-ABI library (``include/fa8.h``): CUDA kernels for
  sm_100a plus their host launchers, compiled with nvcc.
* ``_fa8_torch*.so`` — the PyTorch extension (``csrc/fa8_torch.cpp``) that
  mirrors the reference module's ``flash_attn_fp8_forward`` and calls the C
  ABI; linked against ``libfa8.so`` with an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree. The
reference built its extension with ``-gencode arch=compute_89,code=sm_89``
(setup.py:19-20); this build targets ``compute_100a`` / ``sm_100a`` only.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libfa8.so"
EXT_NAME = "_fa8_torch"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]

CUDA_SOURCES = ["fa8_api.cu", "fa8_aux.cu", "fa8_bwd.cu"]
CUDA_HEADERS = ["fa8_fwd_kernel.cuh", "fa8_softmax.cuh", "sm100_ptx.cuh"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def ext_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / f"{EXT_NAME}{suffix}"


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / s for s in CUDA_SOURCES + CUDA_HEADERS] + [INCLUDE / "fa8.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", "-Xlinker", "-soname=libfa8.so",
           "-o", str(tmp), *[str(CSRC / s) for s in CUDA_SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    import torch.utils.cpp_extension as ce

    build_lib(force=force, verbose=verbose)
    out = ext_path()
    deps = [CSRC / "fa8_torch.cpp", INCLUDE / "fa8.h", LIB]
    if not force and not _stale(out, deps):
        return out
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    incs = ce.include_paths() + [str(Path(cuda_home) / "include"), str(INCLUDE),
                                 sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths() + [str(PKG)]
    abi = "1" if __import__("torch")._C._GLIBCXX_USE_CXX11_ABI else "0"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in incs], str(CSRC / "fa8_torch.cpp"),
           *[f"-L{p}" for p in libdirs],
           "-lfa8", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-ltorch_python", f"-L{Path(cuda_home) / 'lib64'}", "-lcudart",
           "-Wl,-rpath,$ORIGIN", "-o", str(out) + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    os.replace(str(out) + ".tmp", out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
    print(LIB)
    print(ext_path())
