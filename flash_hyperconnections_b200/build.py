"""In-tree build of the two native libraries of the package.

* ``libfhx.so`` -- the CUDA kernels behind the C ABI of ``include/fhx.h`` (nvcc, sm_100a only,
  no framework headers).
* ``_C.so`` -- the PyTorch operator registration (``flash_hypercons::_matrix_exp`` /
  ``_frechet``), a thin C++ shim that links ``libfhx.so`` through ``$ORIGIN``.

Both land next to this file so they travel with the source tree.  ``ensure_built()``
rebuilds only when a source is newer than its output.
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys
import sysconfig

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBFHX = PKG / "libfhx.so"
TORCH_EXT = PKG / "_C.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _nvcc() -> str:
    nvcc = CUDA_HOME / "bin" / "nvcc"
    if nvcc.exists():
        return str(nvcc)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _stale(output: pathlib.Path, sources) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(pathlib.Path(s).stat().st_mtime > mtime for s in sources)


def _run(cmd, verbose: bool):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build command failed ({res.returncode}):\n{' '.join(map(str, cmd))}\n{res.stdout}\n{res.stderr}")
    return res


def cuda_sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "fhx.h"]


def build_libfhx(force: bool = False, verbose: bool = False, extra_flags=()) -> pathlib.Path:
    srcs = cuda_sources()
    if not force and not _stale(LIBFHX, srcs):
        return LIBFHX
    tmp = LIBFHX.with_suffix(".so.tmp")
    cmd = [
        _nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{CSRC}", *extra_flags,
        "-o", tmp, *sorted(CSRC.glob("*.cu")),
    ]
    _run(cmd, verbose)
    os.replace(tmp, LIBFHX)
    return LIBFHX


def build_torch_ext(force: bool = False, verbose: bool = False) -> pathlib.Path:
    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "torch_ops.cpp"
    if not force and not _stale(TORCH_EXT, [src, INCLUDE / "fhx.h", LIBFHX]):
        return TORCH_EXT
    torch_inc = pathlib.Path(torch.__file__).parent / "include"
    torch_lib = pathlib.Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_EXT.with_suffix(".so.tmp")
    cmd = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
        f"-I{torch_inc}", f"-I{torch_inc / 'torch' / 'csrc' / 'api' / 'include'}", f"-I{CUDA_HOME / 'include'}",
        f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}",
        src, "-o", tmp,
        f"-L{PKG}", "-lfhx", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
        "-ltorch_python", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
    ]
    del ce  # include paths are derived from the installed torch directly
    _run(cmd, verbose)
    os.replace(tmp, TORCH_EXT)
    return TORCH_EXT


def ensure_built(force: bool = False, verbose: bool = False):
    build_libfhx(force=force, verbose=verbose)
    build_torch_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    ensure_built(force="--force" in sys.argv, verbose=True)
