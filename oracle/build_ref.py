"""Compile the reference's own CUDA operator from its sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The result, ``oracle/_ref/flash_hypercons_ref.so``, registers the
reference's ``flash_hypercons::_matrix_exp`` / ``_frechet`` operators when loaded with
``torch.ops.load_library`` -- in a process of its own, since this package registers the same
operator names.  It serves as a GPU comparator for parity checks and timing; it is never on
the product path.

Recipe: the two translation units ``csrc/register.cpp`` and ``csrc/matrix_exp.cu`` of the
reference are compiled where they lie (read-only) for sm_100a.  The reference's CUTLASS
submodule is not vendored, so the CuTe headers of the flashinfer wheel on this image stand in
(the kernels use CuTe only for ``cute::array`` and shared-memory views).  Nothing is copied
into this repository; outputs go to oracle/_ref/ only (git-ignored).
"""

from __future__ import annotations

import os
import pathlib
import subprocess
import sys
import sysconfig

# The reference checkout: $FHX_REFERENCE_ROOT, else a "reference" directory beside this repository.
REF = pathlib.Path(os.environ.get("FHX_REFERENCE_ROOT", pathlib.Path(__file__).resolve().parents[2] / "reference"))
OUT_DIR = pathlib.Path(__file__).resolve().parent / "_ref"
OUT = OUT_DIR / "flash_hypercons_ref.so"
CUDA_HOME = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _cute_include() -> pathlib.Path:
    import importlib.util

    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        raise RuntimeError("flashinfer (for its CuTe headers) is not installed")
    inc = pathlib.Path(list(spec.submodule_search_locations)[0]) / "data" / "cutlass" / "include"
    if not (inc / "cute" / "tensor.hpp").exists():
        raise RuntimeError(f"CuTe headers not found under {inc}")
    return inc


def available() -> bool:
    return (REF / "csrc" / "matrix_exp.cu").exists()


def build(force: bool = False, verbose: bool = False) -> pathlib.Path | None:
    if not available():
        return OUT if OUT.exists() else None
    srcs = [REF / "csrc" / "register.cpp", REF / "csrc" / "matrix_exp.cu", REF / "csrc" / "MatrixExpSmall.cuh"]
    if OUT.exists() and not force and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in srcs):
        return OUT
    import torch

    OUT_DIR.mkdir(exist_ok=True)
    tinc = pathlib.Path(torch.__file__).parent / "include"
    tlib = pathlib.Path(torch.__file__).parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{tinc}", f"-I{tinc / 'torch' / 'csrc' / 'api' / 'include'}", f"-I{_cute_include()}",
            f"-I{CUDA_HOME / 'include'}", f"-I{sysconfig.get_paths()['include']}"]
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C"]
    obj_cu = OUT_DIR / "matrix_exp.o"
    obj_cpp = OUT_DIR / "register.o"
    cmds = [
        [str(CUDA_HOME / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
         "--expt-relaxed-constexpr", "-std=c++17", "-Xcompiler", "-fPIC", *defs, *incs, "-c",
         str(REF / "csrc" / "matrix_exp.cu"), "-o", str(obj_cu)],
        ["g++", "-O3", "-std=c++17", "-fPIC", *defs, *incs, "-c", str(REF / "csrc" / "register.cpp"), "-o", str(obj_cpp)],
        ["g++", "-shared", str(obj_cpp), str(obj_cu), "-o", str(OUT), f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch",
         "-ltorch_cpu", "-ltorch_cuda", f"-L{CUDA_HOME / 'lib64'}", "-lcudart", f"-Wl,-rpath,{tlib}"],
    ]
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"reference build failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    for o in (obj_cu, obj_cpp):
        o.unlink(missing_ok=True)
    return OUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
