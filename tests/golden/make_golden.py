"""Golden vectors from the reference's own CUDA kernels (run on a GPU box).

TEST INFRASTRUCTURE ONLY.  Loads oracle/_ref/flash_hypercons_ref.so (the reference's
csrc/register.cpp + csrc/matrix_exp.cu compiled from its sources by oracle/build_ref.py), runs
its operators on seeded inputs and writes tests/golden/reference_kernels.npz:

  for each case "n{N}_{dtype}": A, E (the inputs, as float32 values of the dtype-rounded data),
  Y = _matrix_exp(A) and L = _frechet(A, E) from the reference kernels (float32 values of the
  outputs in the case's dtype).

This process must not import flash_hyperconnections_b200, which registers the same operator names.
Usage (on a machine with an NVIDIA GPU):  python tests/golden/make_golden.py
"""

import pathlib

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parents[2]
LIB = ROOT / "oracle" / "_ref" / "flash_hypercons_ref.so"
OUT = pathlib.Path(__file__).resolve().parent / "reference_kernels.npz"
SIZES = (2, 3, 4, 5, 8, 11, 16, 23, 32)
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
PER_CASE = 4


def main():
    torch.ops.load_library(str(LIB))
    expm, frechet = torch.ops.flash_hypercons._matrix_exp, torch.ops.flash_hypercons._frechet
    rng = np.random.default_rng(9041)
    arrays = {}
    for n in SIZES:
        for name, dtype in DTYPES.items():
            a = rng.standard_normal((PER_CASE, n, n)) / np.sqrt(n)
            # per-matrix norms from about 0.02 to 8 (float16: up to 4, so exp stays representable)
            top = 2.0 if name != "float16" else 1.4
            a = a * np.exp(np.linspace(-4.0, top, PER_CASE))[:, None, None]
            e = rng.standard_normal((PER_CASE, n, n))
            at = torch.from_numpy(a).to(dtype).cuda()
            et = torch.from_numpy(e).to(dtype).cuda()
            y = expm(at)
            l = frechet(at, et)
            torch.cuda.synchronize()
            key = f"n{n}_{name}"
            arrays[key + "_A"] = at.float().cpu().numpy()
            arrays[key + "_E"] = et.float().cpu().numpy()
            arrays[key + "_Y"] = y.float().cpu().numpy()
            arrays[key + "_L"] = l.float().cpu().numpy()
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays) // 4} cases)")


if __name__ == "__main__":
    main()
