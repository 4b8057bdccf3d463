"""The C ABI of include/fhx.h: the library loads, exports every declared symbol, rejects bad
arguments before touching the GPU (CPU tests), and computes through plain pointers with any
strides (GPU tests, guard-banded output buffers)."""

import ctypes
import pathlib
import re

import pytest
import torch

from flash_hyperconnections_b200 import _native
from oracle import expm_oracle as O

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "fhx.h"
DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"^\s*(?:int32_t|uint64_t|size_t|const char\*)\s+(fhx_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("fhx_matrix_exp", "fhx_frechet", "fhx_status_string", "fhx_abi_version", "fhx_workspace_bytes",
                     "fhx_matrix_exp_ws", "fhx_frechet_ws"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _native.load_cabi()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.fhx_abi_version() == 106


def test_status_strings():
    lib = _native.load_cabi()
    for code in range(0, 6):
        assert lib.fhx_status_string(code)
    assert b"unknown" in lib.fhx_status_string(99)
    # no CUDA call has failed on this thread: the remembered error is cudaSuccess
    assert lib.fhx_last_cuda_error() == 0
    assert lib.fhx_last_cuda_error_string()


@pytest.mark.parametrize(
    "n,batch,dtype,expected",
    [(1, 4, 0, 1), (33, 4, 0, 1), (4, -1, 0, 1), (4, 4, 7, 2)],
)
def test_argument_errors_without_gpu(n, batch, dtype, expected):
    # Rejected before any CUDA call is made.
    lib = _native.load_cabi()
    buf = ctypes.c_void_p(1)
    assert lib.fhx_matrix_exp(buf, 16, 4, 1, 0, buf, batch, n, dtype, None) == expected
    assert lib.fhx_frechet(buf, 16, 4, 1, 0, buf, 16, 4, 1, 0, buf, batch, n, dtype, None) == expected


def test_null_pointer_and_stride_errors_without_gpu():
    lib = _native.load_cabi()
    buf = ctypes.c_void_p(1)
    assert lib.fhx_matrix_exp(None, 16, 4, 1, 0, buf, 4, 4, 0, None) == 3
    assert lib.fhx_matrix_exp(buf, 16, 4, 1, 0, None, 4, 4, 0, None) == 3
    assert lib.fhx_matrix_exp(buf, 16, -4, 1, 0, buf, 4, 4, 0, None) == 4
    assert lib.fhx_frechet(buf, 16, 4, 1, 0, None, 16, 4, 1, 0, buf, 4, 4, 0, None) == 3
    # An empty batch is a no-op even with null pointers.
    assert lib.fhx_matrix_exp(None, 0, 0, 0, 0, None, 0, 4, 0, None) == 0


def test_workspace_sizes_and_errors_without_gpu():
    lib = _native.load_cabi()
    # 6 bytes per matrix (key + permutation entry) plus the bin tables, for 5 <= n <= 8 only
    assert lib.fhx_workspace_bytes(1000, 8) >= 6000
    assert lib.fhx_workspace_bytes(1000, 8) == lib.fhx_workspace_bytes(1000, 5)
    assert lib.fhx_workspace_bytes(1000, 4) == 0 and lib.fhx_workspace_bytes(1000, 2) == 0
    # one 2-byte key per matrix for 9 <= n <= 16, rounded up to 256 bytes
    assert lib.fhx_workspace_bytes(1000, 9) == 2048 and lib.fhx_workspace_bytes(1000, 16) == 2048
    assert lib.fhx_workspace_bytes(1000, 17) == 0 and lib.fhx_workspace_bytes(1000, 32) == 0
    assert lib.fhx_workspace_bytes(0, 8) == 0
    buf = ctypes.c_void_p(256)
    need = lib.fhx_workspace_bytes(64, 8)
    # too small a workspace is rejected before any CUDA call
    assert lib.fhx_matrix_exp_ws(buf, 64, 8, 1, 0, buf, 64, 8, 0, buf, need - 1, None) == 6
    assert lib.fhx_frechet_ws(buf, 64, 8, 1, 0, buf, 64, 8, 1, 0, buf, 64, 8, 0, None, 0, None) == 6
    assert lib.fhx_frechet_grouped(buf, 64, 8, 1, 0, buf, 64, 8, 1, 0, buf, 64, 8, 0, None, 0, None) == 6
    assert b"workspace" in lib.fhx_status_string(6)


def _call(lib, a, out, e=None, stream=None):
    stream = torch.cuda.current_stream().cuda_stream if stream is None else stream
    n = a.shape[-1]
    if e is None:
        return lib.fhx_matrix_exp(a.data_ptr(), *a.stride(), int(a.is_neg()), out.data_ptr(), a.shape[0], n,
                                  DT[a.dtype], stream)
    return lib.fhx_frechet(a.data_ptr(), *a.stride(), int(a.is_neg()), e.data_ptr(), *e.stride(), int(e.is_neg()),
                           out.data_ptr(), a.shape[0], n, DT[a.dtype], stream)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [2, 3, 4, 5, 8, 12, 16, 17, 31, 32])
@pytest.mark.parametrize("layout", ["contiguous", "transposed", "strided", "expanded", "offset"])
def test_cabi_parity_with_guard_bands(dtype, n, layout):
    lib = _native.load_cabi()
    batch = 37
    base = (torch.randn(batch, n + 3, n + 5, device="cuda") * 0.3).to(dtype)  # views keep their strides
    if layout == "contiguous":
        a = base[:, :n, :n].contiguous()
    elif layout == "transposed":
        a = base[:, :n, :n].contiguous().mT
    elif layout == "strided":
        a = base[:, 1 : n + 1, 2 : n + 2]
    elif layout == "expanded":
        a = base[:1, :n, :n].expand(batch, n, n)
    else:  # contiguous strides, base address one element past an aligned boundary
        flat = torch.empty(batch * n * n + 1, device="cuda", dtype=dtype)
        a = flat[1:].view(batch, n, n)
        a.copy_(base[:, :n, :n])
    e = (torch.randn(batch, n, n, device="cuda") * 0.5).to(dtype)
    guard = 64
    for direction in (None, e):
        buf = torch.full((guard + batch * n * n + guard,), 1234.5, device="cuda", dtype=dtype)
        out = buf[guard : guard + batch * n * n].view(batch, n, n)
        assert _call(lib, a, out, direction) == 0
        torch.cuda.synchronize()
        assert (buf[:guard] == 1234.5).all() and (buf[-guard:] == 1234.5).all()
        ref = O.exp_fp64(a) if direction is None else O.frechet_fp64(a, direction)
        err = O.per_matrix_error(out, ref).max()
        kind = "float32" if dtype == torch.float32 else "half"
        assert err <= O.tolerance(kind, direction is not None), err
