"""fhx_matrix_exp_noalloc: the exponential for callers that cannot allocate device memory.

Some callers have no device allocator to call (a plugin inside an engine that owns all device
memory and hands it only input and output buffers; a latency-critical path that must not enter
cudaMalloc).  For them the library keeps the grouping workspace of the 5 <= n <= 8 path in a
static device array sized for FHX_NOALLOC_MAX_BATCH matrices.  These tests call it through the
C ABI and compare it with fhx_matrix_exp_ws (same algorithm, caller-allocated workspace) on two
calls in a row -- the second one reuses the array that the first left behind -- with the
reference's per-matrix criterion max|d|/(1+max|ref|) <= 1e-3 (float32) / 5e-2 (half types), and
with the float64 oracle.  This file is collected last, so that a failure here stops a -x run
only after every other test has run.
"""

import ctypes

import pytest
import torch

from flash_hyperconnections_b200 import _native
from oracle import expm_oracle as O

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
MAX_BATCH = 1 << 20  # FHX_NOALLOC_MAX_BATCH in include/fhx.h


def test_noalloc_rejects_batches_beyond_its_scratch_without_gpu():
    lib = _native.load_cabi()
    buf = ctypes.c_void_p(256)
    assert lib.fhx_matrix_exp_noalloc(buf, 64, 8, 1, 0, buf, MAX_BATCH + 1, 8, 0, None) == 7
    assert b"FHX_NOALLOC_MAX_BATCH" in lib.fhx_status_string(7)
    # the usual argument checks come first, and an empty batch is a no-op
    assert lib.fhx_matrix_exp_noalloc(buf, 64, 8, 1, 0, buf, 4, 33, 0, None) == 1
    assert lib.fhx_matrix_exp_noalloc(None, 0, 0, 0, 0, None, 0, 8, 0, None) == 0


def _mixed(batch, n, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(batch, n, n, generator=g) / n**0.5
    top = 1.0 if dtype == torch.float32 else 0.4  # every degree; exp(A) within float16's range
    a = a * torch.pow(10.0, torch.rand(batch, 1, 1, generator=g) * (3 + top) - 3)
    return a.to(dtype).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [5, 8, 4, 16])
def test_noalloc_matches_workspace_entry_point_on_two_calls(n, dtype):
    lib = _native.load_cabi()
    stream = torch.cuda.current_stream().cuda_stream
    kind = "float32" if dtype == torch.float32 else "half"
    # two calls in a row, the second smaller and on other matrices, on a transposed view
    for call, (batch, seed) in enumerate(((3000, 21), (777, 22))):
        a = _mixed(batch, n, dtype, seed)
        if call == 1:
            a = a.mT.contiguous().mT
        nws = lib.fhx_workspace_bytes(batch, n)
        ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")
        ref = torch.empty(batch, n, n, dtype=dtype, device="cuda")
        got = torch.full((batch, n, n), 7.0, dtype=dtype, device="cuda")
        assert lib.fhx_matrix_exp_ws(a.data_ptr(), *a.stride(), 0, ref.data_ptr(), batch, n, DT[dtype], ws.data_ptr(),
                                     nws, stream) == 0
        assert lib.fhx_matrix_exp_noalloc(a.data_ptr(), *a.stride(), 0, got.data_ptr(), batch, n, DT[dtype],
                                          stream) == 0
        torch.cuda.synchronize()
        assert O.per_matrix_error(got, ref).max() <= O.tolerance(kind, False)
        assert O.per_matrix_error(got, O.exp_fp64(a)).max() <= O.tolerance(kind, False)
