"""Both parts of one Frechet launch: ``fhx_matrix_exp_frechet`` (C ABI), forward-mode AD of
``fh.matrix_exp`` on the kernel, and ``fh.matrix_exp_and_grad`` (forward + backward for a known
upstream gradient).  Checked against the float64 oracle with the reference's per-matrix
criterion (max|d|/(1+max|ref|) <= 1e-3 / 5e-3 float32 fwd / bwd, 5e-2 / 1e-1 half types), and
the derivative part bit for bit against ``fhx_frechet`` (same kernel, same program)."""

import ctypes

import pytest
import torch

import flash_hypercons as fh
from flash_hyperconnections_b200 import _native
from oracle import expm_oracle as O

from .conftest import count_fhx_launches, grouping_passes
from .test_routing import op_names

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
SIZES = [2, 3, 4, 5, 8, 9, 16, 17, 32]


def _kind(dtype):
    return "float32" if dtype == torch.float32 else "half"


def test_pair_entry_point_rejects_bad_arguments_without_gpu():
    lib = _native.load_cabi()
    buf = ctypes.c_void_p(1)
    # n out of range, null exp output, null derivative output, negative stride
    assert lib.fhx_matrix_exp_frechet(buf, 16, 4, 1, 0, buf, 16, 4, 1, 0, buf, 0, buf, 4, 33, 0, None, 0, None) == 1
    assert lib.fhx_matrix_exp_frechet(buf, 16, 4, 1, 0, buf, 16, 4, 1, 0, None, 0, buf, 4, 4, 0, None, 0, None) == 3
    assert lib.fhx_matrix_exp_frechet(buf, 16, 4, 1, 0, buf, 16, 4, 1, 0, buf, 0, None, 4, 4, 0, None, 0, None) == 3
    assert lib.fhx_matrix_exp_frechet(buf, 16, 4, 1, 0, buf, -16, 4, 1, 0, buf, 0, buf, 4, 4, 0, None, 0, None) == 4
    assert lib.fhx_matrix_exp_frechet(None, 0, 0, 0, 0, None, 0, 0, 0, 0, None, 0, None, 0, 4, 0, None, 0, None) == 0
    # a workspace smaller than fhx_workspace_bytes is rejected
    assert lib.fhx_matrix_exp_frechet(buf, 64, 8, 1, 0, buf, 64, 8, 1, 0, buf, 0, buf, 4, 8, 0, buf, 1, None) == 6


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("transposed_view", [False, True])
def test_cabi_pair_outputs(dtype, n, transposed_view):
    lib = _native.load_cabi()
    batch = 45
    a = torch.randn(batch, n, n, device="cuda") * (1.2 / n**0.5)
    a[3] *= 4.0  # a few squarings, exp(A) still in the float16 range
    a = a.to(dtype)
    if transposed_view:
        a = a.mT.contiguous().mT
    e = (torch.randn(batch, n, n, device="cuda") * 0.5).to(dtype)
    stream = torch.cuda.current_stream().cuda_stream
    ref_l = torch.empty_like(e)
    nws = lib.fhx_workspace_bytes(batch, n)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")
    assert lib.fhx_frechet_ws(a.data_ptr(), *a.stride(), 0, e.data_ptr(), *e.stride(), 0, ref_l.data_ptr(), batch, n,
                              DT[dtype], ws.data_ptr(), nws, stream) == 0
    for exp_t in (0, 1):
        y = torch.full_like(e, 7.0)
        l = torch.full_like(e, 7.0)
        assert lib.fhx_matrix_exp_frechet(a.data_ptr(), *a.stride(), 0, e.data_ptr(), *e.stride(), 0, y.data_ptr(),
                                          exp_t, l.data_ptr(), batch, n, DT[dtype], ws.data_ptr(), nws, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(l, ref_l)
        ref_y = O.exp_fp64(a)
        if exp_t:
            ref_y = ref_y.mT
        assert O.per_matrix_error(y, ref_y).max() <= O.tolerance(_kind(dtype), False)
        assert O.per_matrix_error(l, O.frechet_fp64(a, e)).max() <= O.tolerance(_kind(dtype), True)


@pytest.mark.gpu
def test_cabi_pair_outputs_nonfinite_rows():
    lib = _native.load_cabi()
    for n in (4, 8, 32):
        a = torch.randn(6, n, n, device="cuda") * 0.3
        e = torch.randn(6, n, n, device="cuda")
        a[1, 0, 0] = float("nan")
        e[4, 1, 1] = float("inf")
        y, l = torch.empty_like(a), torch.empty_like(a)
        assert lib.fhx_matrix_exp_frechet(a.data_ptr(), *a.stride(), 0, e.data_ptr(), *e.stride(), 0, y.data_ptr(), 0,
                                          l.data_ptr(), 6, n, 0, None, 0, torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        for b in (1, 4):
            assert y[b].isnan().all() and l[b].isnan().all()
        ok = [0, 2, 3, 5]
        assert y[ok].isfinite().all() and l[ok].isfinite().all()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [3, 4, 8, 16, 32])
def test_forward_ad_runs_one_frechet_launch(dtype, n):
    a = (torch.randn(4, n, n, device="cuda") * 0.3).to(dtype)
    e = (torch.randn(4, n, n, device="cuda") * 0.3).to(dtype)
    with torch.autograd.forward_ad.dual_level():
        dual = torch.autograd.forward_ad.make_dual(a, e)
        output, names = op_names(lambda: fh.matrix_exp(dual))
        primal, tangent = torch.autograd.forward_ad.unpack_dual(output)
    assert "flash_hypercons::_matrix_exp_frechet" in names
    assert "flash_hypercons::_matrix_exp" not in names
    assert O.per_matrix_error(primal, O.exp_fp64(a)).max() <= O.tolerance(_kind(dtype), False)
    assert O.per_matrix_error(tangent, O.frechet_fp64(a, e)).max() <= O.tolerance(_kind(dtype), True)
    with torch.autograd.forward_ad.dual_level():
        dual = torch.autograd.forward_ad.make_dual(a, e)
        # one Frechet launch (after the grouping passes for 5 <= n <= 8)
        launches = count_fhx_launches(lambda: fh.matrix_exp(dual))
        assert launches == 1 + grouping_passes(n), launches


@pytest.mark.gpu
def test_forward_ad_with_reverse_graph_stays_native():
    # A primal that needs a reverse-mode graph keeps the reference's native rule.
    a = (torch.randn(2, 8, 8, device="cuda") * 0.3).requires_grad_()
    e = torch.randn(2, 8, 8, device="cuda") * 0.3
    with torch.autograd.forward_ad.dual_level():
        dual = torch.autograd.forward_ad.make_dual(a, e)
        output, names = op_names(lambda: fh.matrix_exp(dual))
        primal, tangent = torch.autograd.forward_ad.unpack_dual(output)
    assert not any(name.startswith("flash_hypercons::") for name in names)
    assert O.per_matrix_error(tangent, O.frechet_fp64(a.detach(), e)).max() <= O.tolerance("float32", True)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", SIZES)
def test_matrix_exp_and_grad_matches_autograd(dtype, n):
    a = torch.randn(33, n, n, device="cuda") * (1.2 / n**0.5)
    a[5] *= 4.0  # a few squarings, exp(A) still in the float16 range
    a = a.to(dtype)
    a = a.mT.contiguous().mT  # a transposed view, as config 3 feeds it
    g = torch.randn_like(a)
    y, grad = fh.matrix_exp_and_grad(a, g)
    x = a.detach().requires_grad_()
    y_ref = fh.matrix_exp(x)
    (grad_ref,) = torch.autograd.grad(y_ref, x, g)
    assert torch.equal(grad, grad_ref)  # same Frechet kernel on the same view a.mT
    assert O.per_matrix_error(y, O.exp_fp64(a)).max() <= O.tolerance(_kind(dtype), False)
    assert O.per_matrix_error(grad, O.frechet_fp64(a.mT, g)).max() <= O.tolerance(_kind(dtype), True)
    launches = count_fhx_launches(lambda: fh.matrix_exp_and_grad(a, g))
    assert launches == 1 + grouping_passes(n), launches


def test_matrix_exp_and_grad_cpu_uses_native():
    a = torch.randn(3, 5, 5, dtype=torch.float64) * 0.3
    g = torch.randn_like(a)
    y, grad = fh.matrix_exp_and_grad(a, g)
    torch.testing.assert_close(y, torch.linalg.matrix_exp(a))
    torch.testing.assert_close(grad, O.frechet_fp64(a.mT, g).to(grad))
