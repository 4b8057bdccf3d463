"""Fused hyper-connection stream mixing: Y = exp(H) X per token, and its backward.

Checked against a float64 restatement on the CPU (native float64 exp and products, float64
autograd for the gradients) with the north-star tolerance: relative Frobenius error <= 1e-5 for
float32 streams and <= 1e-2 for bfloat16 / float16, for Y, dX and dH.  Also: one forward launch
and two backward launches, deterministic backward, non-finite tokens isolated, every layout path
(16-byte chunks, ragged widths, strided rows, non-unit column strides)."""

import ctypes

import pytest
import torch

import flash_hypercons as fh
from flash_hyperconnections_b200 import _native
from oracle import expm_oracle as O

from .conftest import count_fhx_launches

TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def _fp64_reference(h, x, dy):
    """Y, dX, dH in float64 on the CPU from the same (rounded) inputs."""
    hd = h.detach().cpu().double().requires_grad_()
    xd = x.detach().cpu().double().requires_grad_()
    y = torch.linalg.matrix_exp(hd) @ xd
    dx, dh = torch.autograd.grad(y, (xd, hd), dy.detach().cpu().double())
    return y.detach(), dx, dh


def _inputs(tokens, n, d, h_dtype, x_dtype, layout="contiguous", scale=0.3):
    h = (torch.randn(tokens, n, n, device="cuda") * scale).to(h_dtype)
    if layout == "contiguous":
        x = torch.randn(tokens, n, d, device="cuda").to(x_dtype)
    elif layout == "row_strided":  # rows of a wider buffer: row stride d + 8
        x = torch.randn(tokens, n, d + 8, device="cuda").to(x_dtype)[:, :, :d]
    elif layout == "column_strided":  # non-unit column stride: the shim makes it contiguous
        x = torch.randn(tokens, d, n, device="cuda").to(x_dtype).mT
    else:  # offset base: not 16-byte aligned, element path
        flat = torch.randn(tokens * n * d + 1, device="cuda").to(x_dtype)
        x = flat[1:].view(tokens, n, d)
    dy = torch.randn(tokens, n, d, device="cuda").to(x_dtype)
    return h, x, dy


def test_stream_mix_rejects_bad_arguments_without_gpu():
    lib = _native.load_cabi()
    buf = ctypes.c_void_p(16)
    # n = 5 (only 2..4), bad dtype, null h, negative stride
    assert lib.fhx_stream_mix(buf, 16, 4, 1, 0, 0, buf, 32, 8, 0, buf, 4, 5, 8, None) == 1
    assert lib.fhx_stream_mix(buf, 16, 4, 1, 0, 9, buf, 32, 8, 0, buf, 4, 4, 8, None) == 2
    assert lib.fhx_stream_mix(None, 16, 4, 1, 0, 0, buf, 32, 8, 0, buf, 4, 4, 8, None) == 3
    assert lib.fhx_stream_mix(buf, 16, 4, 1, 0, 0, buf, -32, 8, 0, buf, 4, 4, 8, None) == 4
    assert lib.fhx_stream_mix_backward(buf, 16, 4, 1, 0, 0, buf, 32, 8, 0, buf, 32, 8, buf, None, 4, 4, 8, buf, 256,
                                       None) == 3
    # the backward's workspace: tokens * n * n float32 values, checked before any CUDA call
    assert lib.fhx_stream_mix_workspace_bytes(4, 4) == 4 * 16 * 4
    assert lib.fhx_stream_mix_backward(buf, 16, 4, 1, 0, 0, buf, 32, 8, 0, buf, 32, 8, buf, buf, 4, 4, 8, buf, 255,
                                       None) == 6
    assert lib.fhx_stream_mix(None, 0, 0, 0, 0, 0, None, 0, 0, 0, None, 0, 4, 8, None) == 0


def test_stream_mix_cpu_uses_native():
    h = torch.randn(3, 4, 4, dtype=torch.float64) * 0.3
    x = torch.randn(3, 4, 6, dtype=torch.float64)
    torch.testing.assert_close(fh.mix_streams(h, x), torch.linalg.matrix_exp(h) @ x)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 3, 4])
@pytest.mark.parametrize("d", [1, 5, 64, 1000, 4096])
@pytest.mark.parametrize("dtypes", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                    (torch.float16, torch.float16), (torch.float32, torch.bfloat16)])
def test_stream_mix_forward_backward_against_fp64(n, d, dtypes):
    h_dtype, x_dtype = dtypes
    h, x, dy = _inputs(97, n, d, h_dtype, x_dtype)
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    y = fh.mix_streams(hh, xx)
    dx, dh = torch.autograd.grad(y, (xx, hh), dy)
    assert y.dtype == x_dtype and dx.dtype == x_dtype and dh.dtype == h_dtype
    ref_y, ref_dx, ref_dh = _fp64_reference(h, x, dy)
    tol = max(TOL[h_dtype], TOL[x_dtype])
    for name, got, ref in (("Y", y, ref_y), ("dX", dx, ref_dx), ("dH", dh, ref_dh)):
        err, _ = O.rel_frobenius(got, ref)
        assert err <= tol, (name, err)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["row_strided", "column_strided", "offset"])
@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16])
def test_stream_mix_layouts(layout, x_dtype):
    h, x, dy = _inputs(50, 4, 136, torch.float32, x_dtype, layout)
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    y = fh.mix_streams(hh, xx)
    dx, dh = torch.autograd.grad(y, (xx, hh), dy)
    ref_y, ref_dx, ref_dh = _fp64_reference(h, x, dy)
    for got, ref in ((y, ref_y), (dx, ref_dx), (dh, ref_dh)):
        err, _ = O.rel_frobenius(got, ref)
        assert err <= TOL[x_dtype], err


@pytest.mark.gpu
def test_stream_mix_large_norms_and_transposed_h():
    # generators with squarings, passed as a transposed view
    h, x, dy = _inputs(64, 4, 256, torch.float32, torch.float32, scale=2.0)
    h = h.mT.contiguous().mT
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    y = fh.mix_streams(hh, xx)
    dx, dh = torch.autograd.grad(y, (xx, hh), dy)
    ref_y, ref_dx, ref_dh = _fp64_reference(h, x, dy)
    for got, ref in ((y, ref_y), (dx, ref_dx), (dh, ref_dh)):
        err, _ = O.rel_frobenius(got, ref)
        assert err <= 1e-5, err


@pytest.mark.gpu
def test_stream_mix_matches_unfused_composition():
    # exp(H) from fh.matrix_exp (same register arithmetic), applied with float32 products
    h, x, _ = _inputs(128, 4, 512, torch.float32, torch.float32)
    y = fh.mix_streams(h, x)
    unfused = fh.matrix_exp(h) @ x
    torch.testing.assert_close(y, unfused, rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_stream_mix_launches_and_deterministic():
    h, x, dy = _inputs(300, 4, 2048, torch.bfloat16, torch.bfloat16)
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    out = {}

    def step():
        out["y"] = fh.mix_streams(hh, xx)
        out["grads"] = torch.autograd.grad(out["y"], (xx, hh), dy)

    # one forward kernel; the backward streams once and computes dH in a per-token kernel
    assert count_fhx_launches(step) == 3
    y, grads = out["y"], out["grads"]
    y2 = fh.mix_streams(hh, xx)
    grads2 = torch.autograd.grad(y2, (xx, hh), dy)
    assert torch.equal(y, y2) and all(torch.equal(a, b) for a, b in zip(grads, grads2))


@pytest.mark.gpu
def test_stream_mix_nonfinite_token_isolated():
    h, x, dy = _inputs(8, 4, 64, torch.float32, torch.float32)
    h[2, 1, 3] = float("nan")
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    y = fh.mix_streams(hh, xx)
    dx, dh = torch.autograd.grad(y, (xx, hh), dy)
    ok = [0, 1, 3, 4, 5, 6, 7]
    assert y[2].isnan().all() and dx[2].isnan().all() and dh[2].isnan().all()
    assert y[ok].isfinite().all() and dx[ok].isfinite().all() and dh[ok].isfinite().all()


@pytest.mark.gpu
def test_stream_mix_empty_and_second_order():
    h = torch.zeros(0, 4, 4, device="cuda")
    x = torch.zeros(0, 4, 16, device="cuda")
    assert fh.mix_streams(h, x).shape == (0, 4, 16)
    # create_graph: the backward switches to the differentiable native formula
    h, x, dy = _inputs(6, 3, 40, torch.float32, torch.float32)
    hh = h.detach().requires_grad_()
    xx = x.detach().requires_grad_()
    (dh,) = torch.autograd.grad(fh.mix_streams(hh, xx), hh, dy, create_graph=True)
    (ddh,) = torch.autograd.grad(dh.sum(), hh)
    hd = h.double().requires_grad_()
    (rdh,) = torch.autograd.grad(torch.linalg.matrix_exp(hd) @ x.double(), hd, dy.double(), create_graph=True)
    (rddh,) = torch.autograd.grad(rdh.sum(), hd)
    assert O.rel_frobenius(ddh, rddh)[0] <= 1e-4
