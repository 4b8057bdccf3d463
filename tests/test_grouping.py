"""Per-matrix results for every n: degree grouping of the 8 x 8 team kernel (5 <= n <= 8,
workspace entry points) and own degrees elsewhere.

With a workspace the 5 <= n <= 8 batch is grouped by (degree, squarings) before the main kernel
and every matrix runs its own degree; the other sizes always do.  So a matrix's result depends
on that matrix alone: its output bits must not change when its neighbours in the batch change.  Checked through ``fh.matrix_exp`` and
its backward (which use the workspace entry points) on mixed-norm batches, plus the C ABI with
and without a workspace against the float64 oracle (reference criterion per matrix)."""

import pytest
import torch

import flash_hypercons as fh
from flash_hyperconnections_b200 import _native
from oracle import expm_oracle as O

pytestmark = pytest.mark.gpu

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _mixed(batch, n, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(batch, n, n, generator=g) / n**0.5
    # every degree and 0-4 squarings (float32); half types stay where exp(A) fits float16
    top = 1.0 if dtype == torch.float32 else 0.4
    a = a * torch.pow(10.0, torch.rand(batch, 1, 1, generator=g) * (3 + top) - 3)
    return a.to(dtype).cuda()


def _fwd_bwd(a, g):
    x = a.detach().requires_grad_()
    y = fh.matrix_exp(x)
    (grad,) = torch.autograd.grad(y, x, g)
    return y.detach(), grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [3, 5, 8, 12, 16, 24])
def test_result_independent_of_neighbours(n, dtype):
    a = _mixed(1000, n, dtype, 7)
    g = torch.randn(1000, n, n, dtype=torch.float32).to(dtype).cuda()
    y, grad = _fwd_bwd(a, g)
    # the same matrices in another order, and among other neighbours
    perm = torch.randperm(1000)
    y_p, grad_p = _fwd_bwd(a[perm], g[perm])
    assert torch.equal(y_p, y[perm]) and torch.equal(grad_p, grad[perm])
    other = _mixed(1000, n, dtype, 8)
    mixed = torch.cat([other[:500], a[::2], other[500:]])
    gm = torch.cat([g[:500], g[::2], g[500:]])
    y_m, grad_m = _fwd_bwd(mixed, gm)
    assert torch.equal(y_m[500:1000], y[::2]) and torch.equal(grad_m[500:1000], grad[::2])
    kind = "float32" if dtype == torch.float32 else "half"
    assert O.per_matrix_error(y, O.exp_fp64(a)).max() <= O.tolerance(kind, False)
    assert O.per_matrix_error(grad, O.frechet_fp64(a.mT, g)).max() <= O.tolerance(kind, True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("n", [5, 8, 11, 16])
@pytest.mark.parametrize("layout", ["contiguous", "transposed", "strided"])
def test_cabi_workspace_paths(n, dtype, layout):
    lib = _native.load_cabi()
    batch = 300
    base = _mixed(batch, n + 2, dtype, 3)
    if layout == "contiguous":
        a = base[:, :n, :n].contiguous()
    elif layout == "transposed":
        a = base[:, :n, :n].contiguous().mT
    else:
        a = base[:, 1:, 1:][:, :n, :n]
    e = torch.randn(batch, n, n).to(dtype).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    nws = lib.fhx_workspace_bytes(batch, n)
    ws = torch.full((nws,), 0xAB, dtype=torch.uint8, device="cuda")  # stale contents must not matter
    kind = "float32" if dtype == torch.float32 else "half"
    for grouped in (False, True):
        y = torch.empty(batch, n, n, dtype=dtype, device="cuda")
        l = torch.empty_like(y)
        if grouped:
            assert lib.fhx_matrix_exp_ws(a.data_ptr(), *a.stride(), 0, y.data_ptr(), batch, n, DT[dtype],
                                         ws.data_ptr(), nws, stream) == 0
            assert lib.fhx_frechet_ws(a.data_ptr(), *a.stride(), 0, e.data_ptr(), *e.stride(), 0, l.data_ptr(), batch,
                                      n, DT[dtype], ws.data_ptr(), nws, stream) == 0
        else:
            assert lib.fhx_matrix_exp(a.data_ptr(), *a.stride(), 0, y.data_ptr(), batch, n, DT[dtype], stream) == 0
            assert lib.fhx_frechet(a.data_ptr(), *a.stride(), 0, e.data_ptr(), *e.stride(), 0, l.data_ptr(), batch, n,
                                   DT[dtype], stream) == 0
        torch.cuda.synchronize()
        assert O.per_matrix_error(y, O.exp_fp64(a)).max() <= O.tolerance(kind, False)
        assert O.per_matrix_error(l, O.frechet_fp64(a, e)).max() <= O.tolerance(kind, True)


def test_grouped_nonfinite_and_degree_one():
    a = _mixed(64, 8, torch.float32, 11)
    a[3, 2, 2] = float("inf")
    a[10] = 0.0  # degree 1: exp(0) = I
    a[11] *= 1e-9
    y = fh.matrix_exp(a)
    assert y[3].isnan().all()
    ok = torch.ones(64, dtype=torch.bool)
    ok[3] = False
    assert y[ok].isfinite().all()
    assert torch.equal(y[10], torch.eye(8, device="cuda"))
    assert O.per_matrix_error(y[ok], O.exp_fp64(a[ok])).max() <= O.tolerance("float32", False)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [5, 7, 8, 9, 12, 13, 16, 24, 32])
@pytest.mark.parametrize("layout", ["contiguous", "transposed"])
def test_backward_reuses_forward_grouping(n, dtype, layout):
    """The autograd backward takes the forward's grouping (5 <= n <= 8) or keys (9 <= n <= 16;
    n >= 17 recomputes the same (m, s)): no grouping pass runs in the backward, and its gradient
    equals a _frechet call that groups or computes the norms afresh, bit for bit."""
    from .conftest import count_fhx_launches

    a = _mixed(2000, n, dtype, 21)
    if layout == "transposed":
        a = a.contiguous().mT
    g = torch.randn(2000, n, n).to(dtype).cuda()
    x = a.detach().requires_grad_()
    y = fh.matrix_exp(x)
    grads = []
    # every kernel of this package in the backward: the Frechet kernel alone (a fresh grouping
    # would add classify and scatter)
    launches = count_fhx_launches(lambda: grads.append(torch.autograd.grad(y, x, g)[0]))
    assert launches == 1, launches
    fresh = torch.ops.flash_hypercons._frechet(a.mT, g)
    assert torch.equal(grads[0], fresh)
    # a second backward of the same graph (retain_graph) reuses it again
    y2 = fh.matrix_exp(x)
    (g1,) = torch.autograd.grad(y2, x, g, retain_graph=True)
    (g2,) = torch.autograd.grad(y2, x, g)
    assert torch.equal(g1, fresh) and torch.equal(g2, fresh)


@pytest.mark.parametrize("n", [5, 7, 8, 9, 12, 13, 16, 24, 32])
def test_cabi_frechet_grouped(n):
    """fhx_frechet_grouped on A^T with the workspace of fhx_matrix_exp_ws on A equals
    fhx_frechet_ws (which groups afresh) bit for bit."""
    lib = _native.load_cabi()
    batch = 1500
    a = _mixed(batch, n, torch.float32, 5)
    e = torch.randn(batch, n, n).cuda()
    at = a.mT
    stream = torch.cuda.current_stream().cuda_stream
    nws = lib.fhx_workspace_bytes(batch, n)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")
    ws2 = torch.empty_like(ws)
    y = torch.empty_like(a)
    l_reuse = torch.empty_like(a)
    l_fresh = torch.empty_like(a)
    assert lib.fhx_matrix_exp_ws(a.data_ptr(), *a.stride(), 0, y.data_ptr(), batch, n, 0, ws.data_ptr(), nws,
                                 stream) == 0
    assert lib.fhx_frechet_grouped(at.data_ptr(), *at.stride(), 0, e.data_ptr(), *e.stride(), 0, l_reuse.data_ptr(),
                                   batch, n, 0, ws.data_ptr(), nws, stream) == 0
    assert lib.fhx_frechet_ws(at.data_ptr(), *at.stride(), 0, e.data_ptr(), *e.stride(), 0, l_fresh.data_ptr(), batch,
                              n, 0, ws2.data_ptr(), nws, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(l_reuse, l_fresh)
    assert O.per_matrix_error(l_reuse, O.frechet_fp64(at, e)).max() <= O.tolerance("float32", True)


def test_grouping_handoff_only_inside_autograd():
    """Direct operator calls never take a grouping left elsewhere: each _frechet call groups
    afresh (two grouping passes and the main kernel), also right after a _matrix_exp call on the
    same tensor, and an autograd forward whose backward never runs leaves nothing behind."""
    from .conftest import count_fhx_launches, grouping_passes

    n = 8
    a = _mixed(512, n, torch.float32, 31)
    g = torch.randn(512, n, n).cuda()
    ops = torch.ops.flash_hypercons
    assert count_fhx_launches(lambda: ops._matrix_exp(a)) == 1 + grouping_passes(n)
    assert count_fhx_launches(lambda: ops._frechet(a.mT, g)) == 1 + grouping_passes(n)
    x = a.detach().requires_grad_()
    fh.matrix_exp(x)  # graph dropped without a backward
    assert count_fhx_launches(lambda: ops._frechet(a.mT, g)) == 1 + grouping_passes(n)


def test_input_changed_before_backward_raises():
    """The reused grouping belongs to the saved input; autograd refuses a backward after the
    input changed in place, so stale keys are never used."""
    a = _mixed(256, 8, torch.float32, 33)
    g = torch.randn(256, 8, 8).cuda()
    x = a.clone().requires_grad_()
    y = fh.matrix_exp(x)
    with torch.no_grad():
        x.mul_(3.0)
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        torch.autograd.grad(y, x, g)


def test_handoff_with_concurrent_threads():
    """Forward + backward from several Python threads at once (each on its own stream; the
    autograd engine runs all of their backward calls on one worker thread per device): every
    thread's gradient equals the one computed alone, so no grouping or key crosses over."""
    import threading

    cases = []
    for i, n in enumerate((6, 8, 12, 16)):
        a = _mixed(3000, n, torch.float32, 40 + i)
        g = torch.randn(3000, n, n, generator=torch.Generator().manual_seed(50 + i)).cuda()
        cases.append((a, g, _fwd_bwd(a, g)))
    torch.cuda.synchronize()
    results = [None] * len(cases)
    errors = []

    def work(k):
        try:
            a, g, _ = cases[k]
            stream = torch.cuda.Stream()
            outs = []
            with torch.cuda.stream(stream):
                for _ in range(20):
                    outs.append(_fwd_bwd(a, g))
            stream.synchronize()
            results[k] = outs
        except Exception as exc:  # surfaced below
            errors.append(exc)

    threads = [threading.Thread(target=work, args=(k,)) for k in range(len(cases))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for (a, g, (y0, g0)), outs in zip(cases, results):
        for y, grad in outs:
            assert torch.equal(y, y0) and torch.equal(grad, g0)


@pytest.mark.parametrize("n", [6, 12])
@pytest.mark.parametrize("batch", [1, 3, 33])
def test_reuse_tiny_batches(n, batch):
    """Grouping / key reuse on batches smaller than a CTA's teams: the autograd gradient equals a
    fresh _frechet call bit for bit and passes the float64 oracle."""
    a = _mixed(batch, n, torch.float32, 60 + batch)
    g = torch.randn(batch, n, n, generator=torch.Generator().manual_seed(70 + batch)).cuda()
    y, grad = _fwd_bwd(a, g)
    assert torch.equal(grad, torch.ops.flash_hypercons._frechet(a.mT, g))
    assert O.per_matrix_error(y, O.exp_fp64(a)).max() <= O.tolerance("float32", False)
    assert O.per_matrix_error(grad, O.frechet_fp64(a.mT, g)).max() <= O.tolerance("float32", True)
