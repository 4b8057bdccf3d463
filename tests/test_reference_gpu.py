"""The reference package's own CUDA kernels, run on the same GPU as a comparator.

oracle/build_ref.py compiles the reference's csrc/register.cpp and csrc/matrix_exp.cu, as they
are, into oracle/_ref/flash_hypercons_ref.so.  That library registers the same operator names
as this package, so tests/ref_gpu_worker.py runs it in a child process.

* test_parity_with_reference_kernels: exp(A) and L(A^T, G) from this package's operators and
  from the reference's operators on the same seeded inputs (all N from 2 to 32 in steps that
  cover every kernel family, float32/bfloat16/float16, contiguous and transposed views).  Both
  must pass the reference's per-matrix criterion against the float64 oracle, they must agree
  with each other within it, and this package's batch-global relative Frobenius error must not
  exceed the reference kernels' own by more than a small factor.
* test_speed_against_reference_kernels (slow): operator-level forward and Frechet time of both
  implementations on the benchmark configurations, CUDA events, same inputs.  Printed, and
  written as JSON to $FHX_REF_GPU_OUT when set.
"""

import json
import os
import pathlib
import subprocess
import sys
import tempfile

import pytest
import torch

import flash_hypercons as fh  # noqa: F401  (registers this package's operators)
from flash_hyperconnections_b200 import workloads as W
from oracle import expm_oracle as O

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "_ref" / "flash_hypercons_ref.so"
WORKER = pathlib.Path(__file__).resolve().parent / "ref_gpu_worker.py"

needs_ref = pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref/flash_hypercons_ref.so not built")


def _run_worker(*args, timeout=900):
    env = dict(os.environ)
    res = subprocess.run([sys.executable, str(WORKER), *map(str, args)], capture_output=True, text=True,
                         timeout=timeout, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]


def _cases():
    gen = torch.Generator().manual_seed(9041)
    cases = {}
    for n in (2, 3, 4, 7, 8, 13, 16, 24, 32):
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            a = torch.randn((48, n, n), generator=gen) / n**0.5
            # norms from ~0.05 to ~20; float16 stays where exp(A) is representable (< 65504)
            spread = 0.5 if dtype == torch.float16 else 1.0
            a = a * torch.exp(spread * torch.randn((48, 1, 1), generator=gen))
            g = torch.randn((48, n, n), generator=gen)
            cases[f"n{n}_{str(dtype)[6:]}"] = (a.to(dtype), g.to(dtype))
        a = torch.randn((48, n, n), generator=gen) / n**0.5
        cases[f"n{n}_float32_mT"] = (a.mT.contiguous().mT, torch.randn((48, n, n), generator=gen))
    return cases


@needs_ref
def test_parity_with_reference_kernels():
    cases = _cases()
    with tempfile.TemporaryDirectory() as tmp:
        inp, out = pathlib.Path(tmp) / "in.pt", pathlib.Path(tmp) / "out.pt"
        torch.save(cases, inp)
        _run_worker("parity", LIB, inp, out)
        ref_out = torch.load(out)
    for name, (a, g) in cases.items():
        ad, gd = a.cuda(), g.cuda()
        y = torch.ops.flash_hypercons._matrix_exp(ad).cpu()
        grad = torch.ops.flash_hypercons._frechet(ad.mT, gd).cpu()
        ref_y, ref_grad = ref_out[name]
        exact_y, exact_grad = O.exp_fp64(a), O.frechet_fp64(a.mT, g)
        kind = "float32" if a.dtype == torch.float32 else "half"
        for ours, theirs, exact, bwd in ((y, ref_y, exact_y, False), (grad, ref_grad, exact_grad, True)):
            tol = O.tolerance(kind, bwd)
            assert O.per_matrix_error(ours, exact).max() <= tol, name
            assert O.per_matrix_error(theirs, exact).max() <= tol, name
            assert O.per_matrix_error(ours, theirs.double()).max() <= tol, name
            fro_ours, _ = O.rel_frobenius(ours, exact)
            fro_theirs, _ = O.rel_frobenius(theirs, exact)
            floor = 2e-6 if kind == "float32" else 4e-3
            print(f"{name} {'bwd' if bwd else 'fwd'}: rel-Frobenius ours {fro_ours:.2e}, reference kernels {fro_theirs:.2e}")
            assert fro_ours <= 4 * fro_theirs + floor, (name, bwd, fro_ours, fro_theirs)


def _time_ours(cfg, batch, reps):
    a, g = W.generate(cfg, 0, min(batch, cfg.batch), device="cuda")
    expm, frechet = torch.ops.flash_hypercons._matrix_exp, torch.ops.flash_hypercons._frechet
    for _ in range(2):
        frechet(a.mT, g)
        expm(a)
    torch.cuda.synchronize()
    # back-to-back calls between two events: the host enqueues ahead of the GPU, so small batches
    # measure the operators' device time rather than per-call host latency
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    for _ in range(reps):
        expm(a)
    ev[1].record()
    for _ in range(reps):
        frechet(a.mT, g)
    ev[2].record()
    torch.cuda.synchronize()
    fwd = ev[0].elapsed_time(ev[1])
    bwd = ev[1].elapsed_time(ev[2])
    count = a.shape[0]
    del a, g
    torch.cuda.empty_cache()
    return {"count": count, "fwd_ms": fwd / reps, "bwd_ms": bwd / reps}


@needs_ref
@pytest.mark.slow
def test_speed_against_reference_kernels():
    rows = {}
    for index in (2, 3, 4, 5):
        cfg = W.CONFIGS[index]
        with tempfile.TemporaryDirectory() as tmp:
            out = pathlib.Path(tmp) / "t.json"
            reps = 200 if cfg.n <= 8 else 5  # enough calls to amortise the first launch's host latency
            _run_worker("time", LIB, index, cfg.batch, reps, out)
            theirs = json.loads(out.read_text())
        ours = _time_ours(cfg, cfg.batch, reps)
        rows[cfg.name] = {"ours": ours, "reference_kernels": theirs,
                          "speedup_fwd_bwd": (theirs["fwd_ms"] + theirs["bwd_ms"]) / (ours["fwd_ms"] + ours["bwd_ms"])}
        print(f"{cfg.name}: ours fwd {ours['fwd_ms']:.3f} ms + bwd {ours['bwd_ms']:.3f} ms; reference kernels fwd "
              f"{theirs['fwd_ms']:.3f} ms + bwd {theirs['bwd_ms']:.3f} ms; speed-up {rows[cfg.name]['speedup_fwd_bwd']:.2f}x")
    path = os.environ.get("FHX_REF_GPU_OUT")
    if path:
        pathlib.Path(path).write_text(json.dumps(rows, indent=1))
    for name, row in rows.items():
        assert row["ours"]["count"] == row["reference_kernels"]["count"], name
