"""Runs the reference package's own CUDA operators (built from its sources into
oracle/_ref/flash_hypercons_ref.so) in a process of its own.

TEST INFRASTRUCTURE ONLY: the reference library registers the same operator names as this
package, so it cannot share a process with it.  This worker never imports
``flash_hyperconnections_b200``; ``workloads.py`` is loaded by file path (it depends on torch
only) so that the timed inputs are the same seeded matrices the parent times.

Usage:
  python tests/ref_gpu_worker.py parity <lib.so> <inputs.pt> <outputs.pt>
      inputs.pt: {name: (A, G)}; writes {name: (exp(A), L(A^T, G))} computed by the reference ops.
  python tests/ref_gpu_worker.py time <lib.so> <config> <batch> <reps> <outputs.json>
      mean ms of the reference forward op and of its Frechet op on L(A^T, G), CUDA events.
"""

from __future__ import annotations

import importlib.util
import json
import pathlib
import sys

import torch

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _workloads():
    spec = importlib.util.spec_from_file_location("_fhx_workloads", ROOT / "flash_hyperconnections_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve their module through sys.modules
    spec.loader.exec_module(mod)
    return mod


def _ops(lib: str):
    torch.ops.load_library(lib)
    return torch.ops.flash_hypercons._matrix_exp, torch.ops.flash_hypercons._frechet


def parity(lib: str, inp: str, out: str) -> None:
    expm, frechet = _ops(lib)
    cases = torch.load(inp)
    res = {}
    for name, (a, g) in cases.items():
        a, g = a.cuda(), g.cuda()
        res[name] = (expm(a).cpu(), frechet(a.mT, g).cpu())
    torch.cuda.synchronize()
    torch.save(res, out)


def timing(lib: str, config: int, batch: int, reps: int, out: str) -> None:
    expm, frechet = _ops(lib)
    W = _workloads()
    cfg = W.CONFIGS[config]
    a, g = W.generate(cfg, 0, min(batch, cfg.batch), device="cuda")
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
    pathlib.Path(out).write_text(json.dumps({"count": a.shape[0], "fwd_ms": fwd / reps, "bwd_ms": bwd / reps}))


if __name__ == "__main__":
    if sys.argv[1] == "parity":
        parity(*sys.argv[2:5])
    elif sys.argv[1] == "time":
        timing(sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5]), sys.argv[6])
    else:
        raise SystemExit(f"unknown mode {sys.argv[1]}")
