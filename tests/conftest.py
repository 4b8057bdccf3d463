import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

HAS_GPU = torch.cuda.is_available() and torch.version.hip is None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "compile: exercises torch.compile")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="requires an NVIDIA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def seed():
    # Same seed as the reference test-suite (tests/conftest.py:13-15 of flash_hypercons).
    torch.manual_seed(9041)


def count_fhx_launches(fn, kernels=None) -> int:
    """Kernels of this package that ``fn()`` launches.  Without ``kernels``: every kernel, from the
    library's own launch counter (``fhx_launch_count``).  With ``kernels``: device kernels whose
    name contains one of them, counted by the CUDA profiler; where the profiler records no device
    activity at all (CUPTI can drop kernel records after earlier profiling sessions in the same
    process), the runtime launch calls recorded on the host side are counted instead, which cannot
    tell the kernels apart: then every launch counts."""
    if kernels is None:
        from flash_hyperconnections_b200 import _native

        lib = _native.load_cabi()
        torch.cuda.synchronize()
        before = lib.fhx_launch_count()
        fn()
        torch.cuda.synchronize()
        return int(lib.fhx_launch_count() - before)

    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    events = prof.key_averages()
    device = [ev for ev in events if str(getattr(ev, "device_type", "")).endswith("CUDA")]
    if device:
        return sum(int(ev.count) for ev in device if any(k in ev.key for k in kernels))
    return sum(int(ev.count) for ev in events if ev.key in ("cudaLaunchKernel", "cudaLaunchKernelExC", "cuLaunchKernel"))


# The main kernels (the grouping passes of 5 <= n <= 8 -- classify, scatter -- excluded).
MAIN_KERNELS = ("expm_team_kernel", "expm_reg_kernel")


def grouping_passes(n: int) -> int:
    """Launches of the degree-grouping passes that precede the main kernel through the operators."""
    return 2 if 5 <= n <= 8 else 0
