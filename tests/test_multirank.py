"""Multi-process logic of the benchmark harness on CPU (gloo, world size 2): every rank
generates its own shard, the shards reproduce the single-process batch bit for bit, the
max-over-ranks reduction and barriers work, and the CPU reference arm runs under torchrun
with rank 0 alone printing its JSON line."""

import hashlib
import json
import os
import socket
import subprocess
import sys

import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _worker(rank, world, port, queue):
    sys.path.insert(0, ROOT)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import bench
    from flash_hyperconnections_b200 import workloads as W

    dist = bench.Dist()
    dist.init("gloo")
    try:
        cfg = W.CONFIGS[3]
        # a 2-chunk prefix of config 3, split over the ranks like the bench splits a config
        per = W.CHUNK
        a, g = W.generate(cfg, rank * per, per)
        dist.barrier()
        slowest = dist.max(float(rank + 1))
        queue.put((rank, _digest(a.mT.contiguous()), _digest(g), slowest))
    finally:
        dist.close()


def test_shards_match_single_process_and_max_reduction():
    from flash_hyperconnections_b200 import workloads as W

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = W.CONFIGS[3]
    a, g = W.generate(cfg, 0, 2 * W.CHUNK)
    for rank, da, dg, slowest in results:
        sl = slice(rank * W.CHUNK, (rank + 1) * W.CHUNK)
        assert da == _digest(a[sl].mT.contiguous()) and dg == _digest(g[sl])
        assert slowest == 2.0


def test_reference_arm_under_torchrun():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"), "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "0", "--cpu-seconds", "1", "--config", "1"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 2
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0


_MAPS_PROBE = """
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--cpu-seconds", "0.5", "--config", "1"]
runpy.run_path(sys.argv_path, run_name="__main__")
maps = open("/proc/self/maps").read()
mapped = sorted({line.split()[-1] for line in maps.splitlines() if "flash_hyperconnections_b200" in line})
print(json.dumps({"mapped": mapped, "package_imported": "flash_hyperconnections_b200" in sys.modules}))
"""


def test_reference_arm_maps_no_native_library_of_this_package():
    """The reference arm times the reference's own CPU path: its process must not load this
    package's native libraries (``_C.so``, ``libfhx.so``), nor import the package at all."""
    code = _MAPS_PROBE.replace("sys.argv_path", repr(os.path.join(ROOT, "bench.py")))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]
    bench_line, probe = lines[0], lines[-1]
    assert bench_line["impl"] == "reference"
    assert probe["mapped"] == [], probe
    assert probe["package_imported"] is False
