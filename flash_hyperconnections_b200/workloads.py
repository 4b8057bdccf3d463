"""Seeded synthetic inputs of the five benchmark configurations.

Every config is generated in fixed chunks of ``CHUNK`` matrices, chunk c drawing from its own
host (CPU) generator seeded with ``seed * 1_000_003 + c``, and then copied to the target
device.  Any contiguous shard that starts on a chunk boundary (every 1/2/4/8-way split of the
configs does) is therefore bit-identical whichever rank, process or device generates it: 1-GPU
and 8-GPU runs, and the CPU baseline, see the same matrices.

1. FP32 [128, 4, 4], entries N(0, 1); upstream gradient all ones.
2. BF16 [65536, 4, 4], entries N(0, 0.1^2) (hyper-connection stream mixing); gradient N(0, 1).
3. FP32 [262144, 8, 8], N(0, 1)/sqrt(8) scaled by 10^U(-3, 1) per matrix, passed as the
   transposed view ``.mT``; gradient N(0, 1).
4. FP16 [1048576, 16, 16], skew-symmetric A = (M - M^T)/2 with M iid N(0, 1/16) (orthogonal
   outputs); gradient N(0, 1).
5. FP32 [1048576, 32, 32], N(0, 1)/sqrt(32) scaled by lognormal(0, 1) per matrix; gradient N(0, 1).
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import torch

CHUNK = 8192


@dataclass(frozen=True)
class Config:
    index: int
    name: str
    batch: int
    n: int
    dtype: torch.dtype
    transposed: bool = False

    @property
    def seed(self) -> int:
        return 9041 + self.index

    @property
    def elem_bytes(self) -> int:
        return torch.tensor([], dtype=self.dtype).element_size()


CONFIGS = {
    1: Config(1, "fp32_b128_n4_randn", 128, 4, torch.float32),
    2: Config(2, "bf16_b65536_n4_hcmix", 65536, 4, torch.bfloat16),
    3: Config(3, "fp32_b262144_n8_multiscale_mT", 262144, 8, torch.float32, transposed=True),
    4: Config(4, "fp16_b1048576_n16_skew", 1048576, 16, torch.float16),
    5: Config(5, "fp32_b1048576_n32_lognormal", 1048576, 32, torch.float32),
}


def _chunk(cfg: Config, c: int, count: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Chunk ``c`` of ``cfg``: ``count`` matrices and gradients, drawn on the host."""
    g = torch.Generator(device="cpu")
    g.manual_seed(cfg.seed * 1_000_003 + c)
    n = cfg.n
    shape = (count, n, n)
    if cfg.index == 1:
        a = torch.randn(shape, generator=g)
        grad = torch.ones(shape)
    elif cfg.index == 2:
        a = torch.randn(shape, generator=g) * 0.1
        grad = torch.randn(shape, generator=g)
    elif cfg.index == 3:
        a = torch.randn(shape, generator=g) / n**0.5
        u = torch.rand((count, 1, 1), generator=g) * 4 - 3
        a = a * torch.pow(10.0, u)
        grad = torch.randn(shape, generator=g)
    elif cfg.index == 4:
        m = torch.randn(shape, generator=g) * 0.25
        a = (m - m.mT) / 2
        grad = torch.randn(shape, generator=g)
    elif cfg.index == 5:
        a = torch.randn(shape, generator=g) / n**0.5
        scale = torch.exp(torch.randn((count, 1, 1), generator=g))
        a = a * scale
        grad = torch.randn(shape, generator=g)
    else:
        raise ValueError(cfg.index)
    return a.to(cfg.dtype), grad.to(cfg.dtype)


def generate(cfg: Config, start: int = 0, count: int | None = None, device="cpu", workers: int | None = None):
    """Matrices [start, start + count) of ``cfg`` and their upstream gradients, on ``device``.

    ``start`` must be a multiple of CHUNK (or 0).  Chunks are drawn on the host in parallel
    (``workers`` threads, each chunk with its own generator, so the result does not depend on
    the thread count) and copied into the output tensors.  For config 3 the returned input is
    the transposed view of a contiguous buffer, as the config prescribes.
    """
    count = cfg.batch - start if count is None else count
    if start % CHUNK:
        raise ValueError("start must be a multiple of CHUNK")
    n = cfg.n
    a = torch.empty((count, n, n), dtype=cfg.dtype, device=device)
    g = torch.empty((count, n, n), dtype=cfg.dtype, device=device)
    jobs = [(start // CHUNK + i, lo, min(CHUNK, count - lo)) for i, lo in enumerate(range(0, count, CHUNK))]

    def fill(job):
        c, lo, take = job
        ca, cg = _chunk(cfg, c, CHUNK if cfg.batch >= CHUNK else cfg.batch)
        a[lo : lo + take].copy_(ca[:take])
        g[lo : lo + take].copy_(cg[:take])

    if workers is None:
        workers = min(16, os.cpu_count() or 1)
    if workers <= 1 or len(jobs) <= 1:
        for job in jobs:
            fill(job)
    else:
        with ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(fill, jobs))
    if cfg.transposed:
        a = a.mT.contiguous().mT  # the stored buffer holds A^T; the view reads as A
    return a, g


def shard(cfg: Config, rank: int, world: int) -> tuple[int, int]:
    """Contiguous equal shard [start, start + count) of rank ``rank`` out of ``world``."""
    if cfg.batch % world:
        raise ValueError(f"batch {cfg.batch} does not split {world} ways")
    count = cfg.batch // world
    return rank * count, count
