"""Seeded synthetic inputs of the five benchmark configurations.

Every config is generated in fixed chunks of ``CHUNK`` matrices, chunk c drawing from its own
generator seeded with ``seed * 1_000_003 + c``.  Any contiguous shard that starts on a chunk
boundary (every 1/2/4/8-way split of the configs does) is therefore bit-identical whichever
rank or process generates it, so 1-GPU and 8-GPU runs see the same matrices.

1. FP32 [128, 4, 4], entries N(0, 1); upstream gradient all ones.
2. BF16 [65536, 4, 4], entries N(0, 0.1^2) (hyper-connection stream mixing); gradient N(0, 1).
3. FP32 [262144, 8, 8], N(0, 1)/sqrt(8) scaled by 10^U(-3, 1) per matrix, passed as the
   transposed view ``.mT``; gradient N(0, 1).
4. FP16 [1048576, 16, 16], skew-symmetric A = (M - M^T)/2 with M iid N(0, 1/16) (orthogonal
   outputs); gradient N(0, 1).
5. FP32 [1048576, 32, 32], N(0, 1)/sqrt(32) scaled by lognormal(0, 1) per matrix; gradient N(0, 1).
"""

from __future__ import annotations

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


def _chunk(cfg: Config, c: int, count: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed * 1_000_003 + c)
    n = cfg.n
    shape = (count, n, n)
    if cfg.index == 1:
        a = torch.randn(shape, generator=g, device=device)
        grad = torch.ones(shape, device=device)
    elif cfg.index == 2:
        a = torch.randn(shape, generator=g, device=device) * 0.1
        grad = torch.randn(shape, generator=g, device=device)
    elif cfg.index == 3:
        a = torch.randn(shape, generator=g, device=device) / n**0.5
        u = torch.rand((count, 1, 1), generator=g, device=device) * 4 - 3
        a = a * torch.pow(10.0, u)
        grad = torch.randn(shape, generator=g, device=device)
    elif cfg.index == 4:
        m = torch.randn(shape, generator=g, device=device) * 0.25
        a = (m - m.mT) / 2
        grad = torch.randn(shape, generator=g, device=device)
    elif cfg.index == 5:
        a = torch.randn(shape, generator=g, device=device) / n**0.5
        scale = torch.exp(torch.randn((count, 1, 1), generator=g, device=device))
        a = a * scale
        grad = torch.randn(shape, generator=g, device=device)
    else:
        raise ValueError(cfg.index)
    return a.to(cfg.dtype), grad.to(cfg.dtype)


def generate(cfg: Config, start: int = 0, count: int | None = None, device="cpu"):
    """Matrices [start, start + count) of ``cfg`` and their upstream gradients.

    ``start`` must be a multiple of CHUNK (or 0).  For config 3 the returned input is the
    transposed view of a contiguous buffer, as the config prescribes.
    """
    count = cfg.batch - start if count is None else count
    if start % CHUNK:
        raise ValueError("start must be a multiple of CHUNK")
    parts_a, parts_g = [], []
    c = start // CHUNK
    remaining = count
    while remaining > 0:
        take = min(CHUNK, remaining)
        a, g = _chunk(cfg, c, CHUNK if cfg.batch >= CHUNK else cfg.batch, device)
        parts_a.append(a[:take])
        parts_g.append(g[:take])
        remaining -= take
        c += 1
    a = torch.cat(parts_a) if len(parts_a) > 1 else parts_a[0]
    g = torch.cat(parts_g) if len(parts_g) > 1 else parts_g[0]
    if cfg.transposed:
        a = a.mT.contiguous().mT  # the stored buffer holds A^T; the view reads as A
    return a, g


def shard(cfg: Config, rank: int, world: int) -> tuple[int, int]:
    """Contiguous equal shard [start, start + count) of rank ``rank`` out of ``world``."""
    if cfg.batch % world:
        raise ValueError(f"batch {cfg.batch} does not split {world} ways")
    count = cfg.batch // world
    return rank * count, count
