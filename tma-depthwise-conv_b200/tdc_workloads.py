"""Seeded synthetic workloads of the NHWC fp16 depthwise 3x3 conv2d forward,
and the batch sharding used when one job spans several GPUs.

The reference benchmarks on unseeded ``randn`` inputs (``tests/bench.py:49-50``)
and tests on ``torch.manual_seed(0)`` inputs (``tests/test_dwconv.py:25-29``);
no dataset is involved.  The workloads below fix shape, padding and value
distribution; ``make_inputs`` draws x first and then w from one generator
seeded with ``seed``, so every process that asks for the same workload gets
the same bytes.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    N: int
    H: int
    W: int
    C: int
    pad: int
    dist: str  # "normal": x~N(0,1), w~N(0,1/9);  "uniform": x~U(-1,1), w~U(-1/3,1/3)

    @property
    def P(self) -> int:
        return self.H + 2 * self.pad - 2

    @property
    def Q(self) -> int:
        return self.W + 2 * self.pad - 2

    def bytes_per_call(self, n: int | None = None) -> int:
        """Algorithmic HBM bytes of one call: read x once, write y once, read w."""
        n = self.N if n is None else n
        return 2 * n * self.H * self.W * self.C + 2 * n * self.P * self.Q * self.C + 2 * 9 * self.C

    def flops_per_call(self, n: int | None = None) -> int:
        n = self.N if n is None else n
        return 18 * n * self.P * self.Q * self.C


WORKLOADS: dict[str, Workload] = {w.name: w for w in [
    Workload("dw3x3_n2_h16_w16_c64", 2, 16, 16, 64, 1, "normal"),
    Workload("dw3x3_n8_h56_w56_c256", 8, 56, 56, 256, 1, "normal"),
    Workload("dw3x3_n16_h112_w224_c128", 16, 112, 224, 128, 1, "normal"),
    Workload("dw3x3_n32_h224_w336_c256", 32, 224, 336, 256, 1, "normal"),
    Workload("dw3x3_n64_h224_w336_c256", 64, 224, 336, 256, 1, "uniform"),
]}

HEADLINE = "dw3x3_n64_h224_w336_c256"


def make_inputs(wl: Workload, device: str | torch.device = "cpu", seed: int = 0,
                n: int | None = None, n_offset: int = 0):
    """(x [n,H,W,C] fp16, w [3,3,C] fp16) for images [n_offset, n_offset+n) of wl.

    Images are drawn one by one from per-image seeds, so a shard of the batch
    is identical to the same slice of the full batch.
    """
    n = wl.N if n is None else n
    dev = torch.device(device)
    x = torch.empty((n, wl.H, wl.W, wl.C), dtype=torch.float16, device=dev)
    g = torch.Generator(device=dev)
    for i in range(n):
        g.manual_seed(seed * 1_000_003 + n_offset + i + 1)
        if wl.dist == "normal":
            x[i].normal_(0.0, 1.0, generator=g)
        else:
            x[i].uniform_(-1.0, 1.0, generator=g)
    g.manual_seed(seed * 1_000_003)
    w = torch.empty((3, 3, wl.C), dtype=torch.float32, device=dev)
    if wl.dist == "normal":
        w.normal_(0.0, 1.0 / 3.0, generator=g)
    else:
        w.uniform_(-1.0 / 3.0, 1.0 / 3.0, generator=g)
    return x, w.to(torch.float16)


def shard_range(n: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) images of an n-image batch owned by `rank`.

    Shards differ in size by at most one image; ranks beyond n get empty shards.
    """
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError("bad world_size/rank")
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
